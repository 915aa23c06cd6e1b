"""CSP pipeline plans for the device-process tests: the reference's captured CSP cases, and a pipeline whose two
processes write one tile in an order the channels do not fix (so it must run as dependency waves)."""

import copy

from golden_cases import load_cases

CASES = load_cases()
CSP_NAMES = [c["name"] for c in CASES if c["plan"]["body"].get("kind") == "pipeline"]


def racy_case() -> dict:
    """The reference's producer / consumer pipeline (test_codegen_cspt_pipeline, first case) with a 4-deep channel
    and the producer storing every tile into tensor 2's tile 0, which the consumer also writes after its first
    receive: the producer runs ahead by up to four tokens, so its later stores and the consumer's first one race."""
    case = copy.deepcopy(next(c for c in CASES if c["name"] == "reftest:test_codegen_cspt_pipeline.py#0"))
    body = case["plan"]["body"]
    body["channels"][0]["capacity"] = 4
    task = body["processes"][0]["body"]["body"]["value"]
    task["tensor_args"][1]["tensor"] = 2
    task["tensor_args"][1]["index"] = [{"const": 0}]
    case["name"] = "racy_pipeline"
    return case
