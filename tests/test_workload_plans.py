"""The plan builders equal what the reference frontend produces (build container only)."""

import pytest

from conftest import import_reference
from pto_wsp_b200 import workloads as W
from pto_wsp_b200.plan import module_to_plan


def _ref_plan(builder, *args, name=None, **kw):
    import_reference()
    from pto_wsp.ir_bridge import workload_to_codegen_ir

    import _frontend_workloads as F

    wl, _ = getattr(F, builder)(*args, **kw)
    return module_to_plan(workload_to_codegen_ir(wl, module_name=name).module)


@pytest.mark.parametrize("args", [(2, 3), (4, 64)])
def test_rmsnorm_plan_matches_frontend(args):
    assert W.rmsnorm_plan(*args) == _ref_plan("rmsnorm", *args, name="rmsnorm")


@pytest.mark.parametrize("args", [(2, 3), (32, 2048)])
def test_softmax_plan_matches_frontend(args):
    assert W.softmax_plan(*args) == _ref_plan("softmax", *args, name="softmax")


@pytest.mark.parametrize("acc", [False, True])
def test_bgemm_plan_matches_frontend(acc):
    assert W.bgemm_plan(2, 256, 384, 512, accumulate=acc) == _ref_plan("bgemm", 2, 256, 384, 512, accumulate=acc,
                                                                        name="bgemm")


def test_decode_plan_matches_frontend():
    assert W.decode_plan(5, 8, 4, 128, 300, 64) == _ref_plan("decode", 5, 8, 4, 128, 300, 64, name="paged_decode")


def test_indexer_plan_matches_frontend():
    assert W.indexer_plan(2, 8, 64, 128, 1024, 64) == _ref_plan("indexer", 2, 8, 64, 128, 1024, 64,
                                                                name="lightning_indexer")
