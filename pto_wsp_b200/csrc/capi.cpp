// extern "C" surface of the cuda_sm100a target (declared in include/ptowsp_cuda.h).
#include <cuda_runtime_api.h>

#include <cstring>

#include "runtime.hpp"

using ptowsp::Error;

struct ptowsp_program {
    std::unique_ptr<ptowsp::Program> p;
};

namespace {

template <class F>
auto guarded(ptowsp_program* h, F&& f, decltype(f()) fail) -> decltype(f()) {
    try {
        auto r = f();
        if (h && h->p) h->p->status = PTOWSP_OK;
        return r;
    } catch (const Error& e) {
        ptowsp::set_error(e.what());
        if (h && h->p) h->p->status = e.code;
    } catch (const std::exception& e) {
        ptowsp::set_error(e.what());
        if (h && h->p) h->p->status = PTOWSP_ERR_PLAN;
    } catch (...) {
        ptowsp::set_error("unknown error");
        if (h && h->p) h->p->status = PTOWSP_ERR_PLAN;
    }
    return fail;
}

}  // namespace

extern "C" {

int ptowsp_cuda_compile(const char* plan_json, size_t plan_len, int device, ptowsp_program** out) {
    if (!plan_json || !out) {
        ptowsp::set_error("ptowsp_cuda_compile: null argument");
        return PTOWSP_ERR_ARG;
    }
    *out = nullptr;
    try {
        auto prog = ptowsp::compile_program(plan_json, plan_len, device);
        *out = new ptowsp_program{std::move(prog)};
        ptowsp::set_error("");
        return PTOWSP_OK;
    } catch (const Error& e) {
        ptowsp::set_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        ptowsp::set_error(e.what());
        return PTOWSP_ERR_PLAN;
    }
}

uint64_t ptowsp_cuda_main(ptowsp_program* prog, RuntimeContext* ctx, CSPTContext* cspt) {
    (void)cspt;  // CSPT timing is not used on this path (the reference passes nullptr, pto_codegen.cpp:3565)
    if (!prog || !prog->p) {
        ptowsp::set_error("ptowsp_cuda_main: null program");
        return 0;
    }
    return guarded(prog, [&] { return ptowsp::run_program(*prog->p, ctx); }, uint64_t{0});
}

uint64_t ptowsp_cuda_run_task(ptowsp_program* prog, const char* kernel_name, const KernelTaskDesc* task) {
    if (!prog || !prog->p || !kernel_name) {
        ptowsp::set_error("ptowsp_cuda_run_task: null argument");
        return 0;
    }
    return guarded(prog, [&] { return ptowsp::run_single_task(*prog->p, kernel_name, task); }, uint64_t{0});
}

int ptowsp_cuda_status(const ptowsp_program* prog) { return (prog && prog->p) ? prog->p->status : PTOWSP_ERR_ARG; }

const char* ptowsp_cuda_last_error(void) { return ptowsp::last_error(); }

int ptowsp_cuda_set_stream(ptowsp_program* prog, void* cuda_stream) {
    if (!prog || !prog->p) return PTOWSP_ERR_ARG;
    prog->p->stream = static_cast<cudaStream_t>(cuda_stream);  // nullptr: the CUDA default stream
    prog->p->stream_set = true;
    return PTOWSP_OK;
}

int ptowsp_cuda_set_option(ptowsp_program* prog, const char* key, int64_t value) {
    if (!prog || !prog->p || !key) return PTOWSP_ERR_ARG;
    auto& p = *prog->p;
    if (!std::strcmp(key, "pipeline_chunks")) p.opt_chunks = value < 1 ? 1 : value;
    else if (!std::strcmp(key, "stage_scratch_mb")) {
        // 1 MiB .. 1 TiB: the byte count (value << 20) stays far inside int64.  A batch keeps the task groups it
        // was planned with, so a changed budget drops the cached task tables (the next run plans again).
        const int64_t mb = value < 1 ? 1 : (value > (int64_t{1} << 20) ? (int64_t{1} << 20) : value);
        if (mb != p.opt_stage_scratch_mb) p.cached.reset();
        p.opt_stage_scratch_mb = mb;
    } else if (!std::strcmp(key, "fused_attention")) {
        p.opt_fused_attention = value != 0;
    } else if (!std::strcmp(key, "csp_device")) {
        // a cached device-process program has no wave records on the device (and waves none for processes)
        if ((value != 0) != (p.opt_csp_device != 0)) p.cached.reset();
        p.opt_csp_device = value != 0;
    } else if (!std::strcmp(key, "decode_chunk")) {
        // 0 (automatic) or a token count, taken as a multiple of 16 inside 512 .. 1536 by the launch
        p.opt_decode_chunk = value < 0 ? 0 : (value > 65536 ? 65536 : value);
    } else if (!std::strcmp(key, "kernel_events")) {
        p.opt_kernel_events = value != 0;
        guarded(prog, [&] { ptowsp::reset_kernel_times(p); return 0; }, 0);
    }
    else if (!std::strcmp(key, "cache_plans")) {
        p.opt_cache = value != 0;
        if (!p.opt_cache) p.cached.reset();
    } else if (!std::strcmp(key, "sync")) p.opt_sync = value != 0;
    else if (!std::strcmp(key, "dry_run")) p.opt_dry = value != 0;
    else {
        ptowsp::set_error(std::string("unknown option ") + key);
        return PTOWSP_ERR_ARG;
    }
    return PTOWSP_OK;
}

int ptowsp_cuda_last_timing(const ptowsp_program* prog, ptowsp_timing* out) {
    if (!prog || !prog->p || !out) return PTOWSP_ERR_ARG;
    *out = prog->p->timing;
    return PTOWSP_OK;
}

const char* ptowsp_cuda_kernel_times(ptowsp_program* prog) {
    if (!prog || !prog->p) return "{}";
    prog->p->kernel_times_json = guarded(prog, [&] { return ptowsp::kernel_times(*prog->p); }, std::string("{}"));
    return prog->p->kernel_times_json.c_str();
}

const char* ptowsp_cuda_describe(ptowsp_program* prog) {
    if (!prog || !prog->p) return "{}";
    prog->p->describe_json = ptowsp::describe_program(*prog->p);
    return prog->p->describe_json.c_str();
}

void ptowsp_cuda_destroy(ptowsp_program* prog) { delete prog; }

int ptowsp_cuda_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                      const int32_t* page_table, const int32_t* kv_len, void* out, int num_requests,
                                      int num_kv_heads, int group, int head_dim, int page_size, int max_pages,
                                      int64_t num_pages, void* stream) {
    const char* msg = "";
    const int rc = ptowsp::dev::paged_decode_noalloc(q, k_cache, v_cache, page_table, kv_len, out, num_requests,
                                                     num_kv_heads, group, head_dim, page_size, max_pages, num_pages,
                                                     static_cast<cudaStream_t>(stream), &msg);
    ptowsp::set_error(msg);
    return rc;
}

size_t ptowsp_cuda_noalloc_scratch_bytes(int num_requests, int num_kv_heads, int group, int max_pages, int page_size) {
    if (num_requests <= 0 && num_kv_heads <= 0) return ptowsp::dev::noalloc_scratch_capacity();
    return ptowsp::dev::noalloc_bytes_needed(num_requests, num_kv_heads, group, max_pages, page_size);
}

int ptowsp_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // extern "C"
