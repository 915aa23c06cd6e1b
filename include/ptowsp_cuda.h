/*
 * ptowsp_cuda.h -- C ABI of the PTO-WSP cuda_sm100a execution target.
 *
 * The reference builds, per workload, a CPU-sim shared library whose entry
 * point is `uint64_t <module>_main(RuntimeContext*, CSPTContext*)` and loads it
 * with dlopen/dlsym (reference: src/python/pto_codegen.cpp:3510-3576).  This
 * library is the CUDA replacement: a workload *plan* (the reference ir::Module
 * serialised as JSON, format "ptowsp-plan/1") is compiled once into a program
 * handle, and each run walks the task loop on the host, builds a device task
 * table and launches sm_100a kernels.  No torch types cross this boundary:
 * plain pointers, sizes and the reference's own callback structs.
 *
 * Threading: a program handle is used by one thread at a time (the reference
 * makes one call per execute(), program.py:678-681).  Errors are reported
 * through return codes plus ptowsp_cuda_last_error() -- the side channel the
 * reference entry ABI does not have.
 */
#ifndef PTOWSP_CUDA_H
#define PTOWSP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PTOWSP_API __attribute__((visibility("default")))
#else
#define PTOWSP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------- */
/* Reference ABI structs, same field order and types as the reference headers */
/* ------------------------------------------------------------------------- */

/* Per-task descriptor (reference: include/pto/wsp/codegen/abi/kernel_abi.hpp:21-41). */
struct KernelTaskDesc {
    const uint64_t* args;        /* axis args, (valid_row, valid_col) per tensor param, scalars */
    uint32_t num_args;
    uint32_t num_axis_args;
    void* const* tensor_ptrs;    /* tile base pointers (device memory for this target) */
    const uint64_t* tensor_strides; /* [s3, s4] per tensor param, in elements */
    uint32_t num_tensors;
    uint32_t kernel_id;
    uint32_t task_id;
};

/* Reference: kernel_abi.hpp:47-62. */
struct TimingConfig {
    uint64_t loop_overhead;
    uint64_t dispatch_overhead;
    uint64_t channel_latency;
};

struct CSPTContext {
    void* ctx;
    void (*advance_cycles)(void* ctx, uint64_t cycles);
    uint64_t (*get_time)(void* ctx);
    const struct TimingConfig* timing;
};

/* Reference: kernel_abi.hpp:70. */
typedef uint64_t (*KernelFn)(const struct KernelTaskDesc* task, struct CSPTContext* cspt);

/* Run-time bindings of one execute() (reference: include/pto/wsp/codegen/abi/workload_abi.hpp:17-41).
 * get_tensor_ptr may return host memory (staged to HBM around the run) or
 * device memory (used in place); the runtime asks the driver which. */
struct RuntimeContext {
    int64_t (*get_axis_size)(void* ctx, const char* name);
    uint64_t (*get_symbol_u64)(void* ctx, uint64_t symbol_id);
    void* (*get_symbol_ptr)(void* ctx, uint64_t symbol_id);
    uint64_t (*get_slot_u64)(void* ctx, uint32_t slot);
    void (*set_slot_u64)(void* ctx, uint32_t slot, uint64_t value);
    void* (*get_tensor_ptr)(void* ctx, uint32_t tensor_id);
    uint64_t (*get_tensor_stride)(void* ctx, uint32_t tensor_id, uint32_t dim);
    KernelFn (*get_kernel)(void* ctx, uint32_t kernel_id);
    void* ctx;
};

/* Reference: workload_abi.hpp:71. */
typedef uint64_t (*WorkloadFn)(struct RuntimeContext* ctx, struct CSPTContext* cspt);

/* ------------------------------------------------------------------------- */
/* cuda_sm100a target                                                          */
/* ------------------------------------------------------------------------- */

typedef struct ptowsp_program ptowsp_program;

enum ptowsp_status {
    PTOWSP_OK = 0,
    PTOWSP_ERR_PLAN = 1,          /* malformed plan / type error (reference: CompileError) */
    PTOWSP_ERR_UNSUPPORTED = 2,   /* op, node or kernel body the GPU target cannot run */
    PTOWSP_ERR_CUDA = 3,          /* CUDA runtime error */
    PTOWSP_ERR_ARG = 4,           /* bad argument (null pointer, missing tensor, ...) */
    PTOWSP_ERR_DEVICE = 5,        /* a kernel reported an error status (bounds, timeout) */
    PTOWSP_ERR_LIMIT = 6          /* a size beyond a documented limit */
};

/* Compile a plan into a program for CUDA device `device`.
 * Replaces compile_codegen(module, CompileOptions{target}) for target
 * "cuda_sm100a" (reference: src/python/pto_codegen.cpp:3352-3434): type checks,
 * matches every kernel to a CUDA implementation, and fails with
 * PTOWSP_ERR_UNSUPPORTED (never a CPU fallback) when one has none. */
PTOWSP_API int ptowsp_cuda_compile(const char* plan_json, size_t plan_len, int device, ptowsp_program** out);

/* Run the workload once.  Replaces the generated entry point
 * `<module>_main(RuntimeContext*, CSPTContext*)` (reference:
 * include/pto/wsp/codegen/abi/workload_abi.hpp:71, emitted by
 * src/python/pto_codegen.cpp:1468-2709).  Returns the makespan of the
 * reference cycle model (Scheduler::issue, pto_codegen.cpp:1562-1606), the same
 * u64 the CPU-sim returns; 0 with ptowsp_cuda_status() != 0 on failure.
 * Blocks until the device work and copies of this run are done. */
PTOWSP_API uint64_t ptowsp_cuda_main(ptowsp_program* prog, struct RuntimeContext* ctx, struct CSPTContext* cspt);

/* Run one task of kernel `kernel_name` (all tensor pointers in `task` are
 * device pointers).  Replaces the per-kernel entry
 * `<kernel>(const KernelTaskDesc*, CSPTContext*)` (reference:
 * include/pto/wsp/codegen/abi/kernel_abi.hpp:70; called per task by the NPU
 * dispatcher, src/python/pto_codegen.cpp:3263-3268).  Returns the kernel's
 * model cycle charge. */
PTOWSP_API uint64_t ptowsp_cuda_run_task(ptowsp_program* prog, const char* kernel_name, const struct KernelTaskDesc* task);

/* Status of the last call on `prog` (0 = ok) and a thread-local message. */
PTOWSP_API int ptowsp_cuda_status(const ptowsp_program* prog);
PTOWSP_API const char* ptowsp_cuda_last_error(void);

/* Launch on this CUDA stream (cudaStream_t); NULL = the CUDA default stream.
 * Until this is called a program uses a private non-blocking stream. */
PTOWSP_API int ptowsp_cuda_set_stream(ptowsp_program* prog, void* cuda_stream);

/* Integer options: "pipeline_chunks" (a static workload with one batch per
 * wave whose host tensors hold 64 MiB or more, with written tensors fully
 * overwritten by one wave and read only by later ones, runs as up to this many
 * chunks of tasks whose host->device copies,
 * kernels and device->host copies overlap on three streams; chunks carry at
 * least 4 MiB of host traffic; 1 turns it off; default 32.  Pinned host memory
 * is needed for the copies to overlap), "stage_scratch_mb" (the HBM scratch a
 * kernel cut into stages may use: its stages run over groups of tasks whose
 * crossing values fit, default 2048), "cache_plans" (reuse the task table
 * of static workloads across runs, default 1), "sync" (0: when every tensor
 * is device memory, return without waiting; errors surface at the next
 * synchronous run, default 1), "dry_run" (1: walk the task loop on the host
 * only -- makespan, task and wave counts -- with no CUDA call, default 0),
 * "kernel_events" (1: bracket every kernel's launches with CUDA events on the
 * launch stream and sum their device time per kernel, read by
 * ptowsp_cuda_kernel_times; setting it clears the sums; default 0),
 * "fused_attention" (0: kernels of the attention pattern run as their stages
 * -- matmul kernels and row programs over HBM scratch -- instead of the fused
 * tcgen05 kernel; default 1), "csp_device" (0: a CSP pipeline body runs as
 * dependency waves instead of one CTA per process with device channels;
 * changing it drops the cached task tables; default 1 -- ptowsp_cuda_describe
 * reports the form a run took and, for waves, why), "decode_chunk" (the
 * split-KV chunk of the built-in paged decode, in tokens, taken as a multiple
 * of 16 inside 512 .. 1536; 0, the default, chooses it per launch: 1536
 * unless the launch has too few tasks for 1.5 chunks per SM, then shorter
 * chunks).
 * "stage_scratch_mb" is clamped to 1 .. 1048576; changing it drops the cached
 * task tables, which were grouped for the old budget. */
PTOWSP_API int ptowsp_cuda_set_option(ptowsp_program* prog, const char* key, int64_t value);

/* Per-kernel device time since "kernel_events" was last set, as JSON
 * {"<kernel>": {"launches": n, "ms": t}, ...} (waits for the recorded events).
 * No counterpart in the reference, whose CPU-sim reports model cycles only.
 * Owned by `prog`, valid until the next call. */
PTOWSP_API const char* ptowsp_cuda_kernel_times(ptowsp_program* prog);

typedef struct ptowsp_timing {
    double gpu_ms;        /* kernel time of the last run (CUDA events; overlapped runs: first to last kernel, copies between them included) */
    double total_ms;      /* wall time of the last ptowsp_cuda_main call */
    uint64_t launches;    /* kernel launches of the last run */
    uint64_t tasks;       /* tasks executed */
    uint64_t waves;       /* dependency waves */
    uint64_t h2d_bytes;   /* host->device bytes staged */
    uint64_t d2h_bytes;   /* device->host bytes staged */
    uint64_t slot_syncs;  /* device reads made for slot_load_u64 (one per device input read, one per load of
                             data that an enqueued task writes, after those tasks finish) */
    uint64_t chunks;      /* chunks of an overlapped host-staged run (copies, kernels and copies back on three
                             streams); 0: staged copies and kernels ran back to back.  A dry run reports the
                             chunks a run with the same buffers would use. */
    uint64_t walks;       /* host walks of the task loop in the last run (0: a cached task table was replayed, or
                             its records were rebuilt on the device) */
    uint64_t expansions;  /* loops whose task records the device rebuilt for new ragged lengths or a new sparse
                             selection, with no host walk and no record upload */
} ptowsp_timing;

PTOWSP_API int ptowsp_cuda_last_timing(const ptowsp_program* prog, ptowsp_timing* out);

/* JSON description of the compiled program (kernel -> implementation, task
 * windows, launch shapes).  Owned by `prog`, valid until the next call. */
PTOWSP_API const char* ptowsp_cuda_describe(ptowsp_program* prog);

PTOWSP_API void ptowsp_cuda_destroy(ptowsp_program* prog);

/* ------------------------------------------------------------------------- */
/* Paged GQA decode that allocates no device memory.  No counterpart in the    */
/* reference (whose CPU-sim allocates nothing on a device); added for callers  */
/* that must not let a library call cudaMalloc/cudaFree during a call: serving */
/* engines that reserve all device memory up front for their own KV-cache pool */
/* (an extra allocation can fail or eat into that pool), and hosts running     */
/* other streams that cannot take the implicit synchronisation those calls can */
/* cause.  The scratch space (task records, split-KV partials, status word)    */
/* lives in one fixed 24 MiB array owned by this library in device memory;     */
/* every GPU that loads the library holds it until the process exits.          */
/*                                                                             */
/* All pointers are device memory on the calling thread's current device:     */
/*   q          f16 [num_requests][num_kv_heads][group][head_dim]              */
/*   k_cache,   f16 [num_pages][page_size][num_kv_heads][head_dim]             */
/*   v_cache                                                                   */
/*   page_table i32 [num_requests][max_pages]   (page ids of each request)     */
/*   kv_len     i32 [num_requests]              (tokens of each request)       */
/*   out        f16 [num_requests][num_kv_heads][group][head_dim]              */
/* head_dim must be 128 and group 1, 2, 4 or 8.  Same math as the             */
/* paged_decode_gqa built-in.  Blocks until the work on `stream` (NULL = the  */
/* default stream) has finished and returns a ptowsp_status:                   */
/* PTOWSP_ERR_LIMIT when the work needs more than the fixed array              */
/* (ptowsp_cuda_noalloc_scratch_bytes tells how much it needs),                */
/* PTOWSP_ERR_DEVICE for a page id outside the cache or a length beyond the   */
/* page table.  Calls share the array: two calls that overlap on the GPU race. */
/* The first call on a device looks up the array's address and loads the     */
/* code of every kernel this entry point can launch (with lazy module loading  */
/* that takes device memory once); make it before any stream capture.  Calls  */
/* after the first take no device memory, whatever their GQA group.           */
PTOWSP_API int ptowsp_cuda_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                const int32_t* page_table, const int32_t* kv_len, void* out,
                                                int num_requests, int num_kv_heads, int group, int head_dim,
                                                int page_size, int max_pages, int64_t num_pages, void* stream);

/* Bytes of the fixed array a ptowsp_cuda_paged_decode_noalloc call with these
 * sizes needs; with num_requests <= 0 and num_kv_heads <= 0, the array's size. */
PTOWSP_API size_t ptowsp_cuda_noalloc_scratch_bytes(int num_requests, int num_kv_heads, int group, int max_pages,
                                                    int page_size);

/* Number of CUDA devices visible to this library (0 without a GPU). */
PTOWSP_API int ptowsp_cuda_device_count(void);

#ifdef __cplusplus
}
#endif

#endif /* PTOWSP_CUDA_H */
