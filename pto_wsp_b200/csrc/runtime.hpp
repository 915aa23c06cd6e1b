// Host runtime of the cuda_sm100a target.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/ptowsp_cuda.h"
#include "device.hpp"
#include "plan.hpp"

namespace ptowsp {

enum class ImplKind : uint8_t { RmsNorm, Softmax, TileProgram, Matmul, MatmulAcc, MatmulEpilogue, PagedDecode,
                                IndexerScore, TopK, Staged, Attention };

// One stage of a generic kernel cut at its contractions: a matmul (tcgen05 tile kernel for f16 params of its
// shapes, else the CUDA-core kernel with the tile program's fused multiply-add order) or a fused row program.
// Values that cross stages live in f32 scratch tiles in HBM, one per task; a row program sees them as params
// num_tensor_params + j.
struct Stage {
    bool mm = false;
    int a = 0, b = 0;            // matmul operands: a tensor param (>= 0) or ~scratch tile (< 0)
    int c = 0;                   // matmul result: scratch tile
    int m = 0, n = 0, k = 0;     // 128 x n = (128 x k) . (k x n) for the tile kernel; any shape on CUDA cores
    bool tc = false;             // f16 params in the tcgen05 tile kernel's shapes
    int tn = 0;                  // its tile width: each task's n columns run as n / tn tiles of 128 x tn
    dev::TileProgram tp{};       // row stage
    int rows = 0;                // its rows per task
    int jit_state = 0;           // 2 compiled (cubin), 1 loaded, -1 failed
    std::string cubin;
    void* fn = nullptr;
    void* fn_vec = nullptr;
};

const char* impl_name(ImplKind k);

// How one kernel definition runs on the GPU.
struct KernelImpl {
    ImplKind kind = ImplKind::TileProgram;
    uint64_t cycles = 0;                 // reference cycle-model charge per task
    std::vector<uint8_t> param_read;     // per tensor param
    std::vector<uint8_t> param_write;    // per tensor param
    dev::TileProgram tp{};               // generic tile program (also the fallback of RmsNorm/Softmax)
    int tp_smem = 0;
    bool tp_ok = false;                  // tile program fits the device
    std::string tp_error;
    dev::TileProgram* tp_dev = nullptr;  // device copy
    int scalar_page_size = 16, scalar_kv_heads = 1;  // paged decode static params
    // fused row kernel of a row-local tile program: 0 not tried, 2 compiled (cubin), 1 loaded, -1 interpreter
    int jit_state = 0;
    std::string jit_cubin;
    void* jit_fn = nullptr;              // CUfunction once loaded
    void* jit_fn_vec = nullptr;          // its vector-access variant, when the program has one
    std::string jit_note;                // why the interpreter runs instead
    // MatmulEpilogue: the kernel's one f16 x f16 -> f32 matmul of params ep_a, ep_b (128 x ep_k by ep_k x ep_n)
    // runs on the tcgen05 tile kernel into scratch; the rest is ep_tp, a row program that reads that tile as
    // param num_tensor_params, built as its own fused kernel
    dev::TileProgram ep_tp{};
    int ep_a = -1, ep_b = -1, ep_n = 0, ep_k = 0;
    int ep_jit_state = 0;                // as jit_state
    std::string ep_cubin;
    void* ep_fn = nullptr;
    void* ep_fn_vec = nullptr;
    // Staged: the stages in order and the [rows, cols] of each f32 scratch tile
    std::vector<Stage> stages;
    std::vector<std::pair<int, int>> scratch_tiles;
    // Attention (fused tcgen05 kernel; the stages above stay as the fallback for views it does not take): tensor
    // param indices of Q, K^T, V and the output, the key count, and the score scale (0 none, 1 the constant
    // at_scale_const, 2 scalar param at_scale_index)
    int at_q = -1, at_kt = -1, at_v = -1, at_o = -1, at_L = 0;
    int at_scale_mode = 0, at_scale_index = -1;
    float at_scale_const = 1.f;
};
// Whether a kernel is the fused attention pattern (Q.K^T [* scale] -> row softmax -> . V -> store; f16 Q and K^T,
// f32 V and output, 128 x 128 Q / output tiles, L keys a multiple of 64); fills the at_* fields.
bool match_attention(KernelImpl& ki, const KernelDef& kd);

// Build (NVRTC) the fused row kernel of kernel `k` when its tile program is row-local (jit_state -> 2 or -1).
void jit_prepare(KernelImpl& ki, const KernelDef& kd, int k);
// Split a generic kernel into a tcgen05 matmul and a fused row-program epilogue when its shape allows
// (kind -> MatmulEpilogue); false leaves the kernel as it is.
bool split_matmul_epilogue(KernelImpl& ki, const KernelDef& kd, int k);
// Cut a generic kernel with contractions into stages (matmuls and fused row programs over f32 scratch tiles) when
// every stage between two contractions is row-local; fills ki.stages (the kind is left to the caller).
bool split_stages(KernelImpl& ki, const KernelDef& kd);
// NVRTC build of a row stage as kernel `name` (+ `name`_v); params past the kernel's own are f32 scratch tiles.
bool build_stage_program(const dev::TileProgram& tp, const KernelDef& kd, const std::string& name, std::string* cubin,
                         std::string* note);

// Per-tensor binding of one run.
struct TensorBinding {
    void* user_ptr = nullptr;       // pointer from RuntimeContext
    bool on_device = false;         // user_ptr is device memory
    char* dev = nullptr;            // device pointer used by kernels
    std::vector<int64_t> strides;   // elements
    int64_t span = 0;               // addressable elements from base
    size_t bytes = 0;
    bool read = false, written = false;
};

struct Batch {  // tasks of one kernel inside one wave
    int kernel = -1;
    const Node* node = nullptr;    // task node whose tensor bindings the batch uses
    std::vector<int64_t> rec;      // host records
    int64_t ntasks = 0;
    int stride = 0;
    size_t dev_off = 0;            // element offset in the device record buffer
    bool aligned_rows = true;      // fast row kernels usable
    int8_t fast_ok = -1;           // hand-written kernel usable for every task (-1: not checked yet)
    // tcgen05 matmul: pairs of tasks that share their A tile and cover adjacent
    // N tiles run as one 128x(2N) tile; their merged records live here.
    int64_t* fast_rec_dev = nullptr;
    int64_t fast_ntasks = 0;
    int fast_n = 0;
    // CTA-pair matmul: units of two (possibly N-merged) tasks 128 rows apart in A and C sharing B,
    // records [oa, ob, oc] x 2 (-1: not checked yet, 0: the tasks do not pair up)
    int64_t* unit_rec_dev = nullptr;
    int64_t nunits = 0;
    int8_t units_ok = -1;
    // matmul + row-program epilogue: records of the matmul stage [oa, ob, scratch offset] and of the epilogue
    // [the batch's records with the scratch offset after the view offsets] (-1 not built, 0 unusable, 1 built)
    int64_t* ep_mm_rec_dev = nullptr;
    int64_t* ep_rec_dev = nullptr;
    int64_t* ep_unit_rec_dev = nullptr;  // matmul stage on CTA pairs: tasks 128 rows apart in A sharing B
    int64_t ep_nunits = 0;
    int8_t ep_ok = -1;
    // device-selected scalars: every task takes the scalars of the leaf of `sel` that its tensor element picks;
    // rows [task, element offset, signed-compare mask, other operand per cond, leaf scalars...]
    const DevSelect* sel = nullptr;
    uint32_t sel_tensor = 0;
    std::vector<uint64_t> sel_rows;
    int sel_row_words = 0;
    uint64_t* sel_dev = nullptr;
    int* sel_tree_dev = nullptr;
    // host-staged pipelining: per chunk and tensor param, the [lo, hi) element range its tasks touch
    int chunk_n = 0;
    std::vector<int64_t> chunk_ranges;
    std::vector<uint8_t> chunk_exact;  // per param: every chunk's tiles cover its range exactly once
    // Staged: [row-stage records (the batch's records with the scratch offsets after the view offsets) |
    // [oa, ob, oc] per task for each matmul stage] (-1 not built, 1 built)
    int64_t* st_rec_dev = nullptr;
    int8_t at_ok = -1;               // Attention: every task's views meet the fused kernel's conditions
    int8_t st_ok = -1;
    uint32_t st_tc_mask = 0;           // matmul stages (in order) that run on the tcgen05 tile kernel
    int64_t st_group = 0;              // tasks per group of stage launches (scratch offsets repeat per group)
    Batch() = default;
    Batch(Batch&& o) noexcept { *this = std::move(o); }
    Batch& operator=(Batch&& o) noexcept {
        kernel = o.kernel; node = o.node; rec = std::move(o.rec); ntasks = o.ntasks; stride = o.stride;
        dev_off = o.dev_off; aligned_rows = o.aligned_rows; fast_ok = o.fast_ok; fast_rec_dev = o.fast_rec_dev;
        fast_ntasks = o.fast_ntasks; fast_n = o.fast_n; chunk_n = o.chunk_n; chunk_ranges = std::move(o.chunk_ranges);
        chunk_exact = std::move(o.chunk_exact);
        unit_rec_dev = o.unit_rec_dev; nunits = o.nunits; units_ok = o.units_ok;
        ep_mm_rec_dev = o.ep_mm_rec_dev; ep_rec_dev = o.ep_rec_dev; ep_ok = o.ep_ok;
        ep_unit_rec_dev = o.ep_unit_rec_dev; ep_nunits = o.ep_nunits;
        o.ep_unit_rec_dev = nullptr;
        st_rec_dev = o.st_rec_dev; st_ok = o.st_ok; st_tc_mask = o.st_tc_mask; st_group = o.st_group;
        o.st_rec_dev = nullptr;
        sel = o.sel; sel_tensor = o.sel_tensor; sel_rows = std::move(o.sel_rows); sel_row_words = o.sel_row_words;
        sel_dev = o.sel_dev; sel_tree_dev = o.sel_tree_dev;
        o.sel_dev = nullptr;
        o.sel_tree_dev = nullptr;
        o.fast_rec_dev = nullptr;
        o.unit_rec_dev = nullptr;
        o.ep_mm_rec_dev = nullptr;
        o.ep_rec_dev = nullptr;
        return *this;
    }
    Batch(const Batch&) = delete;
    Batch& operator=(const Batch&) = delete;
    ~Batch();
};

struct Wave {
    std::vector<Batch> batches;
    std::unordered_map<const Node*, size_t> by_node;  // task node -> batch index
};

// A loop over a ragged axis or a sparse selection whose body is one task, in a workload of that loop alone: its
// task records are affine in the loop variable (record = base + var * delta), so a run with other lengths or
// another selection rebuilds them on the device (expand_records_kernel) instead of walking the loop on the host.
struct LoopExpand {
    char kind = 0;              // 'r' ragged (var = 0 .. sum of lengths - 1), 'c' selection (var = indices[p])
    size_t key_index = 0;       // its entry in LaunchProgram::key
    std::string key_name;       // that entry up to '='
    size_t outer_key_index = SIZE_MAX;  // the entry of its outer-size symbol (which may change with it)
    uint64_t lengths_sym = 0, outer_sym = 0, indptr_sym = 0, indices_sym = 0;
    bool parallel = true;       // ParallelFor (tasks issued from the same ready time) or ForEach (chained)
    bool writes = false;        // the kernel writes a tensor (a selection with repeated indices must be walked)
    std::vector<int64_t> base, delta;  // per record word
    int64_t* base_delta_dev = nullptr; // [base | delta] on the device
    int32_t* vars_dev = nullptr;       // selection indices of the last expanded run
    size_t vars_cap = 0;
};

// A CSP pipeline run on the device: one CTA per process (dev::CspArgs).  The walk builds it when the workload's body
// is one pipeline whose tasks the tile-program interpreter runs, whose channels have one sender and one receiver
// each, and whose data hazards between processes are all ordered by the channels (checked with vector clocks over
// the device's channel semantics: a receive waits for its send, a send for the receive `cap` tokens earlier).
struct CspDevice {
    std::vector<dev::CspOp> ops;            // every process's operations, process after process
    std::vector<int32_t> proc_first;        // [nproc + 1]
    std::vector<int64_t> rec;               // task records (op.rec: word offset)
    std::vector<const Node*> slot_node;     // per kernel slot: a task node of that slot (params, tensor bindings)
    std::vector<int32_t> caps;              // per channel: device capacity (>= 1)
    int smem = 0;                           // interpreter shared memory, the largest slot's
    dev::CspOp* ops_dev = nullptr;
    int32_t* first_dev = nullptr;
    int64_t* rec_dev = nullptr;
    int32_t* caps_dev = nullptr;
    dev::TaskBatch* tb_dev = nullptr;
    const dev::TileProgram** prog_dev = nullptr;
    unsigned* counts_dev = nullptr;
    CspDevice() = default;
    CspDevice(const CspDevice&) = delete;
    CspDevice& operator=(const CspDevice&) = delete;
    ~CspDevice();
};

struct LaunchProgram {  // result of one walk, reusable for static workloads
    std::vector<Wave> waves;
    std::unique_ptr<LoopExpand> expand;  // set when the workload is one loop whose records the device can rebuild
    bool no_pipeline = false;            // records rebuilt on the device: no host copy for chunk planning
    uint64_t makespan = 0;
    uint64_t tasks = 0;
    size_t rec_elems = 0;
    int64_t* rec_dev = nullptr;
    size_t rec_cap = 0;
    std::vector<std::string> key;  // replay log of runtime queries
    std::vector<uint8_t> full_write;  // per tensor: every element overwritten
    std::vector<uint8_t> write_first; // per tensor: every element overwritten in waves before any task reads it
    std::unique_ptr<CspDevice> csp;   // the body is a CSP pipeline the device runs as processes (else waves)
    std::string csp_note;             // why a pipeline body runs as waves (empty when it runs as processes)
    LaunchProgram() = default;
    LaunchProgram(const LaunchProgram&) = delete;
    LaunchProgram& operator=(const LaunchProgram&) = delete;
    ~LaunchProgram();
};

struct Program {
    Plan plan;
    std::vector<KernelImpl> impls;
    std::vector<int> tensor_key_depth;   // coarsest index depth per tensor (hazard keys)
    bool cacheable = true;                // no data-dependent control flow
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    bool stream_set = false;           // caller chose a stream (nullptr = CUDA default stream)
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;  // copy engines of pipelined runs
    std::vector<cudaEvent_t> pipe_events;
    int* err_dev = nullptr;
    int status = 0;
    int64_t opt_cache = 1, opt_chunks = 32, opt_sync = 1, opt_dry = 0, opt_stage_scratch_mb = 2048;
    int64_t opt_kernel_events = 0;       // bracket every batch launch with CUDA events (per-kernel device time)
    int64_t opt_fused_attention = 1;     // 0: attention kernels run their stages instead of the fused kernel
    int64_t opt_csp_device = 1;          // 0: CSP pipelines run as dependency waves instead of device processes
    int64_t opt_decode_chunk = 0;        // paged decode split-KV chunk (tokens); 0: chosen per launch
    std::string csp_mode;                // last run's CSP execution: "" (no pipeline), "device_processes", "waves: why"
    struct KernelEvent { int kernel; cudaEvent_t start, end; };
    std::vector<KernelEvent> kev_pending;  // recorded, not yet read
    std::vector<cudaEvent_t> kev_free;     // event pool
    std::vector<std::pair<uint64_t, double>> kev_totals;  // per kernel: launches, device ms
    std::string kernel_times_json;
    std::vector<char*> dev_bufs;         // host-staged tensor buffers (by tensor id)
    std::vector<size_t> dev_caps;
    void* scratch = nullptr;
    size_t scratch_cap = 0;
    std::unique_ptr<LaunchProgram> cached;
    ptowsp_timing timing{};
    std::string describe_json;

    ~Program();
};

std::unique_ptr<Program> compile_program(const char* text, size_t len, int device);
uint64_t run_program(Program& p, RuntimeContext* ctx);
uint64_t run_single_task(Program& p, const std::string& kernel, const KernelTaskDesc* task);
std::string describe_program(const Program& p);
std::string kernel_times(Program& p);   // per-kernel launches and device ms since the last reset (JSON)
void reset_kernel_times(Program& p);

// Error helpers (thread-local message).
void set_error(const std::string& msg);
const char* last_error();

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

}  // namespace ptowsp
