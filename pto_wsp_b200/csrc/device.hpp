// Structures shared by the host runtime and the sm_100a kernels.
//
// A launch executes a *task batch*: a slice of the device task table.  Each
// task record holds, per kernel tensor param, the element offset of the task's
// tile view from the tensor base (base + sum(idx * stride), the pointer the
// reference computes per task at src/python/pto_codegen.cpp:2570-2592), then
// the task's axis args and scalar args (the u64 `args` of KernelTaskDesc,
// include/pto/wsp/codegen/abi/kernel_abi.hpp:21-41).
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#include <cuda_runtime.h>
#else
#include <cuda_runtime_api.h>
#endif

namespace ptowsp::dev {

constexpr int kMaxParams = 8;

// Device status word bits (set by kernels, read by the host after a run).
enum : int {
    kErrBounds = 1,      // an index computed from task data left its tensor
    kErrTimeout = 2,     // a bounded wait gave up
    kErrShape = 4,       // a runtime size exceeded a kernel's static limit
};

enum ParamType : int { PT_F32 = 0, PT_F16 = 1, PT_I32 = 2, PT_U32 = 3, PT_I64 = 4, PT_U64 = 5, PT_OTHER = 6 };

struct ParamDesc {
    char* base;       // device base pointer of the tensor
    int64_t s3, s4;   // row / column stride of the tile view, in elements
    int64_t numel_span;  // elements addressable from base (bounds checks)
    int rows, cols;   // static tile shape of the kernel param
    int type;         // ParamType
    int elem_bytes;
};

struct TaskBatch {
    const int64_t* rec;  // [ntasks][stride]
    int64_t ntasks;
    int stride;          // nparams + naxis + nscalar
    int nparams, naxis, nscalar;
    ParamDesc p[kMaxParams];
    int* err;            // device status word
};

// ---------------------------------------------------------------------------
// Generic tile program (any pto.* kernel without a hand-written kernel).
// Mirrors the op set of the reference kernel emitter
// (src/python/pto_codegen.cpp:785-1231).
// ---------------------------------------------------------------------------

enum TPOp : int {
    TP_LOAD = 1, TP_STORE, TP_BIN, TP_BINS, TP_EXP, TP_RSQRT, TP_ROWSUM, TP_ROWMAX, TP_ROWMEAN,
    TP_MATMUL, TP_IOTA, TP_TSORT32, TP_EXTRACT, TP_MOV
};
enum TPBin : int { BIN_ADD = 0, BIN_SUB, BIN_MUL, BIN_DIV, BIN_MAX, BIN_MIN };
enum TPMode : int { MODE_FULL = 0, MODE_ROW, MODE_COL };
enum TPWord : int { W_F32 = 0, W_I32 = 1, W_U32 = 2 };

struct TPSlot {
    int off;      // word offset in shared memory
    int rows, cols, pitch;
    int word;     // TPWord
};

struct TPInstr {
    int op, sub, mode;
    int dst, a, b;      // slot ids (or param index for LOAD/STORE)
    int param;          // tensor param index (LOAD/STORE)
    int rows, cols, k;  // shape info
    int scalar_src;     // BINS: -1 = literal `fval`/`ival`; >=0 scalar param index
    int scalar_first;   // BINS div: scalar / tile
    float fval;
    int ival;
};

constexpr int kTPMaxSlots = 64;
constexpr int kTPMaxInstr = 128;

struct TileProgram {
    int ninstr, nslots, smem_words;
    TPSlot slots[kTPMaxSlots];
    TPInstr ins[kTPMaxInstr];
    int scalar_types[kMaxParams];  // per scalar param: 0 f32, 1 i32, 2 i64, 3 bool
};

// ---------------------------------------------------------------------------
// Launchers (defined in the .cu files).  All return cudaSuccess or the launch
// error; `workers` caps the number of CTAs (task window), 0 = automatic.
// ---------------------------------------------------------------------------

// Device-selected scalars: per task row [task, element offset, signed-compare mask, other operand per cond,
// leaf scalars], the cond tree as 4 ints per cond [compare (0 <, 1 <=, 2 >, 3 >=, 4 ==, 5 !=), slot on the
// left, then, else] (children >= 0: cond, < 0: ~leaf); the element is read as slot_load_u64 does (src_type: the
// plan DType code).  Writes the chosen leaf's scalars into the task's record.
cudaError_t launch_select_scalars(int64_t* rec, int stride, int scalar_pos, const uint64_t* rows, int64_t nrows,
                                  int row_words, const int* tree, int nconds, int nscalars, const void* src,
                                  int src_type, int64_t src_span, int* err, cudaStream_t s);

// Task records rebuilt on the device: rec[t][w] = base_delta[w] + var_t * base_delta[stride + w] for t < n, with
// var_t = t (vars == nullptr) or vars[t].
cudaError_t launch_expand_records(int64_t* rec, int stride, int64_t n, const int64_t* base_delta, const int32_t* vars,
                                  cudaStream_t s);

// Tile widths the hand-written RMSNorm / softmax row kernels take (others run the fused row program).
inline bool row_width_supported(int cols) { return cols == 128 || cols == 256 || cols == 512 || cols == 1024; }
cudaError_t launch_rmsnorm_rows(const TaskBatch& b, int workers, cudaStream_t s);
cudaError_t launch_softmax_rows(const TaskBatch& b, int workers, cudaStream_t s);
cudaError_t launch_tile_program(const TaskBatch& b, const TileProgram* prog_dev, int smem_bytes, int workers,
                                cudaStream_t s);
int tile_program_max_smem();

// CSP pipeline on the device (reference CSPT processes, src/python/pto_codegen.cpp:1759-2220): one CTA per
// process runs the process's operations in order -- its tasks through the tile-program interpreter, its sends and
// receives as per-channel counters in global memory (release / acquire at GPU scope, one sender and one receiver
// per channel; a send waits while `cap` tokens are unreceived).  All CTAs are resident together (cooperative
// launch); every wait is bounded (~2 s), after which the status word gets kErrTimeout and the CTA stops.
enum CspOpKind : int { CSP_TASK = 0, CSP_SEND = 1, CSP_RECV = 2 };
struct CspOp {
    int32_t kind;  // CspOpKind
    int32_t arg;   // task: kernel slot; send / receive: channel
    int64_t rec;   // task: word offset of its record in the slot's batch records
};
struct CspArgs {
    const CspOp* ops;                  // every process's operations, process after process
    const int32_t* proc_first;         // [nproc + 1]: each process's first operation
    const TaskBatch* batches;          // per kernel slot: params and record layout (rec = the records' base)
    const TileProgram* const* progs;   // per kernel slot
    unsigned* counts;                  // [2 * nchan]: tokens sent, tokens received (zero before the launch)
    const int32_t* caps;               // [nchan]: tokens a sender may have outstanding (>= 1)
    int nproc, nchan;
    int* err;
};
// False (nothing launched) when the processes cannot all be resident at once.
bool launch_csp_pipeline(const CspArgs& a, int smem_bytes, cudaStream_t s, cudaError_t* err);

// Matmul on CUDA cores, any shape: C[M,N] (f32) = A[M,K] . B[K,N] (f16 or f32) per task, records [oa, ob, oc],
// each output accumulated over k in order with fused multiply-adds (the tile program's arithmetic).
cudaError_t launch_matmul_simt(const TaskBatch& b, int M, int N, int K, int workers, cudaStream_t s);
// Matmul tile task: C[M,N] (f32) = A[M,K] (f16) . B[K,N] (f16) (+ C if accumulate).
// Params: 0 = A, 1 = B, 2 = C (same tensor for InOut).
cudaError_t launch_matmul_tiles(const TaskBatch& b, int accumulate, int workers, cudaStream_t s);
// Shape/stride/alignment conditions of the tcgen05 path (per-task offsets are checked by the host).
bool matmul_tiles_supported(const TaskBatch& b);
// CTA-pair (cta_group::2) matmul over `nunits` units of two tasks (records [oa, ob, oc] x 2, device memory) whose
// A / C tiles are 128 rows apart and whose B tile is shared; false (nothing launched) when pairs cannot be scheduled.
bool launch_matmul_pairs(const TaskBatch& b, const int64_t* units, int64_t nunits, int accumulate, int workers,
                         cudaStream_t s, cudaError_t* err);

// Fused attention tile tasks (attention_tcgen05.cu): per task O[128,128] f32 = softmax(scale * Q . K^T) . V with
// Q [128,128], K^T [128,L] f16 and V [L,128] f32 views (tensor params q_p, kt_p, v_p, o_p), L a multiple of 64; the
// scale is none (mode 0), `scale_const` (1) or the f32 scalar at record position `scale_pos` (2).
bool attention_tiles_supported(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L);
bool attention_task_ok(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L, const int64_t* rec);
cudaError_t launch_attention(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L, int scale_mode,
                             int scale_pos, float scale_const, cudaStream_t s);

// Built-ins.  `chunk_tokens`: split-KV chunk length of the paged decode (0: chosen from the launch's size).
cudaError_t launch_paged_decode(const TaskBatch& b, int page_size, int chunk_tokens, int workers, void* scratch,
                                size_t scratch_bytes, cudaStream_t s);
size_t paged_decode_scratch_bytes(const TaskBatch& b, int page_size);
cudaError_t launch_indexer_score(const TaskBatch& b, int workers, cudaStream_t s);
bool indexer_score_supported(const TaskBatch& b);
cudaError_t launch_topk_select(const TaskBatch& b, int workers, void* scratch, size_t scratch_bytes, cudaStream_t s);
size_t topk_select_scratch_bytes(const TaskBatch& b);
// Whether one row of N scores and K winners fits the one-CTA-per-row kernel's shared memory.
bool topk_supported(int n, int k);

int sm_count();

// Allocation-free paged decode over a fixed device array (decode.cu); returns a
// ptowsp_status code and sets *msg.
int paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* page_table,
                         const int32_t* kv_len, void* out, int requests, int kv_heads, int group, int head_dim,
                         int page_size, int max_pages, int64_t num_pages, cudaStream_t s, const char** msg);
size_t noalloc_scratch_capacity();
size_t noalloc_bytes_needed(int requests, int kv_heads, int group, int max_pages, int page_size);

}  // namespace ptowsp::dev
