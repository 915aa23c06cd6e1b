// Row-wise tile kernels for sm_100a: RMSNorm, softmax, and the generic tile
// program.  These are HBM-bound: each element is read once and written once,
// so the kernels stream rows with 128-bit non-temporal loads, keep a row in
// registers (one warp per row), reduce with warp shuffles and store with
// streaming stores.  A launch covers one task batch; tiles are found through
// the device task table (see device.hpp).
//
// Semantics follow the tile-op sequences the reference emits:
//   RMSNorm  TMUL -> TROWSUM -> TDIVS(cols) -> TRSQRT -> TROWEXPANDMUL -> TSTORE
//            (src/python/pto_codegen.cpp:990-1110, 1112-1130, 1194-1221)
//   softmax  TROWMAX -> TROWEXPANDSUB -> TEXP -> TROWSUM -> TROWEXPANDDIV
// The reference RMSNorm has no epsilon (examples/e2e_rmsnorm/golden.py:6-10).
#include <cuda_fp16.h>

#include <algorithm>

#include "device.hpp"

namespace ptowsp::dev {

namespace {

__device__ __forceinline__ float4 ld_stream(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(float* p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct RmsNormOp {
    template <int V>
    __device__ __forceinline__ static void apply(float4 (&x)[V], int cols) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < V; ++j) ss += x[j].x * x[j].x + x[j].y * x[j].y + x[j].z * x[j].z + x[j].w * x[j].w;
        ss = warp_sum(ss);
        const float mean = ss / static_cast<float>(cols);   // TROWSUM, TDIVS(cols)
        const float inv = 1.0f / sqrtf(mean);                // TRSQRT
#pragma unroll
        for (int j = 0; j < V; ++j) {                        // TROWEXPANDMUL
            x[j].x *= inv;
            x[j].y *= inv;
            x[j].z *= inv;
            x[j].w *= inv;
        }
    }
};

struct SoftmaxOp {
    template <int V>
    __device__ __forceinline__ static void apply(float4 (&x)[V], int) {
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < V; ++j) m = fmaxf(m, fmaxf(fmaxf(x[j].x, x[j].y), fmaxf(x[j].z, x[j].w)));
        m = warp_max(m);                                     // TROWMAX
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < V; ++j) {                        // TROWEXPANDSUB, TEXP
            x[j].x = expf(x[j].x - m);
            x[j].y = expf(x[j].y - m);
            x[j].z = expf(x[j].z - m);
            x[j].w = expf(x[j].w - m);
            s += (x[j].x + x[j].y) + (x[j].z + x[j].w);
        }
        s = warp_sum(s);                                     // TROWSUM
#pragma unroll
        for (int j = 0; j < V; ++j) {                        // TROWEXPANDDIV
            x[j].x = x[j].x / s;
            x[j].y = x[j].y / s;
            x[j].z = x[j].z / s;
            x[j].w = x[j].w / s;
        }
    }
};

// One warp per row; each warp keeps RPW rows (V float4 per lane each) in
// flight.  Param 0 = input tile, param 1 = output tile (both f32, s4 == 1,
// 16-byte aligned rows -- checked by the host before choosing this kernel).
template <class Op, int V, int RPW>
__global__ void __launch_bounds__(256) row_kernel(TaskBatch b) {
    const int R = b.p[0].rows;
    const int cols = V * 128;
    const int64_t total_rows = b.ntasks * static_cast<int64_t>(R);
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const float* __restrict__ xb = reinterpret_cast<const float*>(b.p[0].base);
    float* __restrict__ yb = reinterpret_cast<float*>(b.p[1].base);
    const int64_t xs3 = b.p[0].s3, ys3 = b.p[1].s3;

    for (int64_t row0 = warp * RPW; row0 < total_rows; row0 += nwarps * RPW) {
        float4 v[RPW][V];
        int64_t yoff[RPW];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int64_t row = row0 + r;
            yoff[r] = -1;
            if (row < total_rows) {
                const int64_t task = row / R;
                const int rr = static_cast<int>(row - task * R);
                const int64_t* rec = b.rec + task * b.stride;
                const int64_t xo = rec[0] + rr * xs3;
                yoff[r] = rec[1] + rr * ys3;
                const float* px = xb + xo + lane * 4;
#pragma unroll
                for (int j = 0; j < V; ++j) v[r][j] = ld_stream(px + j * 128);
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            if (yoff[r] < 0) continue;
            Op::template apply<V>(v[r], cols);
            float* py = yb + yoff[r] + lane * 4;
#pragma unroll
            for (int j = 0; j < V; ++j) st_stream(py + j * 128, v[r][j]);
        }
    }
}

template <class Op, int V, int RPW>
cudaError_t launch_rows_t(const TaskBatch& b, int workers, cudaStream_t s) {
    const int threads = 256;
    const int64_t total_rows = b.ntasks * static_cast<int64_t>(b.p[0].rows);
    const int64_t rows_per_block = (threads / 32) * RPW;
    int64_t blocks = (total_rows + rows_per_block - 1) / rows_per_block;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, row_kernel<Op, V, RPW>, threads, 0);
    const int64_t cap = static_cast<int64_t>(std::max(per_sm, 1)) * sm_count();
    blocks = std::min(blocks, cap);
    if (workers > 0) blocks = std::min<int64_t>(blocks, workers);
    blocks = std::max<int64_t>(blocks, 1);
    row_kernel<Op, V, RPW><<<static_cast<unsigned>(blocks), threads, 0, s>>>(b);
    return cudaGetLastError();
}

// Rows in flight per warp for the 128- and 256-column widths (configs 1 and 2).  Measured on one B200 (CUDA events,
// whole config, GB/s): 128 columns with 2 / 3 / 4 / 5 / 6 / 8 / 12 / 16 rows 6275 / 6132 / 6246 / 6222 / 6345 / 6068 /
// 4969 / 5001 -- six rows take 62 registers, so four CTAs of 256 threads fit an SM (32 warps, 192 rows in flight),
// where eight take 71 and leave three (24 warps, the same 192 rows); 256 columns with 2 / 3 / 4 / 5 / 6 / 8 rows
// 5907 / 5232 / 6149 / 5079 / 5871 / 4100; with a minimum of CTAs per SM forced by launch bounds (another box, where
// four rows gave 5804): six rows at three CTAs 5858, five or six at four CTAs and eight at three spill (5052 / 4421 /
// 3719), eight at two CTAs 4122.
#ifndef PTOWSP_ROWS_RPW128
#define PTOWSP_ROWS_RPW128 6
#endif
#ifndef PTOWSP_ROWS_RPW256
#define PTOWSP_ROWS_RPW256 4
#endif

template <class Op>
cudaError_t launch_rows(const TaskBatch& b, int workers, cudaStream_t s) {
    switch (b.p[0].cols) {
        case 128: return launch_rows_t<Op, 1, PTOWSP_ROWS_RPW128>(b, workers, s);
        case 256: return launch_rows_t<Op, 2, PTOWSP_ROWS_RPW256>(b, workers, s);
        case 512: return launch_rows_t<Op, 4, 2>(b, workers, s);
        case 1024: return launch_rows_t<Op, 8, 1>(b, workers, s);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Generic tile program: one CTA per task, tiles in shared memory as 32-bit
// words, instructions executed in order with a barrier between them.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float load_elem_f(const ParamDesc& p, int64_t off) {
    switch (p.type) {
        case PT_F32: return reinterpret_cast<const float*>(p.base)[off];
        case PT_F16: return __half2float(reinterpret_cast<const __half*>(p.base)[off]);
        case PT_I32: return static_cast<float>(reinterpret_cast<const int32_t*>(p.base)[off]);
        case PT_U32: return static_cast<float>(reinterpret_cast<const uint32_t*>(p.base)[off]);
        case PT_I64: return static_cast<float>(reinterpret_cast<const int64_t*>(p.base)[off]);
        case PT_U64: return static_cast<float>(reinterpret_cast<const uint64_t*>(p.base)[off]);
        default: return 0.f;
    }
}

__device__ __forceinline__ uint32_t load_elem_w(const ParamDesc& p, int64_t off, int word) {
    if (word == W_F32) return __float_as_uint(load_elem_f(p, off));
    switch (p.type) {
        case PT_I32: case PT_U32: return reinterpret_cast<const uint32_t*>(p.base)[off];
        case PT_I64: case PT_U64: return static_cast<uint32_t>(reinterpret_cast<const uint64_t*>(p.base)[off]);
        case PT_F32: return static_cast<uint32_t>(static_cast<int32_t>(reinterpret_cast<const float*>(p.base)[off]));
        case PT_F16: return static_cast<uint32_t>(static_cast<int32_t>(__half2float(reinterpret_cast<const __half*>(p.base)[off])));
        default: return 0u;
    }
}

__device__ __forceinline__ void store_elem(const ParamDesc& p, int64_t off, uint32_t w, int word) {
    const float f = word == W_F32 ? __uint_as_float(w) : (word == W_I32 ? static_cast<float>(static_cast<int32_t>(w)) : static_cast<float>(w));
    switch (p.type) {
        case PT_F32: reinterpret_cast<float*>(p.base)[off] = f; break;
        case PT_F16: reinterpret_cast<__half*>(p.base)[off] = __float2half_rn(f); break;
        case PT_I32: reinterpret_cast<int32_t*>(p.base)[off] = word == W_F32 ? static_cast<int32_t>(f) : static_cast<int32_t>(w); break;
        case PT_U32: reinterpret_cast<uint32_t*>(p.base)[off] = word == W_F32 ? static_cast<uint32_t>(f) : w; break;
        case PT_I64: reinterpret_cast<int64_t*>(p.base)[off] = word == W_F32 ? static_cast<int64_t>(f) : static_cast<int64_t>(static_cast<int32_t>(w)); break;
        case PT_U64: reinterpret_cast<uint64_t*>(p.base)[off] = word == W_F32 ? static_cast<uint64_t>(f) : static_cast<uint64_t>(w); break;
        default: break;
    }
}

__device__ __forceinline__ float bin_f(int op, float a, float b) {
    switch (op) {
        case BIN_ADD: return __fadd_rn(a, b);
        case BIN_SUB: return __fsub_rn(a, b);
        case BIN_MUL: return __fmul_rn(a, b);
        case BIN_DIV: return __fdiv_rn(a, b);
        case BIN_MAX: return fmaxf(a, b);
        default: return fminf(a, b);
    }
}

__device__ __forceinline__ int32_t bin_i(int op, int32_t a, int32_t b) {
    switch (op) {
        case BIN_ADD: return a + b;
        case BIN_SUB: return a - b;
        case BIN_MUL: return a * b;
        case BIN_DIV: return b ? a / b : 0;
        case BIN_MAX: return a > b ? a : b;
        default: return a < b ? a : b;
    }
}

// One task of a tile program: its instructions in order over this CTA's shared memory, a block barrier after each
// (every thread of the block calls it).  The record `rec` holds the task's view offsets, axis args and scalars.
__device__ __forceinline__ void tp_run_task(const TaskBatch& b, const TileProgram* __restrict__ prog, const int64_t* rec,
                                            uint32_t* sm) {
    const int ninstr = prog->ninstr;
    for (int ii = 0; ii < ninstr; ++ii) {
        const TPInstr in = prog->ins[ii];
        switch (in.op) {
            case TP_LOAD: {
                const TPSlot d = prog->slots[in.dst];
                const ParamDesc& p = b.p[in.param];
                const int64_t base = rec[in.param];
                for (int e = threadIdx.x; e < in.rows * in.cols; e += blockDim.x) {
                    const int r = e / in.cols, c = e - r * in.cols;
                    const int64_t off = base + r * p.s3 + c * p.s4;
                    uint32_t w = 0;
                    if (off >= 0 && off < p.numel_span) w = load_elem_w(p, off, d.word);
                    else atomicOr(b.err, kErrBounds);
                    sm[d.off + r * d.pitch + c] = w;
                }
                break;
            }
            case TP_STORE: {
                const TPSlot a = prog->slots[in.a];
                const ParamDesc& p = b.p[in.param];
                const int64_t base = rec[in.param];
                for (int e = threadIdx.x; e < in.rows * in.cols; e += blockDim.x) {
                    const int r = e / in.cols, c = e - r * in.cols;
                    const int64_t off = base + r * p.s3 + c * p.s4;
                    const uint32_t w = (r < a.rows && c < a.cols) ? sm[a.off + r * a.pitch + c] : 0u;
                    if (off >= 0 && off < p.numel_span) store_elem(p, off, w, a.word);
                    else atomicOr(b.err, kErrBounds);
                }
                break;
            }
            case TP_MOV: {
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a];
                for (int e = threadIdx.x; e < d.rows * d.cols; e += blockDim.x) {
                    const int r = e / d.cols, c = e - r * d.cols;
                    sm[d.off + r * d.pitch + c] = sm[a.off + r * a.pitch + c];
                }
                break;
            }
            case TP_BIN: {
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a], bb = prog->slots[in.b];
                for (int e = threadIdx.x; e < d.rows * d.cols; e += blockDim.x) {
                    const int r = e / d.cols, c = e - r * d.cols;
                    const uint32_t wa = sm[a.off + r * a.pitch + c];
                    const int bi = in.mode == MODE_FULL ? (bb.off + r * bb.pitch + c)
                                   : in.mode == MODE_ROW ? (bb.off + r) : (bb.off + c);
                    const uint32_t wb = sm[bi];
                    uint32_t out;
                    if (d.word == W_F32) out = __float_as_uint(bin_f(in.sub, __uint_as_float(wa), __uint_as_float(wb)));
                    else out = static_cast<uint32_t>(bin_i(in.sub, static_cast<int32_t>(wa), static_cast<int32_t>(wb)));
                    sm[d.off + r * d.pitch + c] = out;
                }
                break;
            }
            case TP_BINS: {
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a];
                float fs = in.fval;
                int32_t is = in.ival;
                if (in.scalar_src >= 0) {
                    const uint64_t raw = static_cast<uint64_t>(rec[b.nparams + b.naxis + in.scalar_src]);
                    const int st = prog->scalar_types[in.scalar_src];
                    if (st == 0) {
                        fs = __uint_as_float(static_cast<uint32_t>(raw));
                        is = static_cast<int32_t>(fs);
                    } else {
                        is = static_cast<int32_t>(raw);
                        fs = st == 2 ? static_cast<float>(static_cast<int64_t>(raw)) : static_cast<float>(is);
                    }
                }
                for (int e = threadIdx.x; e < d.rows * d.cols; e += blockDim.x) {
                    const int r = e / d.cols, c = e - r * d.cols;
                    const uint32_t wa = sm[a.off + r * a.pitch + c];
                    uint32_t out;
                    if (d.word == W_F32) {
                        const float x = __uint_as_float(wa);
                        out = __float_as_uint(in.scalar_first ? bin_f(in.sub, fs, x) : bin_f(in.sub, x, fs));
                    } else {
                        const int32_t x = static_cast<int32_t>(wa);
                        out = static_cast<uint32_t>(in.scalar_first ? bin_i(in.sub, is, x) : bin_i(in.sub, x, is));
                    }
                    sm[d.off + r * d.pitch + c] = out;
                }
                break;
            }
            case TP_EXP:
            case TP_RSQRT: {
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a];
                for (int e = threadIdx.x; e < d.rows * d.cols; e += blockDim.x) {
                    const int r = e / d.cols, c = e - r * d.cols;
                    const float x = __uint_as_float(sm[a.off + r * a.pitch + c]);
                    const float y = in.op == TP_EXP ? expf(x) : __fdiv_rn(1.0f, sqrtf(x));
                    sm[d.off + r * d.pitch + c] = __float_as_uint(y);
                }
                break;
            }
            case TP_ROWSUM:
            case TP_ROWMAX:
            case TP_ROWMEAN: {
                // Sequential column order per row (one thread per row).
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a];
                for (int r = threadIdx.x; r < d.rows; r += blockDim.x) {
                    float acc = in.op == TP_ROWMAX ? -INFINITY : 0.f;
                    for (int c = 0; c < a.cols; ++c) {
                        const float x = __uint_as_float(sm[a.off + r * a.pitch + c]);
                        acc = in.op == TP_ROWMAX ? fmaxf(acc, x) : __fadd_rn(acc, x);
                    }
                    if (in.op == TP_ROWMEAN) acc = __fdiv_rn(acc, static_cast<float>(in.k));
                    sm[d.off + r * d.pitch] = __float_as_uint(acc);
                }
                break;
            }
            case TP_MATMUL: {
                // f32 accumulation in k order, one fused multiply-add (single rounding) per step.
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a], bb = prog->slots[in.b];
                for (int e = threadIdx.x; e < in.rows * in.cols; e += blockDim.x) {
                    const int r = e / in.cols, c = e - r * in.cols;
                    float acc = 0.f;
                    for (int kk = 0; kk < in.k; ++kk)
                        acc = __fmaf_rn(__uint_as_float(sm[a.off + r * a.pitch + kk]),
                                        __uint_as_float(sm[bb.off + kk * bb.pitch + c]), acc);
                    sm[d.off + r * d.pitch + c] = __float_as_uint(acc);
                }
                break;
            }
            case TP_IOTA: {
                const TPSlot d = prog->slots[in.dst];
                for (int c = threadIdx.x; c < d.cols; c += blockDim.x) sm[d.off + c] = static_cast<uint32_t>(c);
                break;
            }
            case TP_TSORT32: {
                // Stable descending sort of n (<= rows*cols) scores with their indices:
                // rank_i = #{j : s_j > s_i or (s_j == s_i and j < i)}; dst = interleaved (score, index).
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a], ix = prog->slots[in.b];
                const int n = in.k;
                for (int i = threadIdx.x; i < n; i += blockDim.x) {
                    const float si = __uint_as_float(sm[a.off + (i / a.cols) * a.pitch + (i % a.cols)]);
                    int rank = 0;
                    for (int j = 0; j < n; ++j) {
                        const float sj = __uint_as_float(sm[a.off + (j / a.cols) * a.pitch + (j % a.cols)]);
                        rank += (sj > si) || (sj == si && j < i);
                    }
                    const uint32_t idx = sm[ix.off + (i / ix.cols) * ix.pitch + (i % ix.cols)];
                    const int p0 = 2 * rank, p1 = 2 * rank + 1;
                    if (p1 < d.rows * d.cols) {
                        sm[d.off + (p0 / d.cols) * d.pitch + (p0 % d.cols)] = __float_as_uint(si);
                        sm[d.off + (p1 / d.cols) * d.pitch + (p1 % d.cols)] = __float_as_uint(static_cast<float>(idx));
                    }
                }
                break;
            }
            case TP_EXTRACT: {
                const TPSlot d = prog->slots[in.dst], a = prog->slots[in.a];
                for (int i = threadIdx.x; i < in.k; i += blockDim.x) {
                    const int p = 2 * i + 1;
                    const float f = __uint_as_float(sm[a.off + (p / a.cols) * a.pitch + (p % a.cols)]);
                    if (i < d.rows * d.cols) sm[d.off + (i / d.cols) * d.pitch + (i % d.cols)] = static_cast<uint32_t>(static_cast<int32_t>(f));
                }
                break;
            }
            default:
                break;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(256) tile_program_kernel(const __grid_constant__ TaskBatch b,
                                                           const TileProgram* __restrict__ prog) {
    extern __shared__ uint32_t sm[];
    for (int64_t task = blockIdx.x; task < b.ntasks; task += gridDim.x) tp_run_task(b, prog, b.rec + task * b.stride, sm);
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t csp_clock_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One CTA per CSP process (see CspArgs).  A send makes the CTA's earlier task writes visible before its token
// (block barrier, then thread 0's fence and release store); a receive's acquire load, fence and block barrier
// make the sender's writes visible to every thread of the receiving CTA before its next task.
__global__ void __launch_bounds__(256) csp_pipeline_kernel(const __grid_constant__ CspArgs a) {
    extern __shared__ uint32_t sm[];
    __shared__ int s_stop;
    const int p = blockIdx.x;
    if (threadIdx.x == 0) s_stop = 0;
    __syncthreads();
    constexpr uint64_t kWaitNs = 2000000000ull;
    for (int i = a.proc_first[p]; i < a.proc_first[p + 1]; ++i) {
        const CspOp op = a.ops[i];
        if (op.kind == CSP_TASK) {
            const TaskBatch& b = a.batches[op.arg];
            tp_run_task(b, a.progs[op.arg], b.rec + op.rec, sm);  // ends with a block barrier
            continue;
        }
        __syncthreads();  // every thread's writes of the tasks before a send precede the token
        if (threadIdx.x == 0) {
            unsigned* sent = a.counts + 2 * op.arg;
            unsigned* recvd = sent + 1;
            const uint64_t t0 = csp_clock_ns();
            if (op.kind == CSP_SEND) {
                __threadfence();
                const unsigned k = ld_acquire_gpu(sent);  // this CTA is the channel's only sender
                while (k - ld_acquire_gpu(recvd) >= static_cast<unsigned>(a.caps[op.arg]))
                    if (csp_clock_ns() - t0 > kWaitNs) {
                        atomicOr(a.err, kErrTimeout);
                        s_stop = 1;
                        break;
                    }
                if (!s_stop) st_release_gpu(sent, k + 1);
            } else {
                const unsigned k = ld_acquire_gpu(recvd);  // this CTA is the channel's only receiver
                while (ld_acquire_gpu(sent) <= k)
                    if (csp_clock_ns() - t0 > kWaitNs) {
                        atomicOr(a.err, kErrTimeout);
                        s_stop = 1;
                        break;
                    }
                __threadfence();
                if (!s_stop) st_release_gpu(recvd, k + 1);
            }
        }
        __syncthreads();
        if (s_stop) break;
    }
}

}  // namespace

int sm_count() {
    static int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

cudaError_t launch_rmsnorm_rows(const TaskBatch& b, int workers, cudaStream_t s) {
    return launch_rows<RmsNormOp>(b, workers, s);
}

cudaError_t launch_softmax_rows(const TaskBatch& b, int workers, cudaStream_t s) {
    return launch_rows<SoftmaxOp>(b, workers, s);
}

int tile_program_max_smem() { return 227 * 1024; }

namespace {

// Matmul stage on CUDA cores: C[M,N] (f32) = A[M,K] . B[K,N] per task, records [oa, ob, oc].  Every output
// accumulates over k in order with one fused multiply-add per step, as the tile program does, so a staged
// kernel reproduces its results bit for bit; A and B may be f16 (exactly widened) or f32.  One BM x BN block of
// one task per CTA iteration (16 x 16 threads; a thread owns the rows h*64 + 4*ty + i and the columns
// g*64 + 4*tx + j, so its shared-memory reads are float4s that no two lanes of a quarter-warp share), k staged
// through shared memory 16 at a time.
constexpr int kSimtBK = 16;

template <int BM, int BN>
__global__ void __launch_bounds__(256) matmul_simt_kernel(TaskBatch b, int M, int N, int K) {
    constexpr int HM = BM / 64, HN = BN / 64;  // 64-row / 64-column halves per thread
    __shared__ __align__(16) float As[kSimtBK][BM + 4];
    __shared__ __align__(16) float Bs[kSimtBK][BN + 4];
    const ParamDesc &A = b.p[0], &B = b.p[1], &C = b.p[2];
    const int bm_n = (M + BM - 1) / BM, bn_n = (N + BN - 1) / BN;
    const int64_t per_task = static_cast<int64_t>(bm_n) * bn_n;
    const int64_t units = b.ntasks * per_task;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const bool a_f32 = A.type == PT_F32, b_f32 = B.type == PT_F32;  // f32 operands: plain loads, no type switch
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int64_t t = u / per_task;
        const int rem = static_cast<int>(u - t * per_task);
        const int m0 = (rem / bn_n) * BM, n0 = (rem % bn_n) * BN;
        const int64_t* rec = b.rec + t * b.stride;
        const int64_t oa = rec[0], ob = rec[1], oc = rec[2];
        float acc[4 * HM][4 * HN];
#pragma unroll
        for (int i = 0; i < 4 * HM; ++i)
#pragma unroll
            for (int j = 0; j < 4 * HN; ++j) acc[i][j] = 0.f;
        // the next k slice's global loads are issued before the current slice's FMAs (registers ra / rb)
        constexpr int NA = kSimtBK * BM / 256, NB = kSimtBK * BN / 256;
        float ra[NA], rb[NB];
        auto fetch = [&](int k0) {
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int e = threadIdx.x + q * 256;
                const int mm = e / kSimtBK, kk = e % kSimtBK;  // consecutive threads: consecutive k of a row of A
                const int r = m0 + mm, kq = k0 + kk;
                float v = 0.f;
                if (r < M && kq < K) {
                    const int64_t off = oa + r * A.s3 + kq * A.s4;
                    if (off >= 0 && off < A.numel_span)
                        v = a_f32 ? __ldg(reinterpret_cast<const float*>(A.base) + off) : load_elem_f(A, off);
                    else atomicOr(b.err, kErrBounds);
                }
                ra[q] = v;
            }
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int e = threadIdx.x + q * 256;
                const int kk = e / BN, nn = e % BN;  // consecutive threads: consecutive n of a row of B
                const int c = n0 + nn, kq = k0 + kk;
                float v = 0.f;
                if (c < N && kq < K) {
                    const int64_t off = ob + kq * B.s3 + c * B.s4;
                    if (off >= 0 && off < B.numel_span)
                        v = b_f32 ? __ldg(reinterpret_cast<const float*>(B.base) + off) : load_elem_f(B, off);
                    else atomicOr(b.err, kErrBounds);
                }
                rb[q] = v;
            }
        };
        fetch(0);
        for (int k0 = 0; k0 < K; k0 += kSimtBK) {
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int e = threadIdx.x + q * 256;
                As[e % kSimtBK][e / kSimtBK] = ra[q];
            }
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int e = threadIdx.x + q * 256;
                Bs[e / BN][e % BN] = rb[q];
            }
            __syncthreads();
            if (k0 + kSimtBK < K) fetch(k0 + kSimtBK);
            const int kn = min(kSimtBK, K - k0);
            for (int kk = 0; kk < kn; ++kk) {
                float av[4 * HM], bv[4 * HN];
#pragma unroll
                for (int h = 0; h < HM; ++h) {
                    const float4 x = *reinterpret_cast<const float4*>(&As[kk][h * 64 + ty * 4]);
                    av[4 * h] = x.x; av[4 * h + 1] = x.y; av[4 * h + 2] = x.z; av[4 * h + 3] = x.w;
                }
#pragma unroll
                for (int g = 0; g < HN; ++g) {
                    const float4 x = *reinterpret_cast<const float4*>(&Bs[kk][g * 64 + tx * 4]);
                    bv[4 * g] = x.x; bv[4 * g + 1] = x.y; bv[4 * g + 2] = x.z; bv[4 * g + 3] = x.w;
                }
#pragma unroll
                for (int i = 0; i < 4 * HM; ++i)
#pragma unroll
                    for (int j = 0; j < 4 * HN; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4 * HM; ++i)
#pragma unroll
            for (int j = 0; j < 4 * HN; ++j) {
                const int r = m0 + (i / 4) * 64 + ty * 4 + (i % 4), c = n0 + (j / 4) * 64 + tx * 4 + (j % 4);
                if (r >= M || c >= N) continue;
                const int64_t off = oc + r * C.s3 + c * C.s4;
                if (off >= 0 && off < C.numel_span) store_elem(C, off, __float_as_uint(acc[i][j]), W_F32);
                else atomicOr(b.err, kErrBounds);
            }
    }
}

template <int BM, int BN>
cudaError_t launch_simt(const TaskBatch& b, int M, int N, int K, int workers, cudaStream_t s) {
    const int64_t units = b.ntasks * ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, matmul_simt_kernel<BM, BN>, 256, 0);
    int64_t blocks = std::min<int64_t>(units, static_cast<int64_t>(std::max(per_sm, 1)) * sm_count());
    if (workers > 0) blocks = std::min<int64_t>(blocks, workers);
    blocks = std::max<int64_t>(blocks, 1);
    matmul_simt_kernel<BM, BN><<<static_cast<unsigned>(blocks), 256, 0, s>>>(b, M, N, K);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_matmul_simt(const TaskBatch& b, int M, int N, int K, int workers, cudaStream_t s) {
    // Measured on B200: a 64-row tile with N >= 128 runs best as 64 x 128 blocks (llama-style MLP, 64 x 512 x 256:
    // 1.02 ms against 1.25 with 64 x 64); 128-row tiles run best as 64 x 64 blocks (attention P.V, 128 x 128 x
    // 1024: 128 x 128 blocks were 14 % slower -- two CTAs per SM hide the element-wise global loads less well)
    if (M < 128 && N >= 128) return launch_simt<64, 128>(b, M, N, K, workers, s);
    return launch_simt<64, 64>(b, M, N, K, workers, s);
}

bool launch_csp_pipeline(const CspArgs& a, int smem_bytes, cudaStream_t s, cudaError_t* err) {
    if (smem_bytes > 48 * 1024 &&
        cudaFuncSetAttribute(csp_pipeline_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, csp_pipeline_kernel, 256, smem_bytes) != cudaSuccess ||
        static_cast<int64_t>(per_sm) * sm_count() < a.nproc || a.nproc < 1) {
        cudaGetLastError();
        return false;
    }
    // cooperative launch: the runtime guarantees that all CTAs are resident together (processes wait on one another)
    CspArgs args = a;
    void* params[] = {&args};
    *err = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(csp_pipeline_kernel), dim3(static_cast<unsigned>(a.nproc)),
                                       dim3(256), params, static_cast<size_t>(smem_bytes), s);
    return true;
}

cudaError_t launch_tile_program(const TaskBatch& b, const TileProgram* prog_dev, int smem_bytes, int workers,
                                cudaStream_t s) {
    if (smem_bytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(tile_program_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return e;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tile_program_kernel, 256, smem_bytes);
    int64_t blocks = std::min<int64_t>(b.ntasks, static_cast<int64_t>(std::max(per_sm, 1)) * sm_count());
    if (workers > 0) blocks = std::min<int64_t>(blocks, workers);
    blocks = std::max<int64_t>(blocks, 1);
    tile_program_kernel<<<static_cast<unsigned>(blocks), 256, smem_bytes, s>>>(b, prog_dev);
    return cudaGetLastError();
}

namespace {

// DType codes of the plan (plan.hpp): F16, BF16, F32, F64, I8, I16, I32, I64, U8, U16, U32, U64, Bool.
__device__ __forceinline__ uint64_t slot_value(const char* p, int t) {
    switch (t) {
        case 2: return static_cast<uint64_t>(static_cast<int64_t>(*reinterpret_cast<const float*>(p)));
        case 3: return static_cast<uint64_t>(static_cast<int64_t>(*reinterpret_cast<const double*>(p)));
        case 4: return static_cast<uint64_t>(static_cast<int64_t>(*reinterpret_cast<const int8_t*>(p)));
        case 5: return static_cast<uint64_t>(static_cast<int64_t>(*reinterpret_cast<const int16_t*>(p)));
        case 6: return static_cast<uint64_t>(static_cast<int64_t>(*reinterpret_cast<const int32_t*>(p)));
        case 7: case 11: return *reinterpret_cast<const uint64_t*>(p);
        case 8: case 12: return *reinterpret_cast<const uint8_t*>(p);
        case 9: return *reinterpret_cast<const uint16_t*>(p);
        case 10: return *reinterpret_cast<const uint32_t*>(p);
        default: return 0;
    }
}

__global__ void select_scalars_kernel(int64_t* rec, int stride, int scalar_pos, const uint64_t* rows, int64_t nrows,
                                      int row_words, const int* tree, int nconds, int nscalars, const char* src,
                                      int src_type, int elem_bytes, int64_t src_span, int* err) {
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < nrows;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint64_t* row = rows + r * row_words;
        const int64_t t = static_cast<int64_t>(row[0]), off = static_cast<int64_t>(row[1]);
        const uint64_t mask = row[2];
        if (off < 0 || off >= src_span) {
            atomicOr(err, kErrBounds);
            continue;
        }
        const uint64_t v = slot_value(src + off * elem_bytes, src_type);
        int code = 0;
        for (int guard = 0; code >= 0 && guard < nconds; ++guard) {
            const int* c = tree + 4 * code;
            const uint64_t o = row[3 + code];
            const uint64_t x = c[1] ? v : o, y = c[1] ? o : v;
            const bool sg = (mask >> code) & 1ull;
            const int64_t xs = static_cast<int64_t>(x), ys = static_cast<int64_t>(y);
            bool res = false;
            switch (c[0]) {
                case 0: res = sg ? xs < ys : x < y; break;
                case 1: res = sg ? xs <= ys : x <= y; break;
                case 2: res = sg ? xs > ys : x > y; break;
                case 3: res = sg ? xs >= ys : x >= y; break;
                case 4: res = x == y; break;
                default: res = x != y; break;
            }
            code = res ? c[2] : c[3];
        }
        if (code >= 0) {
            atomicOr(err, kErrShape);
            continue;
        }
        const uint64_t* leaf = row + 3 + nconds + static_cast<int64_t>(~code) * nscalars;
        for (int j = 0; j < nscalars; ++j) rec[t * stride + scalar_pos + j] = static_cast<int64_t>(leaf[j]);
    }
}

}  // namespace

cudaError_t launch_select_scalars(int64_t* rec, int stride, int scalar_pos, const uint64_t* rows, int64_t nrows,
                                  int row_words, const int* tree, int nconds, int nscalars, const void* src,
                                  int src_type, int64_t src_span, int* err, cudaStream_t s) {
    if (nrows <= 0) return cudaSuccess;
    static const int bytes[13] = {2, 2, 4, 8, 1, 2, 4, 8, 1, 2, 4, 8, 1};
    if (src_type < 2 || src_type > 12) return cudaErrorInvalidValue;  // f16 / bf16 slot sources are not read
    const int blocks = static_cast<int>(std::min<int64_t>((nrows + 255) / 256, 1024));
    select_scalars_kernel<<<blocks, 256, 0, s>>>(rec, stride, scalar_pos, rows, nrows, row_words, tree, nconds,
                                                 nscalars, static_cast<const char*>(src), src_type, bytes[src_type],
                                                 src_span, err);
    return cudaGetLastError();
}


namespace {
__global__ void expand_records_kernel(int64_t* rec, int stride, int64_t n, const int64_t* bd, const int32_t* vars) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * stride) return;
    const int64_t t = i / stride;
    const int w = static_cast<int>(i % stride);
    const int64_t var = vars ? static_cast<int64_t>(vars[t]) : t;
    rec[i] = bd[w] + var * bd[stride + w];
}
}  // namespace

cudaError_t launch_expand_records(int64_t* rec, int stride, int64_t n, const int64_t* base_delta, const int32_t* vars,
                                  cudaStream_t s) {
    const int64_t total = n * stride;
    if (total <= 0) return cudaSuccess;
    const int64_t blocks = (total + 255) / 256;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    expand_records_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(rec, stride, n, base_delta, vars);
    return cudaGetLastError();
}

}  // namespace ptowsp::dev
