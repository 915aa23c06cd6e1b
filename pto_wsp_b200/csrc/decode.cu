// Built-in paged GQA decode and top-k selection (config 5).
//
// paged_decode_gqa -- one task = (request r, kv head h): the G query heads
// sharing KV head h attend over the request's L = kv_len[r] cached tokens,
// found through the page table (page p of the request holds tokens
// [16p, 16p+16)).  Math as the reference toy kernel
// (examples/flashinfer_decode/pto_wsp_impl.py:38-54, golden.py:7-12):
// softmax(q K^T / sqrt(D)) V, f32 softmax, f16 output (round to nearest even).
//
// HBM-bound: every K/V byte is used for 2*G FLOP (G = 4: ~4 FLOP/B).
// Split-KV: each task is cut into chunks, one CTA each; empty chunks exit at
// once.  The TMA kernel takes 1536 tokens per chunk (the best of 1024 / 1536 /
// 2048 measured on config 4) unless the launch has so few tasks that long
// chunks would leave SMs with one CTA each (a rank's share of config 4 on
// eight GPUs): then shorter ones, down to 512 (decode_chunk_tokens).  The
// CUDA-core kernel takes 512.  For the usual pool layout (16-token pages, 16-byte
// aligned rows) a TMA producer warp streams the pages and four consumer warps
// run both contractions of a page on warp-level MMAs (paged_decode_tma_kernel,
// below); the last CTA of a task merges its chunk partials.  Other layouts use
// a CUDA-core kernel (scores lane-per-token, P.V lane-per-dimension) that
// writes (max, sum, acc[G][128]) per chunk, merged by a second kernel with
// the log-sum-exp rule.  Both store f16.
//
// topk_select -- indices of the K largest of N scores, ordered by score
// descending, ties by lower index (examples/deepseek_lightning_indexer/
// golden.py:6-25).  One CTA per row: the row is staged in shared memory as
// order-preserving 32-bit keys, a 4-pass 8-bit radix select finds the K-th
// key, the K winners (ties at the threshold taken in index order) are
// gathered and bitonic-sorted by (key desc, index asc).  Bit-exact by
// construction.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "device.hpp"
#include "tc_common.cuh"

namespace ptowsp::dev {

namespace {

#ifndef PTOWSP_DECODE_CHUNK
#define PTOWSP_DECODE_CHUNK 1536
#endif
#ifndef PTOWSP_DECODE_STAGES
#define PTOWSP_DECODE_STAGES 8
#endif
constexpr int kChunk = PTOWSP_DECODE_CHUNK;  // longest split-KV chunk of the TMA kernel (tokens)
constexpr int kFbChunk = 512;                // tokens per split-KV chunk of the CUDA-core kernel
constexpr int kMinChunk = 512;               // shortest: the scratch of every launch is sized for 512-token chunks
static_assert(kChunk % 16 == 0 && kMinChunk % 16 == 0 && kMinChunk <= kChunk && kMinChunk >= std::min(kChunk, kFbChunk),
              "chunks hold whole 16-token pages, and no chunk is shorter than the one the scratch is sized for");
constexpr int kDecThreads = 128;  // 4 warps
constexpr int kHeadDim = 128;

// Sum 16 per-lane values over the 16 lanes of a half-warp so that lane l ends
// up holding the total of value (l & 15): each stage halves the values a lane
// carries, so 16 sums cost 15 shuffles instead of 4 x 16.
__device__ __forceinline__ float halfwarp_transpose_reduce(float (&v)[16], int lane) {
#pragma unroll
    for (int n = 16, o = 8; n > 1; n >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = up ? v[i] : v[i + n / 2];
            const float keep = up ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    return v[0];
}

__device__ __forceinline__ void h8_to_f8(const uint4& r, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const float2 x = __half22float2(h[u]);
        f[2 * u] = x.x;
        f[2 * u + 1] = x.y;
    }
}

// One CTA = one 512-token chunk of one (request, kv head) task.  A half-warp
// owns one token at a time, each of its 16 lanes 8 of the 128 head dims
// (one 16-byte load per K or V row); STEPS = 16/G tokens per half-warp are in
// flight per iteration.
template <int G>
__global__ void __launch_bounds__(kDecThreads) paged_decode_chunk_kernel(TaskBatch b, int page_size, int chunks,
                                                                        float* __restrict__ scratch) {
    constexpr int STEPS = 16 / G;
    __shared__ __align__(16) float p_s[kFbChunk][G];  // scores, then probabilities, token-major
    __shared__ float red_s[4][G][kHeadDim];
    __shared__ float stat_s[2][4][G];

    const int64_t task = blockIdx.x / chunks;
    const int chunk = blockIdx.x % chunks;
    if (task >= b.ntasks) return;
    const int64_t* rec = b.rec + task * b.stride;
    const ParamDesc& Pq = b.p[0];
    const ParamDesc& Pk = b.p[1];
    const ParamDesc& Pv = b.p[2];
    const ParamDesc& Ppt = b.p[3];
    const ParamDesc& Pl = b.p[4];
    const int h = static_cast<int>(rec[b.nparams + 1]);
    int32_t L = reinterpret_cast<const int32_t*>(Pl.base)[rec[4]];
    if (L > Ppt.cols * page_size) {  // more tokens than the page table row can address
        if (chunk == 0) atomicOr(b.err, kErrShape);
        L = Ppt.cols * page_size;
    }
    const int t0 = chunk * kFbChunk;
    if (t0 >= L) return;  // empty chunk (also L <= 0: the merge kernel writes zeros)
    const int n = min(kFbChunk, L - t0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hl = lane & 15;        // lane within the half-warp: head dims [8*hl, 8*hl + 8)
    const int hw = tid >> 4;         // half-warp id, 0..7
    const float scale = 1.0f / sqrtf(static_cast<float>(kHeadDim));

    // q slice of this lane (pre-scaled by 1/sqrt(D)) in registers
    float qf[G][8];
    {
        const __half* q = reinterpret_cast<const __half*>(Pq.base) + rec[0];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const uint4 r = *reinterpret_cast<const uint4*>(q + g * Pq.s3 + hl * 8);
            h8_to_f8(r, qf[g]);
#pragma unroll
            for (int j = 0; j < 8; ++j) qf[g][j] *= scale;
        }
    }
    const int32_t* pt = reinterpret_cast<const int32_t*>(Ppt.base) + rec[3];
    const int64_t max_page_k = (Pk.numel_span - (int64_t)(page_size - 1) * Pk.s4 - h * kHeadDim - kHeadDim) / Pk.s3;
    const int64_t max_page_v = (Pv.numel_span - (int64_t)(page_size - 1) * Pv.s4 - h * kHeadDim - kHeadDim) / Pv.s3;
    const int64_t max_page = min(max_page_k, max_page_v);
    const __half* kb = reinterpret_cast<const __half*>(Pk.base) + h * kHeadDim + hl * 8;
    const __half* vb = reinterpret_cast<const __half*>(Pv.base) + h * kHeadDim + hl * 8;
    auto page_of = [&](int tok, bool flag) -> int64_t {
        int64_t page = pt[static_cast<int64_t>(tok / page_size) * Ppt.s4];
        if (page < 0 || page > max_page) {
            if (flag) atomicOr(b.err, kErrBounds);
            page = 0;  // read page 0 harmlessly; the run reports the error
        }
        return page;
    };

    // ---- scores: half-warp per token, STEPS tokens per half-warp in flight ----
    const int my_g = hl % G;  // after the transpose reduction a lane always holds query my_g
    float mymax = -INFINITY;
    for (int base = 0; base < n; base += 8 * STEPS) {
        uint4 raw[STEPS];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const int i = base + st * 8 + hw;
            raw[st] = make_uint4(0, 0, 0, 0);
            if (i < n) {
                const int tok = t0 + i;
                const int64_t page = page_of(tok, true);
                raw[st] = __ldg(reinterpret_cast<const uint4*>(kb + page * Pk.s3 + (tok % page_size) * Pk.s4));
            }
        }
        float part[16];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            float kf[8];
            h8_to_f8(raw[st], kf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float a = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) a = fmaf(kf[j], qf[g][j], a);
                part[st * G + g] = a;
            }
        }
        const float tot = halfwarp_transpose_reduce(part, hl);  // value index hl = st * G + g
        const int i = base + (hl / G) * 8 + hw;
        if (i < n) {
            p_s[i][my_g] = tot;
            mymax = fmaxf(mymax, tot);
        }
    }
    // ---- chunk max ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float m = my_g == g ? mymax : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) stat_s[0][warp][g] = m;
    }
    __syncthreads();
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = fmaxf(fmaxf(stat_s[0][0][g], stat_s[0][1][g]), fmaxf(stat_s[0][2][g], stat_s[0][3][g]));
    // ---- p = exp(s - m), chunk sum ----
    float lsum[G];
#pragma unroll
    for (int g = 0; g < G; ++g) lsum[g] = 0.f;
    for (int i = tid; i < n; i += kDecThreads) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float pv = expf(p_s[i][g] - mx[g]);
            p_s[i][g] = pv;
            lsum[g] += pv;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float sm = lsum[g];
        for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        if (lane == 0) stat_s[1][warp][g] = sm;
    }
    __syncthreads();
    // ---- P.V: half-warp per token, lane per 8 head dims ----
    float acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
    constexpr int PV_STEPS = 4;
    for (int base = 0; base < n; base += 8 * PV_STEPS) {
        uint4 raw[PV_STEPS];
#pragma unroll
        for (int st = 0; st < PV_STEPS; ++st) {
            const int i = base + st * 8 + hw;
            raw[st] = make_uint4(0, 0, 0, 0);
            if (i < n) {
                const int tok = t0 + i;
                const int64_t page = page_of(tok, false);
                raw[st] = __ldg(reinterpret_cast<const uint4*>(vb + page * Pv.s3 + (tok % page_size) * Pv.s4));
            }
        }
#pragma unroll
        for (int st = 0; st < PV_STEPS; ++st) {
            const int i = base + st * 8 + hw;
            if (i < n) {
                float vf[8];
                h8_to_f8(raw[st], vf);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg = p_s[i][g];
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(pg, vf[j], acc[g][j]);
                }
            }
        }
    }
    // the two half-warps of a warp hold different tokens: add them, then one row per warp
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], 16);
    if (lane < 16) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < 8; ++j) red_s[warp][g][hl * 8 + j] = acc[g][j];
    }
    __syncthreads();
    // ---- partial (max, sum, acc) -> scratch ----
    float* part_out = scratch + static_cast<int64_t>(blockIdx.x) * (G * kHeadDim + 2 * G);
    for (int e = tid; e < G * kHeadDim; e += kDecThreads) {
        const int g = e / kHeadDim, d = e % kHeadDim;
        part_out[e] = (red_s[0][g][d] + red_s[1][g][d]) + (red_s[2][g][d] + red_s[3][g][d]);
    }
    if (tid < G) {
        float m = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (g == tid) m = mx[g];  // static register indexing
        part_out[G * kHeadDim + tid] = m;
        part_out[G * kHeadDim + G + tid] = stat_s[1][0][tid] + stat_s[1][1][tid] + stat_s[1][2][tid] + stat_s[1][3][tid];
    }
}

// ---------------------------------------------------------------------------
// TMA + warp-MMA variant (the default for contiguous 16-token page pools).
//
// A producer warp streams, page by page, the task's head slice of K and V
// into an 8-stage shared-memory ring: per page four TMA boxes of 16 tokens x
// 64 dims (2 KB each, 128-byte swizzled so the fragment loads below are free
// of bank conflicts).  Four consumer warps each own every 4th page of the
// chunk.  Per page a warp computes S^T = K Q^T (16 tokens x 8 queries, the G
// real queries padded to 8) with 8 m16n8k16 f16 MMAs, updates its online
// softmax (base-2, scores pre-scaled by log2(e)/sqrt(D)), and accumulates
// O^T += V^T P^T (128 dims x 8 queries) with 8 more; P goes through a
// 256-byte per-warp buffer to change from accumulator to operand layout.
// The contraction per page (16 tokens x G <= 8 queries) is far below the
// 64/128-row minimum of a tcgen05 tile, so warp-level MMAs are the tool here;
// they cut the per-page instruction count about eightfold against CUDA-core
// dot products, which leaves the kernel bound by HBM, not issue.
//
// Chunks of one task are merged by the last of its CTAs to finish (a
// per-task arrival counter, zeroed before each launch): partials go to
// scratch, the last arriving CTA combines them in chunk order (so the result
// does not depend on which CTA came last) and stores f16.  A task with one
// chunk stores directly.  Bounded waits; the producer drains its copies
// before the CTA exits; every CTA that has work arrives on its counter, also
// after a timed-out wait.
// ---------------------------------------------------------------------------

constexpr int kMmaStages = PTOWSP_DECODE_STAGES;
constexpr int kMmaConsumers = 4;
constexpr int kMmaThreads = 32 * (kMmaConsumers + 1);
// Consumer warp w takes pages w, w + 4, ...; with a stage count that is a
// multiple of the consumer count every stage is always read by the same warp,
// which has finished the stage's previous page before it waits on the stage
// again -- so a parity wait can never see the phase before the one it wants.
static_assert(kMmaStages % kMmaConsumers == 0, "each ring stage must belong to one consumer warp");
constexpr int kMmaPage = 16;
constexpr int kHalfBox = kMmaPage * 64 * 2;   // 16 tokens x 64 dims f16 = 2 KB
constexpr int kStageBytes = 4 * kHalfBox;     // K lo, K hi, V lo, V hi
constexpr int kRingBytes = kMmaStages * kStageBytes;
constexpr int kBarOffset = kRingBytes;  // full[S], empty[S], abort, last flag
constexpr int kPageIdsOffset = kBarOffset + ((16 * kMmaStages + 8 + 127) / 128) * 128;  // the chunk's page ids
// per-warp P as two f16 parts (high, then low), 16 tok x 8 q each
constexpr int kPbufOffset = kPageIdsOffset + ((kChunk / 16 * 4 + 127) / 128) * 128;
constexpr int kMmaSmemBytes = kPbufOffset + kMmaConsumers * 512 + 1024;  // + 1024-byte alignment slack

template <int G>
struct MmaCombine {  // per consumer warp, aliased onto the ring once every page has been consumed
    static constexpr int STRIDE = 2 * G + G * kHeadDim;  // m[G], l[G], acc[G][128] (floats)
    static_assert(kMmaConsumers * STRIDE * 4 <= kRingBytes, "combine area fits in the ring");
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// D (16x8 f32) += A (16x16 f16, row) * B (16x8 f16, col)
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// The rounding remainder of pack_h2: x - f16(x), itself rounded to f16.  P = high + low carries ~22 bits of each
// probability into the P.V contraction (f16 alone carries 11, which shows as a 5e-4 relative error of the terms).
__device__ __forceinline__ uint32_t pack_h2_rem(float lo, float hi) {
    return pack_h2(lo - __half2float(__float2half_rn(lo)), hi - __half2float(__float2half_rn(hi)));
}
// Byte offset of (token, dim) inside one page's 128-byte-swizzled K or V slice.
__device__ __forceinline__ uint32_t swz(int tok, int d) {
    return static_cast<uint32_t>((d >> 6) * kHalfBox + tok * 128 + ((((d & 63) >> 3) ^ (tok & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kMmaThreads) paged_decode_tma_kernel(const __grid_constant__ CUtensorMap mk,
                                                                     const __grid_constant__ CUtensorMap mv, TaskBatch b,
                                                                     int chunks, int chunk_tokens,
                                                                     float* __restrict__ partials,
                                                                     unsigned* __restrict__ arrivals) {
    using CB = MmaCombine<G>;
    extern __shared__ uint8_t dsm_raw[];
    uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(dsm + kBarOffset);
    uint64_t* empty = full + kMmaStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMmaStages);
    volatile int* last_flag = abort_flag + 1;

    const int64_t task = blockIdx.x / chunks;
    const int chunk = blockIdx.x % chunks;
    if (task >= b.ntasks) return;
    const int64_t* rec = b.rec + task * b.stride;
    const ParamDesc& Pq = b.p[0];
    const ParamDesc& Ppt = b.p[3];
    const ParamDesc& Pl = b.p[4];
    const int h = static_cast<int>(rec[b.nparams + 1]);
    int32_t L = reinterpret_cast<const int32_t*>(Pl.base)[rec[4]];
    if (L > Ppt.cols * kMmaPage) {
        if (chunk == 0 && threadIdx.x == 0) atomicOr(b.err, kErrShape);
        L = Ppt.cols * kMmaPage;
    }
    const int t0 = chunk * chunk_tokens;
    if (L <= 0 && chunk == 0) {  // no cached tokens: the output is zero
        __half* out = reinterpret_cast<__half*>(b.p[5].base) + rec[5];
        for (int e = threadIdx.x; e < G * kHeadDim; e += kMmaThreads)
            out[(e / kHeadDim) * b.p[5].s3 + e % kHeadDim] = __float2half_rn(0.f);
        return;
    }
    if (t0 >= L) return;  // whole CTA leaves together: no barrier has been touched
    const int nch = (L + chunk_tokens - 1) / chunk_tokens;
    const int n = min(chunk_tokens, L - t0);
    const int npages = (n + kMmaPage - 1) / kMmaPage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int st = 0; st < kMmaStages; ++st) {
            tc::mbar_init(tc::smem_u32(&full[st]), 1);
            tc::mbar_init(tc::smem_u32(&empty[st]), 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // consumer state: lane = (g = lane / 4, tq = lane % 4); this lane's queries are 2tq and 2tq+1
    const int g = lane >> 2, tq = lane & 3;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int k = 0; k < 4; ++k) o[mt][k] = 0.f;

    if (warp == kMmaConsumers) {
        // ---------------- producer ----------------
        // the chunk's page ids are fetched at once by the whole warp and handed to lane 0 in shared memory
        int* page_ids = reinterpret_cast<int*>(dsm + kPageIdsOffset);
        {
            const int32_t* pt = reinterpret_cast<const int32_t*>(Ppt.base) + rec[3];
            const int64_t max_page = b.p[1].numel_span / (int64_t(kMmaPage) * b.p[1].s4) - 1;
            for (int i = lane; i < npages; i += 32) {
                int64_t page = pt[static_cast<int64_t>(t0 / kMmaPage + i) * Ppt.s4];
                if (page < 0 || page > max_page) {
                    atomicOr(b.err, kErrBounds);
                    page = 0;
                }
                page_ids[i] = static_cast<int>(page);
            }
            __syncwarp();
        }
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < npages && !*abort_flag; ++j) {
                const int st = j % kMmaStages;
                if (j >= kMmaStages &&
                    !tc::mbar_wait(tc::smem_u32(&empty[st]), ((j / kMmaStages) - 1) & 1, abort_flag, b.err))
                    break;
                const int64_t page = page_ids[j];
                const uint32_t fb = tc::smem_u32(&full[st]);
                tc::mbar_expect_tx(fb, kStageBytes);
                const uint32_t dst = tc::smem_u32(dsm + st * kStageBytes);
                const int32_t y = static_cast<int32_t>(page * kMmaPage);
                tc::tma_load_2d(dst, &mk, h * kHeadDim, y, fb);
                tc::tma_load_2d(dst + kHalfBox, &mk, h * kHeadDim + 64, y, fb);
                tc::tma_load_2d(dst + 2 * kHalfBox, &mv, h * kHeadDim, y, fb);
                tc::tma_load_2d(dst + 3 * kHalfBox, &mv, h * kHeadDim + 64, y, fb);
                ++issued;
            }
            // drain: the last copy into each stage has landed
            const uint64_t start = tc::globaltimer();
            for (int j = max(0, issued - kMmaStages); j < issued; ++j)
                while (!tc::mbar_try_wait(tc::smem_u32(&full[j % kMmaStages]), (j / kMmaStages) & 1))
                    if (tc::globaltimer() - start > tc::kTimeoutNs) {
                        atomicOr(b.err, kErrTimeout);
                        break;
                    }
        }
    } else {
        // ---------------- consumers ----------------
        // Q^T as the B operand of S^T = K Q^T: b0 = Q[g][16kk + 2tq .. +1], b1 = Q[g][16kk + 2tq + 8 .. +9]
        uint32_t qb[8][2];
        {
            const __half* q = reinterpret_cast<const __half*>(Pq.base) + rec[0] + static_cast<int64_t>(g) * Pq.s3;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                qb[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(q + 16 * kk + 2 * tq) : 0u;
                qb[kk][1] = g < G ? *reinterpret_cast<const uint32_t*>(q + 16 * kk + 2 * tq + 8) : 0u;
            }
        }
        const float sc = 1.4426950408889634f / sqrtf(static_cast<float>(kHeadDim));  // log2(e) / sqrt(D)
        uint8_t* pbuf = dsm + kPbufOffset + warp * 512;  // [high part | low part]
        const uint32_t pbuf_u = tc::smem_u32(pbuf);
        const int mi = lane >> 3, r8 = lane & 7;
        for (int j = warp; j < npages && !*abort_flag; j += kMmaConsumers) {
            const int st = j % kMmaStages;
            if (!tc::mbar_wait(tc::smem_u32(&full[st]), (j / kMmaStages) & 1, abort_flag, b.err)) break;
            const uint32_t kb = tc::smem_u32(dsm + st * kStageBytes);
            const uint32_t vb = kb + 2 * kHalfBox;
            const int valid = min(kMmaPage, n - j * kMmaPage);
            // S^T (16 tokens x 8 queries): A = K rows (token-major), 8 k-steps over the head dims
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t a[4];
                ldsm_x4(kb + swz(r8 + 8 * (mi & 1), 16 * kk + 8 * (mi >> 1)), a);
                mma_16816(s, a, qb[kk][0], qb[kk][1]);
            }
            // s[0], s[1]: token g, queries 2tq, 2tq+1; s[2], s[3]: token g+8
            const float s00 = g < valid ? s[0] * sc : -INFINITY;
            const float s01 = g < valid ? s[1] * sc : -INFINITY;
            const float s10 = g + 8 < valid ? s[2] * sc : -INFINITY;
            const float s11 = g + 8 < valid ? s[3] * sc : -INFINITY;
            float x0 = fmaxf(s00, s10), x1 = fmaxf(s01, s11);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
                x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
            }
            const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);  // finite: token 0 of a page is always valid
            const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
            const float p00 = exp2f(s00 - mn0), p10 = exp2f(s10 - mn0);
            const float p01 = exp2f(s01 - mn1), p11 = exp2f(s11 - mn1);
            l0 = fmaf(l0, c0, p00 + p10);
            l1 = fmaf(l1, c1, p01 + p11);
            m0 = mn0;
            m1 = mn1;
            if (__any_sync(0xffffffffu, c0 != 1.f || c1 != 1.f)) {
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    o[mt][0] *= c0;
                    o[mt][1] *= c1;
                    o[mt][2] *= c0;
                    o[mt][3] *= c1;
                }
            }
            // P (token-major, 16 B per token row) -> B operand P^T via a transposing fragment load, as a high
            // and a low f16 part; both multiply the same V^T fragments
            *reinterpret_cast<uint32_t*>(pbuf + g * 16 + tq * 4) = pack_h2(p00, p01);
            *reinterpret_cast<uint32_t*>(pbuf + (g + 8) * 16 + tq * 4) = pack_h2(p10, p11);
            *reinterpret_cast<uint32_t*>(pbuf + 256 + g * 16 + tq * 4) = pack_h2_rem(p00, p01);
            *reinterpret_cast<uint32_t*>(pbuf + 256 + (g + 8) * 16 + tq * 4) = pack_h2_rem(p10, p11);
            __syncwarp();
            uint32_t pb0, pb1, pl0, pl1;
            ldsm_x2_t(pbuf_u + (lane & 15) * 16, pb0, pb1);
            ldsm_x2_t(pbuf_u + 256 + (lane & 15) * 16, pl0, pl1);
            // O^T (128 dims x 8 queries) += V^T P^T: A = V^T through transposing loads of the token-major rows
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                uint32_t a[4];
                ldsm_x4_t(vb + swz(r8 + 8 * (mi >> 1), 16 * mt + 8 * (mi & 1)), a);
                mma_16816(o[mt], a, pl0, pl1);
                mma_16816(o[mt], a, pb0, pb1);
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&empty[st]));
        }
        // per-lane sums of the same query live in the 8 lanes of equal tq
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, off);
            l1 += __shfl_xor_sync(0xffffffffu, l1, off);
        }
    }
    __syncthreads();  // every page consumed and every copy landed: the ring is free for the combine area
    if (warp < kMmaConsumers) {
        float* cw = reinterpret_cast<float*>(dsm) + warp * CB::STRIDE;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int q = 2 * tq + k;
            if (q < G) {
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    cw[2 * G + q * kHeadDim + 16 * mt + g] = o[mt][k];
                    cw[2 * G + q * kHeadDim + 16 * mt + g + 8] = o[mt][2 + k];
                }
                if (g == 0) {
                    cw[q] = k ? m1 : m0;
                    cw[G + q] = k ? l1 : l0;
                }
            }
        }
    }
    __syncthreads();
    // ---- combine the consumer warps (log-sum-exp, base 2) ----
    const float* cw0 = reinterpret_cast<const float*>(dsm);
    const int pstride = G * kHeadDim + 2 * G;
    __half* out = reinterpret_cast<__half*>(b.p[5].base) + rec[5];
    const int64_t os3 = b.p[5].s3;
    float* part = partials + static_cast<int64_t>(blockIdx.x) * pstride;
    for (int e = threadIdx.x; e < G * kHeadDim + G; e += kMmaThreads) {
        const int gq = e < G * kHeadDim ? e / kHeadDim : e - G * kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kMmaConsumers; ++w) M = fmaxf(M, cw0[w * CB::STRIDE + gq]);
        float a = 0.f, lt = 0.f;
#pragma unroll
        for (int w = 0; w < kMmaConsumers; ++w) {
            const float mw = cw0[w * CB::STRIDE + gq];
            if (mw != -INFINITY) {
                const float f = exp2f(mw - M);
                if (e < G * kHeadDim) a = fmaf(cw0[w * CB::STRIDE + 2 * G + e], f, a);
                lt = fmaf(cw0[w * CB::STRIDE + G + gq], f, lt);
            }
        }
        if (nch == 1) {
            if (e < G * kHeadDim) out[gq * os3 + e % kHeadDim] = __float2half_rn(a / lt);
        } else if (e < G * kHeadDim) {
            part[e] = a;
        } else {
            part[G * kHeadDim + gq] = M;
            part[G * kHeadDim + G + gq] = lt;
        }
    }
    if (nch == 1) return;
    // ---- the last CTA of the task to arrive merges its chunks ----
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *last_flag = atomicAdd(&arrivals[task], 1u) == static_cast<unsigned>(nch - 1);
    __syncthreads();
    if (!*last_flag) return;
    __threadfence();
    const float* base = partials + task * chunks * static_cast<int64_t>(pstride);
    // The chunks' maxima and denominators go through shared memory once (the upper half of the ring, free now):
    // per query the running maximum, each chunk's weight exp2(m_c - M) and the denominator; then every output
    // element issues its chunks' loads together.  Same operations in the same order as a per-element loop.
    static_assert(kMmaConsumers * CB::STRIDE * 4 <= kRingBytes / 2, "merge scratch above the combine area");
    float* mw = reinterpret_cast<float*>(dsm + kRingBytes / 2);  // [nch][G] weights, [nch][G] sums, M[G], den[G]
    if ((2 * nch + 2) * G * static_cast<int>(sizeof(float)) <= kRingBytes / 2) {
        float* lsum = mw + nch * G;
        float* Mq = lsum + nch * G;
        float* Dq = Mq + G;
        for (int i = threadIdx.x; i < nch * G; i += kMmaThreads) {
            const int c = i / G, gq = i - c * G;
            mw[i] = __ldcg(base + c * pstride + G * kHeadDim + gq);
            lsum[i] = __ldcg(base + c * pstride + G * kHeadDim + G + gq);
        }
        __syncthreads();
        if (threadIdx.x < G) {
            const int gq = threadIdx.x;
            float M = -INFINITY;
            for (int c = 0; c < nch; ++c) M = fmaxf(M, mw[c * G + gq]);
            float den = 0.f;
            for (int c = 0; c < nch; ++c) {
                const float mc = mw[c * G + gq];
                float w = -1.f;  // chunk without a finite maximum: skipped
                if (mc != -INFINITY) {
                    w = exp2f(mc - M);
                    den = fmaf(lsum[c * G + gq], w, den);
                }
                mw[c * G + gq] = w;
            }
            Mq[gq] = M;
            Dq[gq] = den;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < G * kHeadDim; e += kMmaThreads) {
            const int gq = e / kHeadDim;
            float num = 0.f;
            for (int c0 = 0; c0 < nch; c0 += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = c0 + j < nch ? __ldcg(base + (c0 + j) * pstride + e) : 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (c0 + j < nch) {
                        const float w = mw[(c0 + j) * G + gq];
                        if (w >= 0.f) num = fmaf(v[j], w, num);
                    }
                }
            }
            out[gq * os3 + e % kHeadDim] = __float2half_rn(num / Dq[gq]);
        }
        return;
    }
    for (int e = threadIdx.x; e < G * kHeadDim; e += kMmaThreads) {  // very long requests: per element
        const int gq = e / kHeadDim;
        float M = -INFINITY;
        for (int c = 0; c < nch; ++c) M = fmaxf(M, __ldcg(base + c * pstride + G * kHeadDim + gq));
        float num = 0.f, den = 0.f;
        for (int c = 0; c < nch; ++c) {
            const float mc = __ldcg(base + c * pstride + G * kHeadDim + gq);
            if (mc == -INFINITY) continue;
            const float w = exp2f(mc - M);
            num = fmaf(__ldcg(base + c * pstride + e), w, num);
            den = fmaf(__ldcg(base + c * pstride + G * kHeadDim + G + gq), w, den);
        }
        out[gq * os3 + e % kHeadDim] = __float2half_rn(num / den);
    }
}

template <int G>
__global__ void __launch_bounds__(kDecThreads) paged_decode_merge_kernel(TaskBatch b, int page_size, int chunks,
                                                                        const float* __restrict__ scratch) {
    const int64_t task = blockIdx.x;
    if (task >= b.ntasks) return;
    const int64_t* rec = b.rec + task * b.stride;
    const int32_t L = min(reinterpret_cast<const int32_t*>(b.p[4].base)[rec[4]], b.p[3].cols * page_size);
    __half* out = reinterpret_cast<__half*>(b.p[5].base) + rec[5];
    const int64_t os3 = b.p[5].s3;
    const int nch = L > 0 ? min(chunks, (L + kFbChunk - 1) / kFbChunk) : 0;
    const int stride = G * kHeadDim + 2 * G;
    const float* base = scratch + task * chunks * static_cast<int64_t>(stride);
    for (int e = threadIdx.x; e < G * kHeadDim; e += kDecThreads) {
        const int g = e / kHeadDim, d = e % kHeadDim;
        float M = -INFINITY;
        for (int c = 0; c < nch; ++c) M = fmaxf(M, base[c * stride + G * kHeadDim + g]);
        float num = 0.f, den = 0.f;
        for (int c = 0; c < nch; ++c) {
            const float w = expf(base[c * stride + G * kHeadDim + g] - M);
            num = fmaf(base[c * stride + e], w, num);
            den = fmaf(base[c * stride + G * kHeadDim + G + g], w, den);
        }
        out[g * os3 + d] = __float2half_rn(nch > 0 ? num / den : 0.f);
    }
}

int decode_chunks(const TaskBatch& b, int page_size, int chunk_tokens) {
    const int64_t max_tokens = static_cast<int64_t>(b.p[3].cols) * page_size;
    return static_cast<int>(std::max<int64_t>(1, (max_tokens + chunk_tokens - 1) / chunk_tokens));
}

bool decode_tma_ok(const TaskBatch& b, int page_size) {
    const ParamDesc& K = b.p[1];
    const ParamDesc& V = b.p[2];
    return page_size == kMmaPage && K.s3 == kMmaPage * K.s4 && V.s3 == kMmaPage * V.s4 && K.s4 == V.s4 &&
           K.s4 % 64 == 0 && K.s4 >= kHeadDim && b.p[0].s3 % 2 == 0 &&
           ((reinterpret_cast<uintptr_t>(K.base) | reinterpret_cast<uintptr_t>(V.base)) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(b.p[0].base) & 3) == 0;
}

// Scratch of one decode launch: [arrival counters, one per task, 256-byte padded | chunk partials].
size_t decode_arrivals_bytes(int64_t ntasks) { return (static_cast<size_t>(ntasks) * sizeof(unsigned) + 255) & ~size_t(255); }

// Tokens per chunk of the TMA kernel: `requested` (a multiple of 16 in [kMinChunk, kChunk]) when it is not 0;
// otherwise the longest of 1536 / 1024 / 768 / 512 that still gives the launch at least 1.5 chunks with work per
// SM, counting half of each task's longest possible length as its mean.  Shorter chunks only pay when the long ones
// leave SMs with a single CTA (one CTA's 8-page ring cannot draw an SM's share of HBM); above that their extra
// CTAs and merges cost more than the shorter tail gains.  Measured on config-4 request mixes (ms per launch, chunk
// 512 / 768 / 1024 / 1536): 64 requests 0.207 / 0.196 / 0.190 / 0.188, 32 requests 0.115 / 0.112 / 0.108 / 0.107,
// 16 requests 0.067 / 0.063 / 0.068 / 0.054, 8 requests 0.042 / 0.034 / 0.038 / 0.047 -- the rule takes 1536 for
// the first three (16 requests: ~305 chunks with work at 1536 on 148 SMs) and 768 for the last (a rank's share of
// config 4 on eight GPUs: ~134 at 1536, ~201 at 1024, ~268 at 768).
int decode_chunk_tokens(const TaskBatch& b, int page_size, int requested) {
    if (requested > 0) return std::min(kChunk, std::max(kMinChunk, requested / 16 * 16));
    const double max_tokens = static_cast<double>(b.p[3].cols) * page_size;
    const double want = 1.5 * sm_count();
    for (int c : {1536, 1024, 768})
        if (c <= kChunk && static_cast<double>(b.ntasks) * max_tokens / (2.0 * c) >= want) return c;
    return kMinChunk;
}

template <int G>
cudaError_t launch_decode_g(const TaskBatch& b, int page_size, void* scratch, cudaStream_t s, int chunk_request) {
    if (b.ntasks <= 0) return cudaSuccess;
    unsigned* arrivals = static_cast<unsigned*>(scratch);
    float* partials = reinterpret_cast<float*>(static_cast<char*>(scratch) + decode_arrivals_bytes(b.ntasks));
    if (decode_tma_ok(b, page_size)) {
        const int chunk_tokens = decode_chunk_tokens(b, page_size, chunk_request);
        const int chunks = decode_chunks(b, page_size, chunk_tokens);
        const int64_t grid = b.ntasks * chunks;
        if (grid > 0x7fffffff) return cudaErrorInvalidValue;
        const ParamDesc& K = b.p[1];
        const ParamDesc& V = b.p[2];
        CUtensorMap mk, mv;
        const int64_t krows = (K.numel_span + K.s4 - 1) / K.s4, vrows = (V.numel_span + V.s4 - 1) / V.s4;
        if (tc::make_map_f16(&mk, K.base, K.s4, krows, 64, kMmaPage) &&
            tc::make_map_f16(&mv, V.base, V.s4, vrows, 64, kMmaPage)) {
            cudaError_t e = cudaSuccess;
            if (chunks > 1) e = cudaMemsetAsync(arrivals, 0, static_cast<size_t>(b.ntasks) * sizeof(unsigned), s);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_decode_tma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kMmaSmemBytes);
            if (e == cudaSuccess)  // all of the unified L1 as shared memory: three CTAs per SM
                e = cudaFuncSetAttribute(paged_decode_tma_kernel<G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            paged_decode_tma_kernel<G><<<static_cast<unsigned>(grid), kMmaThreads, kMmaSmemBytes, s>>>(
                mk, mv, b, chunks, chunk_tokens, partials, arrivals);
            return cudaGetLastError();
        }
    }
    const int chunks = decode_chunks(b, page_size, kFbChunk);
    const int64_t grid = b.ntasks * chunks;
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    paged_decode_chunk_kernel<G><<<static_cast<unsigned>(grid), kDecThreads, 0, s>>>(b, page_size, chunks, partials);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    paged_decode_merge_kernel<G><<<static_cast<unsigned>(b.ntasks), kDecThreads, 0, s>>>(b, page_size, chunks, partials);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// top-k
// ---------------------------------------------------------------------------

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kHistCopies = 16;                    // lane-private copies of the 256-bin histogram (lanes l, l+16 share one)
constexpr int kTopkSmemMax = 227 * 1024 - 2048;    // opt-in dynamic shared memory less this kernel's static part
constexpr int kCandMax = 8192;                     // candidate list (sampled bound, or the last radix pass)
constexpr int kTieMax = 512;                       // ties at the threshold ranked pairwise up to this many

__device__ __forceinline__ uint32_t order_key(float f) {
    // Larger float -> larger unsigned key; -0.0 and +0.0 map to the same key.
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) == 0) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (key, index) composite: larger key first, then lower index first, as one unsigned compare.
__device__ __forceinline__ unsigned long long topk_composite(uint32_t key, int index) {
    return (static_cast<unsigned long long>(key) << 32) | (0xffffffffu - static_cast<uint32_t>(index));
}

struct TopkLayout {  // dynamic shared memory, in bytes
    int keys, scratch, comp, cand, cand_cap, total;
    __host__ __device__ TopkLayout(int n, int k2) {
        keys = 0;
        scratch = ((n * 4 + 15) / 16) * 16;  // histogram during the select; tie list / per-warp counts after it
        comp = scratch + 256 * kHistCopies * 4;
        cand = comp + k2 * 8;
        const int room = (kTopkSmemMax - cand) / 8;
        cand_cap = room < 0 ? 0 : (room > kCandMax ? kCandMax : room);
        total = cand + cand_cap * 8;
    }
};

// Append `v` for every lane with `p` set to buf[*counter ...] (one shared atomic per warp; slots in lane
// order within the warp).  The counter keeps counting past `cap`, so an overflow is visible; nothing is
// stored at or beyond `cap`.
__device__ __forceinline__ void warp_append(bool p, unsigned long long v, unsigned long long* buf, uint32_t* counter,
                                            uint32_t cap, int lane) {
    const unsigned bal = __ballot_sync(0xffffffffu, p);
    if (bal == 0u) return;
    uint32_t pos = 0;
    if (lane == 0) pos = atomicAdd(counter, static_cast<uint32_t>(__popc(bal)));
    pos = __shfl_sync(0xffffffffu, pos, 0) + __popc(bal & ((1u << lane) - 1u));
    if (p && pos < cap) buf[pos] = v;
}

// warp_append for four values per lane with one atomic per warp: values of slot j of every lane come before
// those of slot j + 1.
__device__ __forceinline__ void warp_append4(const bool (&p)[4], const unsigned long long (&v)[4], unsigned long long* buf,
                                             uint32_t* counter, uint32_t cap, int lane) {
    unsigned bal[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) bal[j] = __ballot_sync(0xffffffffu, p[j]);
    if ((bal[0] | bal[1] | bal[2] | bal[3]) == 0u) return;
    uint32_t pos = 0;
    if (lane == 0)
        pos = atomicAdd(counter, static_cast<uint32_t>(__popc(bal[0]) + __popc(bal[1]) + __popc(bal[2]) + __popc(bal[3])));
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const unsigned below = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t at = pos + __popc(bal[j] & below);
        if (p[j] && at < cap) buf[at] = v[j];
        pos += __popc(bal[j]);
    }
}

// Bitonic sort, descending, of the K2 composites in `comp` with E of them per thread in registers: thread t
// holds elements E*t .. E*t+E-1 (K2 / E threads, whole warps, take part).  Strides below E are compare-exchanges
// inside the thread, strides below 32*E shuffles with lane ^ (stride / E), longer ones go through shared memory
// (one block barrier each).  Then the first K indices are written to `dst`.  Every thread of the block calls it.
template <int E>
__device__ __forceinline__ void bitonic_sort_store(unsigned long long* comp, int K2, int K, int32_t* dst, int64_t ds) {
    const int t = threadIdx.x;
    const int nthr = K2 / E;
    const bool active = t < nthr;
    const int et = E * t;
    unsigned long long e[E];
    __syncthreads();  // the gather wrote across warps
#pragma unroll
    for (int j = 0; j < E; ++j) e[j] = active ? comp[et + j] : 0ull;
    for (int size = 2; size <= K2; size <<= 1) {
        int stride = size >> 1;
        if (stride >= 32 * E) {
            if (active) {
#pragma unroll
                for (int j = 0; j < E; ++j) comp[et + j] = e[j];
            }
            for (; stride >= 32 * E; stride >>= 1) {
                __syncthreads();
                if (active) {
#pragma unroll
                    for (int q = 0; q < E / 2; ++q) {
                        const int p = t + q * nthr;
                        const int lo = 2 * p - (p & (stride - 1));
                        const int hi = lo + stride;
                        const bool desc = (lo & size) == 0;
                        const unsigned long long x = comp[lo], y = comp[hi];
                        if ((x < y) == desc) {
                            comp[lo] = y;
                            comp[hi] = x;
                        }
                    }
                }
            }
            __syncthreads();
            if (active) {
#pragma unroll
                for (int j = 0; j < E; ++j) e[j] = comp[et + j];
            }
        }
        if (active) {
            // strides >= E: the partner is the same slot of lane ^ (stride / E); whether this thread keeps the
            // larger value depends only on the thread (E*t + j and E*t agree on every bit >= E)
            const bool up = (et & size) == 0;
            for (; stride >= E; stride >>= 1) {
                const bool keep_max = ((et & stride) == 0) == up;
                const int lx = stride / E;
#pragma unroll
                for (int j = 0; j < E; ++j) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, e[j], lx);
                    if ((other > e[j]) == keep_max) e[j] = other;
                }
            }
#pragma unroll
            for (int st = E / 2; st >= 1; st >>= 1) {
                if (st <= stride) {
#pragma unroll
                    for (int j = 0; j < E; ++j) {
                        if ((j & st) == 0) {
                            const bool desc = size > E / 2 ? up : (j & size) == 0;
                            const unsigned long long a = e[j], c = e[j + st];
                            if ((a < c) == desc) {
                                e[j] = c;
                                e[j + st] = a;
                            }
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < E; ++j) {
        const int i = et + j;
        if (active && i < K) dst[i * ds] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(e[j] & 0xffffffffull));
    }
}

// The warp's 32 values sorted in descending order across the lanes (bitonic network over shuffles): lane i gets
// the (i+1)-th largest.
__device__ __forceinline__ uint32_t warp_sort_desc(uint32_t v, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
        const bool desc = size == 32 || (lane & size) == 0;
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, v, stride);
            const bool keep_max = ((lane & stride) == 0) == desc;
            v = keep_max ? max(v, o) : min(v, o);
        }
    }
    return v;
}

// Radix-select digit choice from 256 bin totals: the digit d (bits shift .. shift+7) with
// count(digit > d) < need <= count(digit >= d); every thread gets back the prefix extended by d and the rank
// still needed inside that digit, s_eq the digit's count.  Call with bin_tot complete and visible to warp 0;
// two block barriers.
__device__ __forceinline__ void topk_pick_digit(const uint32_t* bin_tot, uint32_t* s_prefix, uint32_t* s_need,
                                                uint32_t* s_eq, int shift, uint32_t& prefix, uint32_t& need, int lane,
                                                int wid) {
    if (wid == 0) {
        // lane l holds bins 8l .. 8l+7
        uint32_t c[8], local = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            c[j] = bin_tot[8 * lane + j];
            local += c[j];
        }
        uint32_t suf = local;  // sum over lanes l .. 31
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t n = __shfl_down_sync(0xffffffffu, suf, o);
            if (lane + o < 32) suf += n;
        }
        const uint32_t above = suf - local;
        if (above < need && need <= suf) {
            uint32_t acc = above;
            int d = 8 * lane;
            uint32_t rem = need - above, cnt_d = 0;
#pragma unroll
            for (int j = 7; j >= 0; --j) {
                if (acc + c[j] >= need) {
                    d = 8 * lane + j;
                    rem = need - acc;
                    cnt_d = c[j];
                    break;
                }
                acc += c[j];
            }
            *s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
            *s_need = rem;
            *s_eq = cnt_d;
        }
    }
    __syncthreads();
    prefix = *s_prefix;
    need = *s_need;
    __syncthreads();  // the totals and the shared results are free for the next pass
}

// Sums the lane-private histogram copies into bin_tot, then picks the digit (topk_pick_digit).
__device__ __forceinline__ void topk_radix_digit(const uint32_t* hist, uint32_t* bin_tot, uint32_t* s_prefix,
                                                 uint32_t* s_need, uint32_t* s_eq, int shift, uint32_t& prefix,
                                                 uint32_t& need, int lane, int wid) {
    __syncthreads();
    for (int bin = wid * 8; bin < wid * 8 + 8; ++bin) {
        const uint32_t v = lane < kHistCopies ? hist[bin * kHistCopies + lane] : 0u;
        const uint32_t t = __reduce_add_sync(0xffffffffu, v);
        if (lane == 0) bin_tot[bin] = t;
    }
    __syncthreads();
    topk_pick_digit(bin_tot, s_prefix, s_need, s_eq, shift, prefix, need, lane, wid);
}

// One CTA per row.  (1) Keys: the row as order-preserving 32-bit keys in
// shared memory.  (2) Sampled bound: the 16-bit bucket of a high-ranked key of
// an evenly spaced 1024-key sample bounds the threshold from below; the keys
// at or above it are listed (about 1.5 K of them for 2048 of 32768).
// (3) Select: the exact K-th largest key by a 4-pass 8-bit radix select over
// that list -- or, when the bound missed (skewed rows), over the row, pass 2
// then sending keys above the 16-bit prefix straight to the composite buffer
// and listing those matching it for pass 3.  Each pass histograms the keys
// that match the digits chosen so far into lane-private copies of a 256-bin
// histogram, sums the copies, and one warp finds the digit of the K-th key.
// (4) Gather: the listed keys above the threshold join the winners; keys
// equal to the threshold join them too when all are taken, otherwise the
// `need` of lowest index (the reference's stable order) are ranked by index.
// (5) Bitonic sort of the (key, ~index) composites, descending.  Winners land
// in arbitrary slots; the sort's total order makes the result exact.
__global__ void __launch_bounds__(kTopkThreads) topk_select_kernel(TaskBatch b) {
    extern __shared__ __align__(16) uint8_t tsm[];
    __shared__ uint32_t bin_tot[256];
    __shared__ uint32_t s_prefix, s_need, s_eq, s_ncand, s_nwin, s_ntie, s_nsmall;
    __shared__ uint32_t s_small[32];  // the last few keys of the selection (listed path)
    const int64_t task = blockIdx.x;
    if (task >= b.ntasks) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the scores' producer has completed (dependent launch)
    const int64_t* rec = b.rec + task * b.stride;
    const ParamDesc& S = b.p[0];
    const ParamDesc& O = b.p[1];
    const int N = S.cols, K = O.cols;
    int K2 = 1;
    while (K2 < K) K2 <<= 1;
    const TopkLayout lay(N, K2);
    uint32_t* ks = reinterpret_cast<uint32_t*>(tsm + lay.keys);
    const uint4* ks4 = reinterpret_cast<const uint4*>(ks);
    uint32_t* hist = reinterpret_cast<uint32_t*>(tsm + lay.scratch);
    unsigned long long* comp = reinterpret_cast<unsigned long long*>(tsm + lay.comp);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(tsm + lay.cand);
    const uint32_t cand_cap = static_cast<uint32_t>(lay.cand_cap);
    const float* src = reinterpret_cast<const float*>(S.base) + rec[0];
    const int64_t ss = S.s4;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int n4 = (N + 3) >> 2;  // 16-byte groups of keys (the last one may be partial; the buffer is padded)
    uint32_t* hl = hist + (lane & (kHistCopies - 1));

    // (1) keys
    if (threadIdx.x == 0) {
        s_ncand = 0u;
        s_nwin = 0u;
        s_ntie = 0u;
    }
    int head = 0;  // keys [0, head) come in 16-byte vectors, eight per thread in flight
    if (ss == 1 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const int f4 = N >> 2;
        head = f4 << 2;
        const float4* src4 = reinterpret_cast<const float4*>(src);
        uint4* w4 = reinterpret_cast<uint4*>(ks);
        for (int base = 0; base < f4; base += 8 * kTopkThreads) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * kTopkThreads + threadIdx.x;
                if (i < f4) v[j] = __ldg(src4 + i);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * kTopkThreads + threadIdx.x;
                if (i < f4) w4[i] = make_uint4(order_key(v[j].x), order_key(v[j].y), order_key(v[j].z), order_key(v[j].w));
            }
        }
    }
    for (int i0 = head; i0 < N; i0 += 8 * kTopkThreads) {  // strided rows and the ragged tail
        uint32_t kk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * kTopkThreads + threadIdx.x;
            kk[j] = i < N ? order_key(src[static_cast<int64_t>(i) * ss]) : 0u;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * kTopkThreads + threadIdx.x;
            if (i < N) ks[i] = kk[j];
        }
    }
    __syncthreads();

    // (2) A lower bound for the threshold from an evenly spaced sample of 1024 keys, one per thread: every warp
    // sorts its 32 and takes its c-th largest, c = r / 32 rounded up, with r four standard deviations above the
    // expected number of winners in the sample; the bound is the median of the 32 warps' values (about the
    // quantile of r / 1024, where a warp's c-th largest falls below it as often as above).  Every key at or above
    // it is listed; when that gives between K and the list's capacity keys, the exact selection runs over the
    // list alone.  Otherwise (a skewed row) the full-row passes below run.
    bool from_cand = false;
    {
        const float expect = static_cast<float>(K) * kTopkThreads / static_cast<float>(N);
        const int r = static_cast<int>(ceilf(expect + 4.f * sqrtf(expect) + 4.f));
        if (N >= 4 * kTopkThreads && r < kTopkThreads / 4 && cand_cap >= static_cast<uint32_t>(K)) {
            const int c = (r + 31) / 32;  // 1 .. 8
            const uint32_t smp = warp_sort_desc(ks[static_cast<int64_t>(threadIdx.x) * N / kTopkThreads], lane);
            const uint32_t wc_th = __shfl_sync(0xffffffffu, smp, c - 1);
            if (lane == 0) bin_tot[wid] = wc_th;
            __syncthreads();
            if (wid == 0) {
                const uint32_t m = warp_sort_desc(bin_tot[lane], lane);
                if (lane == kTopkWarps / 2) s_prefix = m;  // the lower median of the warps' values
            }
            __syncthreads();
            const uint32_t lo = s_prefix;
            // every warp lists its keys >= lo into its own segment of the list (no shared counter), then the
            // segments are packed to the front
            const unsigned below = (1u << lane) - 1u;
            const uint32_t seg = cand_cap / kTopkWarps;
            uint32_t wc = 0;  // keys this warp found (the same in every lane)
            for (int base = 0; base < n4; base += kTopkThreads) {  // warps step together (ballots)
                const int q = base + threadIdx.x;
                const uint4 k4 = q < n4 ? ks4[q] : make_uint4(0u, 0u, 0u, 0u);
                const int lim = N - 4 * q;
                const uint32_t kk[4] = {k4.x, k4.y, k4.z, k4.w};
                unsigned bal[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) bal[j] = __ballot_sync(0xffffffffu, j < lim && kk[j] >= lo);
                if ((bal[0] | bal[1] | bal[2] | bal[3]) == 0u) continue;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t at = wc + __popc(bal[j] & below);
                    if (((bal[j] >> lane) & 1u) && at < seg) cand[wid * seg + at] = topk_composite(kk[j], 4 * q + j);
                    wc += __popc(bal[j]);
                }
            }
            uint32_t* wcnt = hist;  // the histogram is free until the next pass
            if (lane == 0) wcnt[wid] = wc;
            __syncthreads();
            uint32_t off = 0, tot = 0;
            bool over = false;
            for (int w = 0; w < kTopkWarps; ++w) {
                const uint32_t c = wcnt[w];
                if (w < wid) off += c;
                tot += c;
                over = over || c > seg;
            }
            from_cand = !over && tot >= static_cast<uint32_t>(K) && tot <= cand_cap;
            if (from_cand) {
                unsigned long long v[kCandMax / kTopkWarps / 32];
#pragma unroll
                for (int e = 0; e < kCandMax / kTopkWarps / 32; ++e) {
                    const uint32_t i = lane + 32u * e;
                    v[e] = i < wc ? cand[wid * seg + i] : 0ull;
                }
                __syncthreads();  // every segment is in registers before any is overwritten
#pragma unroll
                for (int e = 0; e < kCandMax / kTopkWarps / 32; ++e) {
                    const uint32_t i = lane + 32u * e;
                    if (i < wc) cand[off + i] = v[e];
                }
                if (threadIdx.x == 0) s_ncand = tot;
            }
            __syncthreads();
        }
    }

    // (3) radix select, most significant digit first: over the listed keys, or over the row (pass 2 then sorts the
    // row out: keys above the 16-bit prefix go straight to the composite buffer, keys matching it are listed for
    // pass 3 and the gather)
    uint32_t prefix = 0, need = static_cast<uint32_t>(K);
    int first_pass = 0;
    if (from_cand) {
        // the leading bytes every listed key shares need no pass: each would pick that byte, `need` unchanged
        const int nc = static_cast<int>(s_ncand);
        uint32_t ka = 0xffffffffu, ko = 0u;
        for (int i = threadIdx.x; i < nc; i += kTopkThreads) {
            const uint32_t k = static_cast<uint32_t>(cand[i] >> 32);
            ka &= k;
            ko |= k;
        }
        ka = __reduce_and_sync(0xffffffffu, ka);
        ko = __reduce_or_sync(0xffffffffu, ko);
        if (lane == 0) {
            bin_tot[wid] = ka;
            bin_tot[kTopkWarps + wid] = ko;
        }
        __syncthreads();
        ka = bin_tot[lane];
        ko = bin_tot[kTopkWarps + lane];
        ka = __reduce_and_sync(0xffffffffu, ka);
        ko = __reduce_or_sync(0xffffffffu, ko);
        first_pass = (ka ^ ko) == 0u ? 4 : __clz(static_cast<int>(ka ^ ko)) / 8;
        if (first_pass > 0) prefix = ka & (0xffffffffu << (32 - 8 * first_pass));
        if (first_pass == 4 && threadIdx.x == 0) s_eq = static_cast<uint32_t>(nc);  // one key value: all equal it
        __syncthreads();  // the totals area is free again; s_eq set
    }
    for (int pass = first_pass; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        const uint32_t hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = threadIdx.x; i < 256 * kHistCopies; i += kTopkThreads) hist[i] = 0u;
        __syncthreads();  // previous totals read, counters zeroed
        if (from_cand || (pass == 3 && s_ncand <= cand_cap)) {
            const int nc = static_cast<int>(s_ncand);
            for (int i = threadIdx.x; i < nc; i += kTopkThreads) {
                const uint32_t k = static_cast<uint32_t>(cand[i] >> 32);
                if ((k & hmask) == prefix) atomicAdd(hl + ((k >> shift) & 255u) * kHistCopies, 1u);
            }
        } else {
            for (int base = 0; base < n4; base += kTopkThreads) {  // warps step together (ballots below)
                const int q = base + threadIdx.x;
                const uint4 k4 = q < n4 ? ks4[q] : make_uint4(0u, 0u, 0u, 0u);
                const int lim = N - 4 * q;  // keys of this group inside the row
                const uint32_t kk[4] = {k4.x, k4.y, k4.z, k4.w};
                bool m[4], w[4];
                unsigned long long c[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t k = kk[j];
                    m[j] = j < lim && (k & hmask) == prefix;
                    w[j] = j < lim && (k & hmask) > prefix;
                    c[j] = topk_composite(k, 4 * q + j);
                    if (m[j]) atomicAdd(hl + ((k >> shift) & 255u) * kHistCopies, 1u);
                }
                if (pass == 2) {
                    warp_append4(m, c, cand, &s_ncand, cand_cap, lane);
                    warp_append4(w, c, comp, &s_nwin, static_cast<uint32_t>(K), lane);
                }
            }
        }
        topk_radix_digit(hist, bin_tot, &s_prefix, &s_need, &s_eq, shift, prefix, need, lane, wid);
        if (from_cand && pass < 3 && s_eq <= 32u) {
            // at most 32 listed keys still match the decided prefix: list them and let one warp sort them and
            // pick the need-th largest, instead of the remaining passes
            const uint32_t pm = 0xffffffffu << shift;
            const int nc = static_cast<int>(s_ncand);
            if (threadIdx.x == 0) s_nsmall = 0u;
            __syncthreads();
            for (int i = threadIdx.x; i < nc; i += kTopkThreads) {
                const uint32_t k = static_cast<uint32_t>(cand[i] >> 32);
                if ((k & pm) == prefix) s_small[atomicAdd(&s_nsmall, 1u) & 31u] = k;
            }
            __syncthreads();
            if (wid == 0) {
                const uint32_t m = s_eq;  // == the number listed
                const bool in = static_cast<uint32_t>(lane) < m;
                const uint32_t v = warp_sort_desc(in ? s_small[lane] : 0u, lane);
                const uint32_t t = __shfl_sync(0xffffffffu, v, static_cast<int>(need) - 1);
                const unsigned gt = __ballot_sync(0xffffffffu, in && v > t), eq = __ballot_sync(0xffffffffu, in && v == t);
                if (lane == 0) {
                    s_prefix = t;
                    s_need = need - static_cast<uint32_t>(__popc(gt));
                    s_eq = static_cast<uint32_t>(__popc(eq));
                }
            }
            __syncthreads();
            prefix = s_prefix;
            need = s_need;
            __syncthreads();  // before the shared words are reused
            break;
        }
    }
    const uint32_t thr = prefix;       // the K-th largest key; `need` keys equal to it are taken
    const bool all_eq = s_eq == need;  // no tie to break: every key equal to the threshold is taken
    const uint32_t n_gt = static_cast<uint32_t>(K) - need;  // keys strictly above the threshold
    unsigned long long* tie = reinterpret_cast<unsigned long long*>(hist);  // histogram no longer needed

    // (4) gather the rest of the winners from the candidates (or, if they overflowed, from the row)
    if (s_ncand <= cand_cap) {
        const int nc = static_cast<int>(s_ncand);
        for (int base = 0; base < nc; base += kTopkThreads) {
            const int i = base + threadIdx.x;
            const unsigned long long c = i < nc ? cand[i] : 0ull;
            const uint32_t k = static_cast<uint32_t>(c >> 32);
            warp_append(i < nc && (k > thr || (all_eq && k == thr)), c, comp, &s_nwin, static_cast<uint32_t>(K), lane);
            if (!all_eq) warp_append(i < nc && k == thr, c, tie, &s_ntie, kTieMax, lane);
        }
    } else {
        const uint32_t p16 = thr & 0xffff0000u;
        for (int base = 0; base < N; base += kTopkThreads) {
            const int i = base + threadIdx.x;
            const uint32_t k = i < N ? ks[i] : 0u;
            const bool in = i < N && (k & 0xffff0000u) == p16;
            warp_append(in && (k > thr || (all_eq && k == thr)), topk_composite(k, i), comp, &s_nwin,
                        static_cast<uint32_t>(K), lane);
            if (!all_eq) warp_append(in && k == thr, topk_composite(k, i), tie, &s_ntie, kTieMax, lane);
        }
    }
    __syncthreads();
    if (!all_eq) {
        if (s_ntie <= static_cast<uint32_t>(kTieMax)) {
            // rank the equal keys by index (same key: the larger composite has the lower index)
            const int m = static_cast<int>(s_ntie);
            for (int j = threadIdx.x; j < m; j += kTopkThreads) {
                const unsigned long long c = tie[j];
                uint32_t r = 0;
                for (int q = 0; q < m; ++q) r += tie[q] > c;
                if (r < need) comp[n_gt + r] = c;
            }
        } else {
            // many ties: an index-ordered sweep over the row.  Warp w owns the contiguous segment
            // [w * seg, (w + 1) * seg); the ballots of each round stay in registers (lane r holds rounds r and
            // r + 32), one scan of the warp totals gives each warp its first rank.
            uint32_t* cnt = hist;
            const int rounds = (N + kTopkThreads - 1) / kTopkThreads;
            const int s0 = wid * rounds * 32;
            unsigned eq_lo = 0, eq_hi = 0;
            uint32_t n_w = 0;
            for (int r = 0; r < rounds; ++r) {
                const int i = s0 + r * 32 + lane;
                const unsigned me = __ballot_sync(0xffffffffu, i < N && ks[i] == thr);
                n_w += __popc(me);
                if (lane == (r & 31)) {
                    if (r < 32) eq_lo = me;
                    else eq_hi = me;
                }
            }
            __syncthreads();  // the tie list is no longer read
            if (lane == 0) cnt[wid] = n_w;
            __syncthreads();
            if (wid == 0) {
                const uint32_t v = cnt[lane];
                uint32_t inc = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t n = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += n;
                }
                cnt[lane] = inc - v;
            }
            __syncthreads();
            uint32_t pe = cnt[wid];
            for (int r = 0; r < rounds && pe < need; ++r) {
                const unsigned me = __shfl_sync(0xffffffffu, r < 32 ? eq_lo : eq_hi, r & 31);
                const uint32_t rank = pe + __popc(me & ((1u << lane) - 1u));
                if (((me >> lane) & 1u) && rank < need) comp[n_gt + rank] = topk_composite(thr, s0 + r * 32 + lane);
                pe += __popc(me);
            }
        }
    }
    for (int i = threadIdx.x; i < K2; i += kTopkThreads)
        if (i >= K) comp[i] = 0ull;  // padding sorts last

    // (5) bitonic sort of K2 composites, descending (key desc, then index asc via the inverted index).
    int32_t* dst = reinterpret_cast<int32_t*>(O.base) + rec[1];
    if (K2 >= 128 && K2 <= 4 * kTopkThreads) {
        bitonic_sort_store<4>(comp, K2, K, dst, O.s4);
        return;
    }
    if (K2 == 64) {
        bitonic_sort_store<2>(comp, K2, K, dst, O.s4);
        return;
    }
    // other sizes: every stage in shared memory.  Pair p touches elements of the 64-element block of
    // warp p / 32, so a stage whose stride is below 64 and follows such a stage needs only the warp.
    int prev_stride = 1 << 30;  // the gather wrote across warps: the first stage synchronises the block
    for (int size = 2; size <= K2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32 * 2 || prev_stride >= 32 * 2) __syncthreads();
            else __syncwarp();
            for (int p = threadIdx.x; p < K2 / 2; p += kTopkThreads) {
                const int lo = 2 * p - (p & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const unsigned long long a = comp[lo], c = comp[hi];
                if ((a < c) == desc) {
                    comp[lo] = c;
                    comp[hi] = a;
                }
            }
            prev_stride = stride;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < K; i += kTopkThreads)
        dst[i * O.s4] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(comp[i] & 0xffffffffull));
}

}  // namespace

size_t paged_decode_scratch_bytes(const TaskBatch& b, int page_size) {

    const int G = b.p[0].rows;
    return decode_arrivals_bytes(b.ntasks) +
           static_cast<size_t>(b.ntasks) * decode_chunks(b, page_size, std::min(kChunk, kFbChunk)) *
               (G * kHeadDim + 2 * G) * sizeof(float);
}

cudaError_t launch_paged_decode(const TaskBatch& b, int page_size, int chunk_tokens, int, void* scratch,
                                size_t scratch_bytes, cudaStream_t s) {
    if (scratch_bytes < paged_decode_scratch_bytes(b, page_size)) return cudaErrorInvalidValue;
    switch (b.p[0].rows) {
        case 1: return launch_decode_g<1>(b, page_size, scratch, s, chunk_tokens);
        case 2: return launch_decode_g<2>(b, page_size, scratch, s, chunk_tokens);
        case 4: return launch_decode_g<4>(b, page_size, scratch, s, chunk_tokens);
        case 8: return launch_decode_g<8>(b, page_size, scratch, s, chunk_tokens);
        default: return cudaErrorInvalidValue;
    }
}

size_t topk_select_scratch_bytes(const TaskBatch&) { return 0; }

int topk_smem_bytes(int n, int k) {
    int k2 = 1;
    while (k2 < k) k2 <<= 1;
    return TopkLayout(n, k2).total;
}

bool topk_supported(int n, int k) {
    return n >= 1 && n <= 65535 && k >= 1 && k <= n && k <= 4096 && topk_smem_bytes(n, k) <= 227 * 1024 - 2048;  // opt-in max less static
}

cudaError_t launch_topk_select(const TaskBatch& b, int, void*, size_t, cudaStream_t s) {
    if (!topk_supported(b.p[0].cols, b.p[1].cols)) return cudaErrorInvalidValue;
    const int smem = topk_smem_bytes(b.p[0].cols, b.p[1].cols);
    if (b.ntasks <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(topk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // Programmatic dependent launch: the grid may be scheduled while the kernel before it on the stream (the
    // indexer's scoring, which allows it) finishes; every CTA waits for that kernel's completion and memory
    // (griddepcontrol.wait) before it reads a score.  After any other kernel it behaves as a plain launch.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(b.ntasks));
    cfg.blockDim = dim3(kTopkThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, topk_select_kernel, b);
}

}  // namespace ptowsp::dev

namespace ptowsp::dev {

// ===========================================================================
// Paged GQA decode without any device allocation.
//
// Some callers cannot let a library call cudaMalloc on their hot path: a
// serving engine that reserved all device memory up front for its own KV-cache
// pool (an extra allocation can fail, or carve memory out of that pool), or a
// host that runs other streams concurrently and cannot afford the implicit
// device-wide synchronisation cudaMalloc/cudaFree can cause.  For them this
// entry point keeps its scratch (task records, split-KV partial results and
// the status word) in one fixed array in device memory that belongs to this
// library, instead of the program's grown-on-demand buffer.
//
// Costs and rules, in the caller's terms:
//  * the array is kPtowspNoAllocScratchBytes (24 MiB) and every GPU that loads
//    this library keeps it until the process exits;
//  * a workload that needs more (records + partials, see
//    ptowsp_noalloc_bytes_needed) is rejected with PTOWSP_ERR_LIMIT;
//  * all calls share the one array and it keeps whatever the last call left:
//    the call clears the status word itself, and everything else it reads it
//    writes first -- but two calls whose work overlaps on the GPU (different
//    streams, or different host threads) race on the array;
//  * the first call on a device looks up the array's device address (with that
//    device current) and loads every kernel the entry point can launch (lazy
//    module loading would otherwise load code, and take device memory, at a
//    later call); make that first call before any stream capture, and count
//    on later calls, not the first, to take no device memory.
// ===========================================================================

namespace {

constexpr size_t kPtowspNoAllocScratchBytes = size_t(24) << 20;
constexpr int kNoAllocRecStride = 10;  // 6 view offsets, 2 axis args, 2 scalar args

static __device__ __align__(256) unsigned char g_noalloc_scratch[kPtowspNoAllocScratchBytes];

// Layout inside the array: [status word | 252 B pad | task records | partials].
constexpr size_t kNoAllocRecOffset = 256;

__global__ void noalloc_fill_records(int64_t* rec, int requests, int kv_heads, int group, int head_dim, int max_pages,
                                     int page_size) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<int64_t>(requests) * kv_heads) return;
    const int64_t r = t / kv_heads, h = t % kv_heads;
    int64_t* o = rec + t * kNoAllocRecStride;
    o[0] = t * group * head_dim;  // q[r][h]
    o[1] = 0;                     // k cache (whole pool)
    o[2] = 0;                     // v cache (whole pool)
    o[3] = r * max_pages;         // page_table[r]
    o[4] = r;                     // kv_len[r]
    o[5] = t * group * head_dim;  // out[r][h]
    o[6] = r;
    o[7] = h;
    o[8] = page_size;
    o[9] = kv_heads;
}

void* noalloc_scratch_address(int device, cudaError_t* err) {
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    if (device < 0 || device >= 64) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device]) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // device `device` is current here
        if (*err != cudaSuccess) return nullptr;
        // With lazy module loading a kernel's code is put on the device at its first launch, which takes device
        // memory.  Load every kernel this entry point can launch now, at the first call on the device, so that no
        // later call -- whatever its GQA group or launch path -- loads anything.
        cudaFuncAttributes fa;
        const void* kernels[] = {
            reinterpret_cast<const void*>(noalloc_fill_records),
            reinterpret_cast<const void*>(paged_decode_tma_kernel<1>), reinterpret_cast<const void*>(paged_decode_tma_kernel<2>),
            reinterpret_cast<const void*>(paged_decode_tma_kernel<4>), reinterpret_cast<const void*>(paged_decode_tma_kernel<8>),
            reinterpret_cast<const void*>(paged_decode_chunk_kernel<1>), reinterpret_cast<const void*>(paged_decode_chunk_kernel<2>),
            reinterpret_cast<const void*>(paged_decode_chunk_kernel<4>), reinterpret_cast<const void*>(paged_decode_chunk_kernel<8>),
            reinterpret_cast<const void*>(paged_decode_merge_kernel<1>), reinterpret_cast<const void*>(paged_decode_merge_kernel<2>),
            reinterpret_cast<const void*>(paged_decode_merge_kernel<4>), reinterpret_cast<const void*>(paged_decode_merge_kernel<8>)};
        for (const void* k : kernels) {
            *err = cudaFuncGetAttributes(&fa, k);
            if (*err != cudaSuccess) return nullptr;
        }
        addr[device] = p;
    }
    *err = cudaSuccess;
    return addr[device];
}

}  // namespace

size_t noalloc_scratch_capacity() { return kPtowspNoAllocScratchBytes; }

size_t noalloc_bytes_needed(int requests, int kv_heads, int group, int max_pages, int page_size) {
    const size_t tasks = static_cast<size_t>(requests) * kv_heads;
    const int64_t max_tokens = static_cast<int64_t>(max_pages) * page_size;
    const int64_t chunk_tokens = std::min(kChunk, kFbChunk);
    const size_t chunks = static_cast<size_t>(std::max<int64_t>(1, (max_tokens + chunk_tokens - 1) / chunk_tokens));
    return kNoAllocRecOffset + tasks * kNoAllocRecStride * sizeof(int64_t) + decode_arrivals_bytes(tasks) +
           tasks * chunks * (static_cast<size_t>(group) * kHeadDim + 2 * group) * sizeof(float);
}

// Returns a ptowsp_status code; *msg names the failure.
int paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* page_table,
                         const int32_t* kv_len, void* out, int requests, int kv_heads, int group, int head_dim,
                         int page_size, int max_pages, int64_t num_pages, cudaStream_t s, const char** msg) {
    *msg = "";
    if (!q || !k_cache || !v_cache || !page_table || !kv_len || !out) {
        *msg = "paged_decode_noalloc: null pointer";
        return 4;
    }
    if (requests <= 0 || kv_heads <= 0 || page_size <= 0 || max_pages <= 0 || num_pages <= 0) {
        *msg = "paged_decode_noalloc: sizes must be positive";
        return 4;
    }
    if (head_dim != kHeadDim || !(group == 1 || group == 2 || group == 4 || group == 8)) {
        *msg = "paged_decode_noalloc: head_dim must be 128 and the GQA group 1, 2, 4 or 8";
        return 2;
    }
    const size_t need = noalloc_bytes_needed(requests, kv_heads, group, max_pages, page_size);
    if (need > kPtowspNoAllocScratchBytes) {
        *msg = "paged_decode_noalloc: requests x kv_heads x ceil(max_pages*page_size/512) x (group*128+2*group)*4 B "
               "of partials plus task records and counters exceed the fixed 24 MiB scratch array";
        return 6;
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return 3;
    }
    char* base = static_cast<char*>(noalloc_scratch_address(device, &e));
    if (!base) {
        *msg = cudaGetErrorString(e);
        return 3;
    }
    int* status = reinterpret_cast<int*>(base);
    int64_t* rec = reinterpret_cast<int64_t*>(base + kNoAllocRecOffset);
    const size_t tasks = static_cast<size_t>(requests) * kv_heads;
    void* dec_scratch = base + kNoAllocRecOffset + tasks * kNoAllocRecStride * sizeof(int64_t);

    e = cudaMemsetAsync(status, 0, sizeof(int), s);  // the status word must start at zero
    if (e == cudaSuccess) {
        noalloc_fill_records<<<static_cast<unsigned>((tasks + 127) / 128), 128, 0, s>>>(rec, requests, kv_heads, group,
                                                                                        kHeadDim, max_pages, page_size);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return 3;
    }
    TaskBatch b{};
    b.rec = rec;
    b.ntasks = static_cast<int64_t>(tasks);
    b.stride = kNoAllocRecStride;
    b.nparams = 6;
    b.naxis = 2;
    b.nscalar = 2;
    b.err = status;
    const int64_t cache_span = num_pages * page_size * kv_heads * static_cast<int64_t>(kHeadDim);
    auto param = [](void* p, int64_t s3, int64_t s4, int64_t span, int rows, int cols, int type, int eb) {
        ParamDesc d{};
        d.base = static_cast<char*>(p);
        d.s3 = s3;
        d.s4 = s4;
        d.numel_span = span;
        d.rows = rows;
        d.cols = cols;
        d.type = type;
        d.elem_bytes = eb;
        return d;
    };
    const int64_t qspan = static_cast<int64_t>(tasks) * group * kHeadDim;
    b.p[0] = param(const_cast<void*>(q), kHeadDim, 1, qspan, group, kHeadDim, PT_F16, 2);
    b.p[1] = param(const_cast<void*>(k_cache), static_cast<int64_t>(page_size) * kv_heads * kHeadDim,
                   static_cast<int64_t>(kv_heads) * kHeadDim, cache_span, page_size, kv_heads * kHeadDim, PT_F16, 2);
    b.p[2] = param(const_cast<void*>(v_cache), static_cast<int64_t>(page_size) * kv_heads * kHeadDim,
                   static_cast<int64_t>(kv_heads) * kHeadDim, cache_span, page_size, kv_heads * kHeadDim, PT_F16, 2);
    b.p[3] = param(const_cast<int32_t*>(page_table), 0, 1, static_cast<int64_t>(requests) * max_pages, 1, max_pages,
                   PT_I32, 4);
    b.p[4] = param(const_cast<int32_t*>(kv_len), 0, 1, requests, 1, 1, PT_I32, 4);
    b.p[5] = param(out, kHeadDim, 1, qspan, group, kHeadDim, PT_F16, 2);
    switch (group) {
        case 1: e = launch_decode_g<1>(b, page_size, dec_scratch, s, 0); break;
        case 2: e = launch_decode_g<2>(b, page_size, dec_scratch, s, 0); break;
        case 4: e = launch_decode_g<4>(b, page_size, dec_scratch, s, 0); break;
        default: e = launch_decode_g<8>(b, page_size, dec_scratch, s, 0); break;
    }
    if (e != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return 3;
    }
    int host_status = 0;
    e = cudaMemcpyAsync(&host_status, status, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        *msg = cudaGetErrorString(e);
        return 3;
    }
    if (host_status) {
        *msg = (host_status & kErrBounds) ? "paged_decode_noalloc: a page id is outside the KV cache"
                                          : "paged_decode_noalloc: kv_len exceeds max_pages * page_size";
        return 5;
    }
    return 0;
}

}  // namespace ptowsp::dev
