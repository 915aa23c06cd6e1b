// Matmul tile tasks on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// A task is the reference's Matmul kernel instance (src/python/pto_codegen.cpp:
// 817-929): C[M,N] (f32) = A[M,K] (f16) . B[K,N] (f16), optionally C += A.B
// (the InOut accumulate form of examples/bgemm/pto_wsp_impl.py:56-76).  M = 128
// rows; N in {64,128,256}; K a multiple of 64.
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: per 64-wide K step, one 128x64 A box (K-major)
//               and N/64 boxes of 64(N)x64(K) B (MN-major, straight from the
//               row-major B view -- no transpose pass), 128-byte swizzle, into a
//               STAGES-deep shared-memory ring guarded by mbarriers.
//   warp 1      owns TMEM (2 accumulators of N f32 columns) and issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N, K=16) from one
//               thread; tcgen05.commit frees ring slots / publishes finished
//               accumulators.
//   warps 2-5   epilogue: tcgen05.ld 32x32b rows out of TMEM (warp w reads TMEM
//               lanes 32*(w%4)..), optional C add, 128-bit stores.  Two TMEM
//               accumulators let the epilogue of tile i overlap tile i+1's MMAs.
// Every mbarrier wait is bounded (~2 s of %globaltimer): on timeout the CTA
// records kErrTimeout, drains its own copies and MMAs, frees TMEM and returns.
// When the tasks pair up along M the CTA-pair kernel below runs instead.
// No cluster multicast anywhere (loads read this GPU's memory only).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "device.hpp"
#include "tc_common.cuh"

namespace ptowsp::dev {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int THREADS = 192;

struct MMArgs {
    const int64_t* rec;
    int64_t ntasks;
    int stride;
    int64_t a_pitch, b_pitch;  // elements per row of the A / B tensor maps
    float* c;                  // C base
    int64_t c_pitch;           // C row stride (elements)
    int k_steps;               // K / 64
    int accumulate;
    int* err;
};

using namespace tc;

template <int BN>
struct Smem {
    // as many ring stages as fit next to the barriers in the 227 KB per CTA (7 for N=128, 4 for N=256)
    static constexpr int STAGES_FIT = (232448 - 1280) / (BM * BK * 2 + BN * BK * 2);
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int A_BYTES = BM * BK * 2;              // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;              // BN/64 boxes of 8 KB
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static_assert(STAGES >= 2, "ring too small");
    static constexpr int BAR_OFF = RING;                      // barriers after the ring
    static constexpr int TOTAL = RING + 256 + 1024;           // + barriers/flags + alignment slack
    static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          MMArgs args) {
    using S = Smem<BN>;
    constexpr int STAGES = S::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
    // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], drain
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* drain = bars + 2 * STAGES + 4;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), 4 * 32);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(S::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int64_t first = blockIdx.x, step = gridDim.x;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, last_parity = 0;
            for (int64_t t = first; t < args.ntasks && !*abort_flag; t += step) {
                const int64_t* rec = args.rec + t * args.stride;
                const int64_t oa = rec[0], ob = rec[1];
                const int32_t ax = static_cast<int32_t>(oa % args.a_pitch), ay = static_cast<int32_t>(oa / args.a_pitch);
                const int32_t bx = static_cast<int32_t>(ob % args.b_pitch), by = static_cast<int32_t>(ob / args.b_pitch);
                for (int kb = 0; kb < args.k_steps; ++kb) {
                    if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, args.err)) break;
                    const uint32_t fb = smem_u32(&full[stage]);
                    mbar_expect_tx(fb, S::STAGE_BYTES);
                    uint8_t* sa = smem + stage * S::STAGE_BYTES;
                    uint8_t* sb = sa + S::A_BYTES;
                    tma_load_2d(smem_u32(sa), &tmap_a, ax + kb * BK, ay, fb);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tma_load_2d(smem_u32(sb + j * 8192), &tmap_b, bx + j * 64, by + kb * BK, fb);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // drain: every copy this CTA issued has landed before shared memory goes away
            for (int s = 0; s < STAGES; ++s)
                if (issued_mask & (1u << s)) {
                    const uint32_t fb = smem_u32(&full[s]);
                    const uint32_t par = (last_parity >> s) & 1u;
                    uint64_t start = globaltimer();
                    while (!mbar_try_wait(fb, par)) {
                        if (globaltimer() - start > kTimeoutNs) {
                            atomicOr(args.err, kErrTimeout);
                            break;
                        }
                    }
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_f16(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool issued = false;
            for (int64_t t = first; t < args.ntasks && !*abort_flag; t += step) {
                if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, args.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < args.k_steps; ++kb) {
                    if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, args.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * S::STAGE_BYTES);
                    const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // A: K-major, 128-byte rows, 8-row atoms 1024 B apart; step 32 B per K=16.
                        const uint64_t ad = smem_desc(sa + kk * 32, 16, 1024);
                        // B: MN-major, 64-element (128 B) N chunks 8 KB apart (LBO), 8-row K atoms 1 KB apart (SBO);
                        // step 16 K-rows (2 KB) per K=16.
                        const uint64_t bd = smem_desc(sb + kk * 2048, 8192, 1024);
                        mma_f16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(smem_u32(&empty[stage]));
                    issued = true;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(smem_u32(&tfull[acc]));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // drain: all MMAs this thread issued have completed before TMEM is freed
            if (issued) {
                mma_commit(smem_u32(drain));
                const uint64_t start = globaltimer();
                while (!mbar_try_wait(smem_u32(drain), 0)) {
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        break;
                    }
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int64_t t = first; t < args.ntasks && !*abort_flag; t += step) {
            if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, args.err)) break;
            tc_fence_after();
            const int64_t oc = args.rec[t * args.stride + 2];
            float* crow = args.c + oc + static_cast<int64_t>(row) * args.c_pitch;
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc) {
                float v[32];
                tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN + cc * 32), v);
                float4* dst = reinterpret_cast<float4*>(crow + cc * 32);
                if (args.accumulate) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 o = dst[i];
                        v[4 * i + 0] += o.x;
                        v[4 * i + 1] += o.y;
                        v[4 * i + 2] += o.z;
                        v[4 * i + 3] += o.w;
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&tempty[acc]));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(S::TMEM_COLS) : "memory");
    }
}

template <int BN>
cudaError_t launch_bn(const TaskBatch& b, int accumulate, int workers, cudaStream_t s) {
    const ParamDesc& A = b.p[0];
    const ParamDesc& B = b.p[1];
    const ParamDesc& C = b.p[2];
    CUtensorMap ma, mb;
    const int64_t a_rows = (A.numel_span + A.s3 - 1) / A.s3;
    const int64_t b_rows = (B.numel_span + B.s3 - 1) / B.s3;
    if (!make_map_f16(&ma, A.base, A.s3, a_rows, BK, BM)) return cudaErrorInvalidValue;
    if (!make_map_f16(&mb, B.base, B.s3, b_rows, 64, BK)) return cudaErrorInvalidValue;
    MMArgs args;
    args.rec = b.rec;
    args.ntasks = b.ntasks;
    args.stride = b.stride;
    args.a_pitch = A.s3;
    args.b_pitch = B.s3;
    args.c = reinterpret_cast<float*>(C.base);
    args.c_pitch = C.s3;
    args.k_steps = A.cols / BK;
    args.accumulate = accumulate;
    args.err = b.err;
    const int smem = Smem<BN>::TOTAL;
    cudaError_t e = cudaFuncSetAttribute(matmul_tcgen05_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int64_t grid = std::min<int64_t>(b.ntasks, sm_count());
    if (workers > 0) grid = std::min<int64_t>(grid, workers);
    grid = std::max<int64_t>(grid, 1);
    matmul_tcgen05_kernel<BN><<<static_cast<unsigned>(grid), THREADS, smem, s>>>(ma, mb, args);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// CTA-pair variant (the default when the tasks pair up along M).
//
// Two CTAs of a 2-CTA cluster share each MMA (tcgen05 cta_group::2, M = 256):
// a unit is two tasks whose A tiles are 128 rows apart and whose B tile is the
// same; CTA r computes task r's 128 x BN tile of C from its own A rows and its
// half (BN/2 columns) of the shared B tile.  Per 64-wide K step an SM then
// stages 16 KB of A and BN*64 B of B instead of 16 KB + BN*128 B, which both
// cuts the L2 -> SM traffic by a third (BN = 256) and lets a deeper ring fit.
// Barrier protocol as in the CTA-pair indexer kernel: both CTAs' TMA bytes
// land on the leader's full barrier, the leader issues the MMAs and commits
// to each CTA's barriers, one lane per epilogue warp of either CTA releases an
// accumulator on the leader, and cluster barriers bracket setup and teardown.
// ---------------------------------------------------------------------------

template <int BN>
struct PairSmem {
    static constexpr int A_BYTES = BM * BK * 2;              // 16 KB
    static constexpr int B_BYTES = (BN / 2) * BK * 2;        // this CTA's half of B: (BN/2)/64 boxes of 8 KB
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int OUT_BYTES = 4 * 2 * 32 * 32 * 4;    // epilogue staging: 2 tiles of 32 x 32 f32 per warp
    static constexpr int STAGES_FIT = (232448 - 1280 - OUT_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static constexpr int OUT_OFF = RING;                      // 1024-aligned: the 128-byte swizzle repeats per 1 KB
    static constexpr int BAR_OFF = OUT_OFF + OUT_BYTES;
    static constexpr int TOTAL = BAR_OFF + 256 + 1024;
    static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_c, MMArgs args) {
    using S = PairSmem<BN>;
    constexpr int STAGES = S::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
    uint64_t* full = bars;                      // [STAGES]  waited on in the leader
    uint64_t* empty = bars + STAGES;            // [STAGES]  both CTAs
    uint64_t* tfull = bars + 2 * STAGES;        // [2]       both CTAs
    uint64_t* tempty = bars + 2 * STAGES + 2;   // [2]       waited on in the leader
    uint64_t* drain = bars + 2 * STAGES + 4;    //           leader
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);

    const uint32_t rank = cluster_ctarank();  // 0: leader
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), 2 * 4);  // one lane of each epilogue warp of both CTAs
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(S::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t lead_bars = mapa_shared(smem_u32(bars), 0);
    const uint32_t peer_bars = mapa_shared(smem_u32(bars), 1);
    auto lead = [&](const uint64_t* b) { return lead_bars + static_cast<uint32_t>((b - bars) * 8); };
    auto peer = [&](const uint64_t* b) { return peer_bars + static_cast<uint32_t>((b - bars) * 8); };
    const int64_t first = blockIdx.x >> 1, step = gridDim.x >> 1;  // units: two tasks (6 record words)

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_parity = 0;
            for (int64_t u = first; u < args.ntasks && !*abort_flag; u += step) {
                const int64_t* rec = args.rec + u * 6 + rank * 3;
                const int64_t oa = rec[0], ob = rec[1];
                const int32_t ax = static_cast<int32_t>(oa % args.a_pitch), ay = static_cast<int32_t>(oa / args.a_pitch);
                const int32_t bx = static_cast<int32_t>(ob % args.b_pitch) + static_cast<int32_t>(rank) * (BN / 2);
                const int32_t by = static_cast<int32_t>(ob / args.b_pitch);
                for (int kb = 0; kb < args.k_steps; ++kb) {
                    if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, args.err)) break;
                    if (rank == 0) mbar_expect_tx(smem_u32(&full[stage]), 2 * S::STAGE_BYTES);
                    uint8_t* sa = smem + stage * S::STAGE_BYTES;
                    uint8_t* sb = sa + S::A_BYTES;
                    tma_load_2d_pair(smem_u32(sa), &tmap_a, ax + kb * BK, ay, lead(&full[stage]));
#pragma unroll
                    for (int j = 0; j < BN / 128; ++j)
                        tma_load_2d_pair(smem_u32(sb + j * 8192), &tmap_b, bx + j * 64, by + kb * BK, lead(&full[stage]));
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (rank == 0) {
                // drain: the pair's last copy into each stage has landed before shared memory goes away
                const uint64_t start = globaltimer();
                for (int s = 0; s < STAGES; ++s)
                    if (issued_mask & (1u << s))
                        while (!mbar_try_wait(smem_u32(&full[s]), (last_parity >> s) & 1u))
                            if (globaltimer() - start > kTimeoutNs) {
                                atomicOr(args.err, kErrTimeout);
                                break;
                            }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_f16(2 * BM, BN);  // M = 256 over the pair, B MN-major
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool issued = false;
            for (int64_t u = first; u < args.ntasks && !*abort_flag; u += step) {
                if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, args.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < args.k_steps; ++kb) {
                    if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, args.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * S::STAGE_BYTES);
                    const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = smem_desc(sa + kk * 32, 16, 1024);
                        const uint64_t bd = smem_desc(sb + kk * 2048, 8192, 1024);
                        mma_f16_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit_pair(lead(&empty[stage]));
                    mma_commit_pair(peer(&empty[stage]));
                    issued = true;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair(lead(&tfull[acc]));
                mma_commit_pair(peer(&tfull[acc]));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (issued) {
                mma_commit_pair(lead(drain));
                const uint64_t start = globaltimer();
                while (!mbar_try_wait(smem_u32(drain), 0))
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        break;
                    }
            }
        }
    } else {
        // epilogue (warps 2..5): this CTA's 128 rows x BN columns of its task's C tile.  Plain stores go
        // through shared memory: each warp stages a 32 x 32 f32 tile (128-byte swizzled, so the row-per-lane
        // writes hit distinct banks) and one lane sends it with a TMA store -- whole 128-byte rows instead of
        // 16-byte pieces of 32 rows per instruction.  The accumulate form reads C back and stores directly.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        uint8_t* out_stage = smem + S::OUT_OFF + (warp - 2) * (2 * 32 * 32 * 4);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int64_t u = first; u < args.ntasks && !*abort_flag; u += step) {
            if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, args.err)) break;
            tc_fence_after();
            const int64_t oc = args.rec[u * 6 + rank * 3 + 2];
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            if (args.accumulate) {
                float* crow = args.c + oc + static_cast<int64_t>(row) * args.c_pitch;
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld32_async(tbase + static_cast<uint32_t>(cc * 32), v);
                    tmem_wait_ld();
                    reg_fence(v);
                    float4* dst = reinterpret_cast<float4*>(crow + cc * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 c0 = dst[i];
                        dst[i] = make_float4(__uint_as_float(v[4 * i]) + c0.x, __uint_as_float(v[4 * i + 1]) + c0.y,
                                             __uint_as_float(v[4 * i + 2]) + c0.z, __uint_as_float(v[4 * i + 3]) + c0.w);
                    }
                }
            } else {
                const int32_t cx = static_cast<int32_t>(oc % args.c_pitch);
                const int32_t cy = static_cast<int32_t>(oc / args.c_pitch) + quarter * 32;
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld32_async(tbase + static_cast<uint32_t>(cc * 32), v);
                    tmem_wait_ld();
                    reg_fence(v);
                    uint8_t* buf = out_stage + (cc & 1) * (32 * 32 * 4);
                    if (cc >= 2) {
                        if (lane == 0) tma_store_wait_read<1>();  // the store that last read `buf` is done with it
                        __syncwarp();
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                            make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmap_c, cx + cc * 32, cy, smem_u32(buf));
                        tma_store_commit();
                    }
                }
                if (lane == 0) tma_store_wait_read<0>();  // the staging tiles are free for the next unit
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead(&tempty[acc]));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) tma_store_wait_all();  // every C tile written before the CTA retires
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader has drained the pair's copies and MMAs
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(S::TMEM_COLS) : "memory");
}

// CTA-pair launch over `units` (6 record words each); false when the pairs cannot be scheduled.
template <int BN>
bool launch_pair_bn(const TaskBatch& b, const int64_t* units, int64_t nunits, int accumulate, int workers, cudaStream_t s,
                    cudaError_t* err) {
    const ParamDesc& A = b.p[0];
    const ParamDesc& B = b.p[1];
    const ParamDesc& C = b.p[2];
    CUtensorMap ma, mb;
    const int64_t a_rows = (A.numel_span + A.s3 - 1) / A.s3;
    const int64_t b_rows = (B.numel_span + B.s3 - 1) / B.s3;
    if (!make_map_f16(&ma, A.base, A.s3, a_rows, BK, BM)) return false;
    if (!make_map_f16(&mb, B.base, B.s3, b_rows, 64, BK)) return false;
    CUtensorMap mc;
    const int64_t c_rows = (C.numel_span + C.s3 - 1) / C.s3;
    if (!make_map_f32(&mc, C.base, C.s3, c_rows, 32, 32)) return false;
    MMArgs args;
    args.rec = units;
    args.ntasks = nunits;
    args.stride = 6;
    args.a_pitch = A.s3;
    args.b_pitch = B.s3;
    args.c = reinterpret_cast<float*>(C.base);
    args.c_pitch = C.s3;
    args.k_steps = A.cols / BK;
    args.accumulate = accumulate;
    args.err = b.err;
    const int smem = PairSmem<BN>::TOTAL;
    if (cudaFuncSetAttribute(matmul_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int64_t pairs = std::max<int64_t>(1, sm_count() / 2);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    int resident = 0;  // pairs that fit at once: the persistent schedule needs all of them resident
    if (cudaOccupancyMaxActiveClusters(&resident, matmul_pair_kernel<BN>, &cfg) != cudaSuccess || resident < 1) {
        cudaGetLastError();
        return false;
    }
    pairs = std::min<int64_t>({pairs, resident, nunits});
    if (workers > 0) pairs = std::min<int64_t>(pairs, std::max(1, workers / 2));
    pairs = std::max<int64_t>(pairs, 1);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    *err = cudaLaunchKernelEx(&cfg, matmul_pair_kernel<BN>, ma, mb, mc, args);
    return true;
}

}  // namespace

bool matmul_tiles_supported(const TaskBatch& b) {
    const ParamDesc& A = b.p[0];
    const ParamDesc& B = b.p[1];
    const ParamDesc& C = b.p[2];
    if (A.rows != BM || A.cols % BK != 0 || A.cols < BK || B.rows != A.cols) return false;
    if (!(B.cols == 64 || B.cols == 128 || B.cols == 256) || C.rows != BM || C.cols != B.cols) return false;
    if (A.s4 != 1 || B.s4 != 1 || C.s4 != 1) return false;
    if (A.s3 % 8 || B.s3 % 8 || C.s3 % 4) return false;
    if ((reinterpret_cast<uintptr_t>(A.base) | reinterpret_cast<uintptr_t>(B.base) | reinterpret_cast<uintptr_t>(C.base)) & 15)
        return false;
    return true;
}

bool launch_matmul_pairs(const TaskBatch& b, const int64_t* units, int64_t nunits, int accumulate, int workers,
                         cudaStream_t s, cudaError_t* err) {
    switch (b.p[1].cols) {
        case 128: return launch_pair_bn<128>(b, units, nunits, accumulate, workers, s, err);
        case 256: return launch_pair_bn<256>(b, units, nunits, accumulate, workers, s, err);
        default: return false;
    }
}

cudaError_t launch_matmul_tiles(const TaskBatch& b, int accumulate, int workers, cudaStream_t s) {
    switch (b.p[1].cols) {
        case 64: return launch_bn<64>(b, accumulate, workers, s);
        case 128: return launch_bn<128>(b, accumulate, workers, s);
        case 256: return launch_bn<256>(b, accumulate, workers, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace ptowsp::dev
