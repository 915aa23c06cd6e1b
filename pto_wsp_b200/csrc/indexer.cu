// Built-in lightning-indexer scoring on tcgen05.
//
// One task = one batch element b:  scores[q, t] = sum_h w[q, h] * relu(q_{q,h} . k_t)
// for Q = 8 queries x H = 64 index heads, D = 128, T keys (the score the
// reference's toy top-k example takes as input, examples/deepseek_lightning_
// indexer/golden.py; DeepSeek "lightning indexer").  The contraction is
// Q*H x D x T per batch: 2*512*128 FLOP per 256-byte key row = 512 FLOP/B,
// above the HBM ridge, so it runs on the tensor cores:
//
//   * the batch's 512 q rows stay resident in shared memory (128 KB, four
//     128-byte-swizzled TMA boxes, K-major), loaded once per task;
//   * key tiles of 128 rows stream through a 3-stage TMA ring (A operand,
//     K-major straight from the row-major key matrix);
//   * per key tile two tcgen05.mma groups (M = 128 keys, N = 256 = 4 queries x
//     64 heads, K = 128 in 8 steps) fill two 256-column TMEM accumulators;
//   * eight epilogue warps (two per TMEM lane quarter, each owning 2 of the
//     slot's 4 queries) pull their 128 logits per key with four tcgen05.ld in
//     flight and one wait, release the accumulator at once, then apply relu,
//     reduce over heads with the per-query weights (fixed head order) and
//     store coalesced score rows -- while the MMA warp already fills the slot
//     again.
// Bounded waits and drains as in matmul_tcgen05.cu.  No cluster multicast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "device.hpp"
#include "tc_common.cuh"

namespace ptowsp::dev {

namespace {

using namespace tc;

constexpr int KT = 128;           // keys per tile (MMA M)
constexpr int QH = 512;           // q rows per task (8 queries x 64 heads)
constexpr int NH = 256;           // q rows per MMA (N)
constexpr int HEADS = 64;
constexpr int D = 128;
constexpr int STAGES = 3;
constexpr int EPI_WARPS = 8;      // two per TMEM lane quarter, each taking 2 of a slot's 4 queries
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int Q_BYTES = QH * D * 2;        // 128 KB
constexpr int Q_BOX = NH * 64 * 2;         // 32 KB: 256 rows x 64 d
constexpr int K_STAGE = KT * D * 2;        // 32 KB: two 16 KB boxes of 128 keys x 64 d
constexpr int K_BOX = KT * 64 * 2;
constexpr int BAR_OFF = Q_BYTES + STAGES * K_STAGE;
constexpr int SMEM = BAR_OFF + 256 + 1024;
constexpr int TMEM_COLS = 512;

struct IdxArgs {
    const int64_t* rec;
    int64_t ntasks;
    int stride;
    int tiles;                   // key tiles per task
    const float* w;              // weights base
    int64_t w_s3;
    float* s;                    // scores base
    int64_t s_s3;
    int queries;                 // 8
    int* err;
};

__global__ void __launch_bounds__(THREADS, 1)
    indexer_score_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                         IdxArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* qs = smem;
    uint8_t* ks = smem + Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* qfull = bars + 2 * STAGES + 4;
    uint64_t* qempty = bars + 2 * STAGES + 5;
    uint64_t* drain = bars + 2 * STAGES + 6;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 7);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), EPI_WARPS * 32);
        }
        mbar_init(smem_u32(qfull), 1);
        mbar_init(smem_u32(qempty), 1);
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_k)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int64_t U = args.ntasks * args.tiles;
    const int64_t u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_parity = 0;
            int64_t cur = -1;
            uint32_t nswitch = 0;
            bool q_loaded = false;
            for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
                const int64_t task = u / args.tiles;
                const int tile = static_cast<int>(u % args.tiles);
                const int64_t* rec = args.rec + task * args.stride;
                if (task != cur) {
                    if (nswitch > 0 && !mbar_wait(smem_u32(qempty), (nswitch - 1) & 1u, abort_flag, args.err)) break;
                    const uint32_t qb = smem_u32(qfull);
                    mbar_expect_tx(qb, Q_BYTES);
                    const int32_t qrow = static_cast<int32_t>(rec[0] / D);
#pragma unroll
                    for (int hq = 0; hq < 2; ++hq)
#pragma unroll
                        for (int dh = 0; dh < 2; ++dh)
                            tma_load_2d(smem_u32(qs + (hq * 2 + dh) * Q_BOX), &tmap_q, dh * 64, qrow + hq * NH, qb);
                    q_loaded = true;
                    ++nswitch;
                    cur = task;
                }
                if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, args.err)) break;
                const uint32_t fb = smem_u32(&full[stage]);
                mbar_expect_tx(fb, K_STAGE);
                const int32_t krow = static_cast<int32_t>(rec[1] / D) + tile * KT;
#pragma unroll
                for (int dh = 0; dh < 2; ++dh)
                    tma_load_2d(smem_u32(ks + stage * K_STAGE + dh * K_BOX), &tmap_k, dh * 64, krow, fb);
                issued_mask |= 1u << stage;
                last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            // drain the copies this CTA issued
            const uint64_t start = globaltimer();
            for (int s = 0; s < STAGES; ++s)
                if (issued_mask & (1u << s))
                    while (!mbar_try_wait(smem_u32(&full[s]), (last_parity >> s) & 1u))
                        if (globaltimer() - start > kTimeoutNs) {
                            atomicOr(args.err, kErrTimeout);
                            break;
                        }
            if (q_loaded)
                while (!mbar_try_wait(smem_u32(qfull), (nswitch - 1) & 1u))
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        break;
                    }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(KT, NH, 0);
            int stage = 0, slot = 0;
            uint32_t phase = 0, slot_phase = 0;
            int64_t cur = -1;
            uint32_t nswitch = 0;
            bool issued = false;
            for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
                const int64_t task = u / args.tiles;
                if (task != cur) {
                    if (!mbar_wait(smem_u32(qfull), nswitch & 1u, abort_flag, args.err)) break;
                    ++nswitch;
                    cur = task;
                }
                if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, args.err)) break;
                tc_fence_after();
                const uint32_t ka = smem_u32(ks + stage * K_STAGE);
                bool ok = true;
                for (int hq = 0; hq < 2; ++hq) {
                    if (!mbar_wait(smem_u32(&tempty[slot]), slot_phase ^ 1u, abort_flag, args.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * NH);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint64_t ad = smem_desc(ka + (kk >> 2) * K_BOX + (kk & 3) * 32, 16, 1024);
                        const uint64_t bd = smem_desc(smem_u32(qs + (hq * 2 + (kk >> 2)) * Q_BOX) + (kk & 3) * 32, 16, 1024);
                        mma_f16(d_tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(smem_u32(&tfull[slot]));
                    issued = true;
                    if (++slot == 2) {
                        slot = 0;
                        slot_phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(smem_u32(&empty[stage]));
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (u + 1 == u1 || (u + 1) / args.tiles != task) mma_commit(smem_u32(qempty));
            }
            if (issued) {
                mma_commit(smem_u32(drain));
                const uint64_t start = globaltimer();
                while (!mbar_try_wait(smem_u32(drain), 0))
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        break;
                    }
            }
        }
    } else {
        const int quarter = warp & 3;       // the TMEM lanes (keys) this warp may read
        const int half = (warp - 2) >> 2;   // queries 2*half and 2*half+1 of each 4-query slot
        const int row = quarter * 32 + lane;
        int slot = 0;
        uint32_t slot_phase = 0;
        for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
            const int64_t task = u / args.tiles;
            const int tile = static_cast<int>(u % args.tiles);
            const int64_t* rec = args.rec + task * args.stride;
            const float* w = args.w + rec[2];
            float* s = args.s + rec[3] + static_cast<int64_t>(tile) * KT + row;
            bool ok = true;
            for (int hq = 0; hq < 2; ++hq) {
                if (!mbar_wait(smem_u32(&tfull[slot]), slot_phase, abort_flag, args.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // this warp's 2 queries x 64 heads: four 32-column loads in flight, one wait
                uint32_t v[4][32];
                const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(slot * NH + half * 2 * HEADS);
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32_async(tbase + static_cast<uint32_t>(c * 32), v[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 4; ++c) reg_fence(v[c]);
                tc_fence_before();
                mbar_arrive(smem_u32(&tempty[slot]));  // the accumulator is in registers: release it
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const int q = hq * 4 + half * 2 + qq;
                    const float4* wq = reinterpret_cast<const float4*>(w + q * args.w_s3);
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // four partial sums over heads h = 4j + c, j ascending
#pragma unroll
                    for (int hc = 0; hc < 2; ++hc) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 wv = __ldg(wq + hc * 8 + j);  // same address in every lane: one L1 broadcast
                            const uint32_t* x = &v[2 * qq + hc][4 * j];
                            acc[0] = fmaf(wv.x, fmaxf(__uint_as_float(x[0]), 0.f), acc[0]);
                            acc[1] = fmaf(wv.y, fmaxf(__uint_as_float(x[1]), 0.f), acc[1]);
                            acc[2] = fmaf(wv.z, fmaxf(__uint_as_float(x[2]), 0.f), acc[2]);
                            acc[3] = fmaf(wv.w, fmaxf(__uint_as_float(x[3]), 0.f), acc[3]);
                        }
                    }
                    s[q * args.s_s3] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
                }
                if (++slot == 2) {
                    slot = 0;
                    slot_phase ^= 1u;
                }
            }
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
}

// ---------------------------------------------------------------------------
// CTA-pair variant (the default when the key count is a multiple of 256).
//
// Two CTAs of a 2-CTA cluster, on two SMs, share each MMA (tcgen05 cta_group::2,
// M = 256 keys: 128 per CTA; N = 256 q rows: each CTA holds the 128 q rows of its
// half of N).  Every CTA therefore keeps only half of the batch's q rows (64 KB)
// and streams only its own 128 keys per unit, and each SM's tensor core reads
// half of the B operand per MMA -- the one-CTA form reads all of it and stalls on
// that.  The freed shared memory deepens the key ring to 4 stages.
//
//   * both CTAs' TMA loads count their bytes on the leader CTA's (rank 0) full /
//     q barriers (a shared::cluster address), the leader alone posts the expected
//     byte counts and issues the MMAs;
//   * MMA completion is committed to the barrier of each CTA that waits for it
//     (accumulator full, ring stage free, q rows free);
//   * each CTA's 16 epilogue warps (four per TMEM lane quarter, one query of the
//     slot each) read their own TMEM (the CTA's 128 keys x 256 columns); one
//     lane per epilogue warp of either CTA releases the accumulator on the
//     leader's barrier (32 arrivals per phase);
//   * a cluster barrier after setup (barriers initialised, TMEM allocated) and
//     before teardown (the leader has drained every copy and MMA of the pair);
//     every wait before it is bounded, so both CTAs always reach it.
// ---------------------------------------------------------------------------

constexpr int P_KT = 128;                         // keys per CTA per unit; the pair covers 256
constexpr int P_UNIT = 2 * P_KT;
constexpr int P_STAGES = 4;
constexpr int P_QBOX = 128 * 64 * 2;              // 16 KB: 128 q rows x 64 d
constexpr int P_Q_BYTES = 4 * P_QBOX;             // 64 KB: this CTA's q rows of both slots, both d halves
constexpr int P_K_STAGE = P_KT * D * 2;           // 32 KB: two 16 KB boxes of 128 keys x 64 d
constexpr int P_BAR_OFF = P_Q_BYTES + P_STAGES * P_K_STAGE;
constexpr int P_SMEM = P_BAR_OFF + 256 + 1024;
constexpr int P_EPI_WARPS = 16;                   // four per TMEM lane quarter, one query of the slot each
constexpr int P_THREADS = 64 + 32 * P_EPI_WARPS;

__global__ void __launch_bounds__(P_THREADS, 1)
    indexer_score_pair_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                              IdxArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* qs = smem;
    uint8_t* ks = smem + P_Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_BAR_OFF);
    uint64_t* full = bars;                          // [P_STAGES]  used in the leader
    uint64_t* empty = bars + P_STAGES;              // [P_STAGES]  both CTAs
    uint64_t* tfull = bars + 2 * P_STAGES;          // [2]         both CTAs
    uint64_t* tempty = bars + 2 * P_STAGES + 2;     // [2]         used in the leader
    uint64_t* qfull = bars + 2 * P_STAGES + 4;      //             used in the leader
    uint64_t* qempty = bars + 2 * P_STAGES + 5;     //             both CTAs
    uint64_t* drain = bars + 2 * P_STAGES + 6;      //             leader
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * P_STAGES + 7);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 8);

    const uint32_t rank = cluster_ctarank();  // 0: leader
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), 2 * P_EPI_WARPS);
        }
        mbar_init(smem_u32(qfull), 1);
        mbar_init(smem_u32(qempty), 1);
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_k)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
    // a kernel launched after this one as a programmatic dependent (the top-k) may be scheduled now; it waits
    // for this grid's completion before it reads a score
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t lead_bars = mapa_shared(smem_u32(bars), 0);  // the leader's barrier block
    const uint32_t peer_bars = mapa_shared(smem_u32(bars), 1);
    auto lead = [&](const uint64_t* b) { return lead_bars + static_cast<uint32_t>((b - bars) * 8); };
    auto peer = [&](const uint64_t* b) { return peer_bars + static_cast<uint32_t>((b - bars) * 8); };

    const int64_t npairs = gridDim.x >> 1, pair = blockIdx.x >> 1;
    const int64_t U = args.ntasks * args.tiles;  // units of 256 keys
    const int64_t u0 = U * pair / npairs, u1 = U * (pair + 1) / npairs;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_parity = 0;
            int64_t cur = -1;
            uint32_t nswitch = 0;
            for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
                const int64_t task = u / args.tiles;
                const int tile = static_cast<int>(u % args.tiles);
                const int64_t* rec = args.rec + task * args.stride;
                if (task != cur) {
                    if (nswitch > 0 && !mbar_wait(smem_u32(qempty), (nswitch - 1) & 1u, abort_flag, args.err)) break;
                    if (rank == 0) mbar_expect_tx(smem_u32(qfull), 2 * P_Q_BYTES);
                    const int32_t qrow = static_cast<int32_t>(rec[0] / D) + static_cast<int32_t>(rank) * 128;
#pragma unroll
                    for (int hq = 0; hq < 2; ++hq)
#pragma unroll
                        for (int dh = 0; dh < 2; ++dh)
                            tma_load_2d_pair(smem_u32(qs + (hq * 2 + dh) * P_QBOX), &tmap_q, dh * 64, qrow + hq * NH,
                                             lead(qfull));
                    ++nswitch;
                    cur = task;
                }
                if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, args.err)) break;
                if (rank == 0) mbar_expect_tx(smem_u32(&full[stage]), 2 * P_K_STAGE);
                const int32_t krow = static_cast<int32_t>(rec[1] / D) + tile * P_UNIT + static_cast<int32_t>(rank) * P_KT;
#pragma unroll
                for (int dh = 0; dh < 2; ++dh)
                    tma_load_2d_pair(smem_u32(ks + stage * P_K_STAGE + dh * K_BOX), &tmap_k, dh * 64, krow, lead(&full[stage]));
                issued_mask |= 1u << stage;
                last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == P_STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (rank == 0) {
                // drain: the pair's last copy into each stage (and the last q rows) have landed
                const uint64_t start = globaltimer();
                for (int s = 0; s < P_STAGES; ++s)
                    if (issued_mask & (1u << s))
                        while (!mbar_try_wait(smem_u32(&full[s]), (last_parity >> s) & 1u))
                            if (globaltimer() - start > kTimeoutNs) {
                                atomicOr(args.err, kErrTimeout);
                                break;
                            }
                if (nswitch > 0)
                    while (!mbar_try_wait(smem_u32(qfull), (nswitch - 1) & 1u))
                        if (globaltimer() - start > kTimeoutNs) {
                            atomicOr(args.err, kErrTimeout);
                            break;
                        }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_f16(P_UNIT, NH, 0);  // M = 256 over the pair, N = 256, B K-major
            int stage = 0, slot = 0;
            uint32_t phase = 0, slot_phase = 0;
            int64_t cur = -1;
            uint32_t nswitch = 0;
            bool issued = false;
            for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
                const int64_t task = u / args.tiles;
                if (task != cur) {
                    if (!mbar_wait(smem_u32(qfull), nswitch & 1u, abort_flag, args.err)) break;
                    ++nswitch;
                    cur = task;
                }
                if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, args.err)) break;
                tc_fence_after();
                const uint32_t ka = smem_u32(ks + stage * P_K_STAGE);
                bool ok = true;
                for (int hq = 0; hq < 2; ++hq) {
                    if (!mbar_wait(smem_u32(&tempty[slot]), slot_phase ^ 1u, abort_flag, args.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * NH);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint64_t ad = smem_desc(ka + (kk >> 2) * K_BOX + (kk & 3) * 32, 16, 1024);
                        const uint64_t bd = smem_desc(smem_u32(qs + (hq * 2 + (kk >> 2)) * P_QBOX) + (kk & 3) * 32, 16, 1024);
                        mma_f16_pair(d_tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
                    }
                    mma_commit_pair(lead(&tfull[slot]));
                    mma_commit_pair(peer(&tfull[slot]));
                    issued = true;
                    if (++slot == 2) {
                        slot = 0;
                        slot_phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair(lead(&empty[stage]));
                mma_commit_pair(peer(&empty[stage]));
                if (++stage == P_STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (u + 1 == u1 || (u + 1) / args.tiles != task) {
                    mma_commit_pair(lead(qempty));
                    mma_commit_pair(peer(qempty));
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
        const int quarter = warp & 3;     // the TMEM lanes (keys) this warp may read
        const int ql = (warp - 2) >> 2;   // the query of each 4-query slot this warp reduces
        const int row = quarter * 32 + lane;
        int slot = 0;
        uint32_t slot_phase = 0;
        for (int64_t u = u0; u < u1 && !*abort_flag; ++u) {
            const int64_t task = u / args.tiles;
            const int tile = static_cast<int>(u % args.tiles);
            const int64_t* rec = args.rec + task * args.stride;
            const float* w = args.w + rec[2];
            float* s = args.s + rec[3] + static_cast<int64_t>(tile) * P_UNIT + static_cast<int64_t>(rank) * P_KT + row;
            bool ok = true;
            for (int hq = 0; hq < 2; ++hq) {
                if (!mbar_wait(smem_u32(&tfull[slot]), slot_phase, abort_flag, args.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // this warp's query: 64 heads in two 32-column loads, one wait
                uint32_t v[2][32];
                const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(slot * NH + ql * HEADS);
                tmem_ld32_async(tbase, v[0]);
                tmem_ld32_async(tbase + 32u, v[1]);
                tmem_wait_ld();
                reg_fence(v[0]);
                reg_fence(v[1]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(lead(&tempty[slot]));  // accumulator in registers: release it
                const int q = hq * 4 + ql;
                const float4* wq = reinterpret_cast<const float4*>(w + q * args.w_s3);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};  // four partial sums over heads h = 4j + c, j ascending
#pragma unroll
                for (int hc = 0; hc < 2; ++hc) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 wv = __ldg(wq + hc * 8 + j);  // same address in every lane: one L1 broadcast
                        const uint32_t* x = &v[hc][4 * j];
                        acc[0] = fmaf(wv.x, fmaxf(__uint_as_float(x[0]), 0.f), acc[0]);
                        acc[1] = fmaf(wv.y, fmaxf(__uint_as_float(x[1]), 0.f), acc[1]);
                        acc[2] = fmaf(wv.z, fmaxf(__uint_as_float(x[2]), 0.f), acc[2]);
                        acc[3] = fmaf(wv.w, fmaxf(__uint_as_float(x[3]), 0.f), acc[3]);
                    }
                }
                s[q * args.s_s3] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
                if (++slot == 2) {
                    slot = 0;
                    slot_phase ^= 1u;
                }
            }
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader has drained the pair's copies and MMAs; no cross-CTA access after this
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
}

}  // namespace

bool indexer_score_supported(const TaskBatch& b) {
    const ParamDesc& Q = b.p[0];
    const ParamDesc& K = b.p[1];
    const ParamDesc& W = b.p[2];
    const ParamDesc& S = b.p[3];
    if (Q.rows != QH || Q.cols != D || K.cols != D || K.rows % KT || W.rows != 8 || W.cols != HEADS) return false;
    if (S.rows != 8 || S.cols != K.rows) return false;
    if (W.s3 % 4 || (reinterpret_cast<uintptr_t>(W.base) & 15)) return false;  // float4 weight rows
    if (Q.s3 != D || K.s3 != D || Q.s4 != 1 || K.s4 != 1 || W.s4 != 1 || S.s4 != 1) return false;
    if ((reinterpret_cast<uintptr_t>(Q.base) | reinterpret_cast<uintptr_t>(K.base)) & 15) return false;
    return true;
}

namespace {

// CTA-pair launch; false (nothing launched) when the pairs cannot be scheduled.
bool launch_indexer_pairs(const TaskBatch& b, int workers, cudaStream_t s, cudaError_t* err) {
    const ParamDesc& Q = b.p[0];
    const ParamDesc& K = b.p[1];
    if (K.rows % P_UNIT) return false;
    CUtensorMap mq, mk;
    if (!make_map_f16(&mq, Q.base, D, (Q.numel_span + D - 1) / D, 64, 128)) return false;
    if (!make_map_f16(&mk, K.base, D, (K.numel_span + D - 1) / D, 64, P_KT)) return false;
    IdxArgs a;
    a.rec = b.rec;
    a.ntasks = b.ntasks;
    a.stride = b.stride;
    a.tiles = K.rows / P_UNIT;
    a.w = reinterpret_cast<const float*>(b.p[2].base);
    a.w_s3 = b.p[2].s3;
    a.s = reinterpret_cast<float*>(b.p[3].base);
    a.s_s3 = b.p[3].s3;
    a.queries = 8;
    a.err = b.err;
    if (cudaFuncSetAttribute(indexer_score_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = P_SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int64_t pairs = std::max<int64_t>(1, sm_count() / 2);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    int resident = 0;  // pairs that fit on the GPU at once: the persistent schedule needs all of them resident
    if (cudaOccupancyMaxActiveClusters(&resident, indexer_score_pair_kernel, &cfg) != cudaSuccess || resident < 1) {
        cudaGetLastError();
        return false;
    }
    pairs = std::min<int64_t>({pairs, resident, b.ntasks * a.tiles});
    if (workers > 0) pairs = std::min<int64_t>(pairs, std::max(1, workers / 2));
    pairs = std::max<int64_t>(pairs, 1);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    *err = cudaLaunchKernelEx(&cfg, indexer_score_pair_kernel, mq, mk, a);
    return true;
}

}  // namespace

cudaError_t launch_indexer_score(const TaskBatch& b, int workers, cudaStream_t s) {
    if (!indexer_score_supported(b)) return cudaErrorInvalidValue;
    cudaError_t pe = cudaSuccess;
    if (launch_indexer_pairs(b, workers, s, &pe)) return pe;
    const ParamDesc& Q = b.p[0];
    const ParamDesc& K = b.p[1];
    CUtensorMap mq, mk;
    if (!make_map_f16(&mq, Q.base, D, (Q.numel_span + D - 1) / D, 64, NH)) return cudaErrorInvalidValue;
    if (!make_map_f16(&mk, K.base, D, (K.numel_span + D - 1) / D, 64, KT)) return cudaErrorInvalidValue;
    IdxArgs a;
    a.rec = b.rec;
    a.ntasks = b.ntasks;
    a.stride = b.stride;
    a.tiles = K.rows / KT;
    a.w = reinterpret_cast<const float*>(b.p[2].base);
    a.w_s3 = b.p[2].s3;
    a.s = reinterpret_cast<float*>(b.p[3].base);
    a.s_s3 = b.p[3].s3;
    a.queries = 8;
    a.err = b.err;
    cudaError_t e = cudaFuncSetAttribute(indexer_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    const int64_t units = b.ntasks * a.tiles;
    int64_t grid = std::min<int64_t>(units, sm_count());
    if (workers > 0) grid = std::min<int64_t>(grid, workers);
    grid = std::max<int64_t>(grid, 1);
    indexer_score_kernel<<<static_cast<unsigned>(grid), THREADS, SMEM, s>>>(mq, mk, a);
    return cudaGetLastError();
}

}  // namespace ptowsp::dev
