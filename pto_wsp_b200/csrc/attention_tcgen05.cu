// Fused attention tile task on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), flash form.
//
// A task is a generic `pto.*` kernel of the shape the reference attention example writes
// (examples/attention/pto_wsp_impl.py:51-68; emitter ops src/python/pto_codegen.cpp:817-1219):
//
//     S = Q . K^T  [* scale]      Q [128, 128] f16, K^T [128, L] f16 (the task's tile views)
//     W = exp(S - rowmax(S)) / rowsum(...)     f32
//     O = W . V                   V [L, 128] f32, O [128, 128] f32 (stored to the `out` view)
//
// (pto has no cast, so W, the f32 result of the softmax, multiplies an f32 V: the emitter takes a matmul only with
// both operands f16 or both f32.)  The staged form runs this as four launches with S and W in HBM scratch and the
// second contraction on CUDA cores; here S and O live in TMEM and W in shared memory, and both contractions run
// on the tensor cores:
//   * S_j = Q . K^T_j: tcgen05.mma kind::f16 (exact f16 products, f32 accumulation);
//   * O += W_j . V_j: kind::f16 on f16 operands in a three-term split, P_hi.V_hi + P_hi.V_lo + P_lo.V_hi, where
//     x_hi = x with its low 13 mantissa bits cleared (an exact f16) and x_lo = f16(x - x_hi): the pair carries
//     ~22 bits of x, so every product keeps the f32 tile program's accuracy (one f16 pass would leave 2^-11
//     relative error per term; a bf16 split, 2^-17).  f16's exponent range is narrow, so both operands are scaled by powers of two: P (at most
//     2^8, see the lazy max below) by 2^7, and V by 2^k with k chosen from the largest |V| seen so far in the
//     task (|V| 2^k < 2^15).  A V block that raises that maximum lowers k, and O is rescaled by the exact power
//     of two before the block's terms accumulate; values far below the maximum lose only bits far below the
//     result's rounding.  The twelve MMAs per block (M = N = 128, K = 16) run at the f16 tensor rate.  P is the
//     A operand straight from TMEM (packed f16 pairs written over the S block it came from), V the B operand
//     from shared memory in its own row-major layout (MN-major).
// Keys go in blocks of 64 (S in blocks of 128: the N = 128 MMA reads Q once for two key blocks and runs at twice the
// rate of N = 64, whose operand reads saturate shared memory) with an online softmax in the base-2 domain; the running row max is kept lazily (a row's O
// and sum are rescaled only when its max grows by more than 2^8), which changes no result beyond rounding.  The row
// sum uses the f32 probabilities and divides O once at the end, together with the two scales.
//
// One CTA per task, 10 warps:
//   warp 0      TMA producer: Q once (two 128 x 64 K-major f16 boxes), per S block the K^T of its two key blocks
//               (four 64 x 64 MN-major f16 boxes, two stages of 32 KB), 128-byte swizzle.
//   warp 1      owns TMEM (three S/P buffers of 128 columns: S block J in buffer J % 3, key block j's S in its
//               columns 64 (j % 2) .. +63, then [P_hi | P_lo] over those 64, two f16 per column; O: columns
//               384-511) and issues the MMAs from one thread, S blocks up to three ahead:
//               S_0 S_1 S_2 PV_0 PV_1 S_3 PV_2 PV_3 S_4 ...  The softmax never waits for an S.  S block J+3 reuses
//               buffer J % 3: it is issued after PV_{2J+1}, and the tensor pipe runs one thread's MMAs in order, so
//               both P.V blocks have read their P before S block J+3 lands.
//   warps 2-5   softmax and epilogue, one row per thread (warp w reads TMEM lanes 32 (w % 4) ..): tcgen05.ld of
//               the S row into registers, max, exponentials, P_hi / P_lo stored into the row's TMEM lane with
//               tcgen05.st (and O rescaled in TMEM when the row max or V's scale moves); at the end O / sum
//               stored to the out row.
//   warps 6-9   read each V block from global memory (the next one's loads in flight), find its largest |V|,
//               scale it, split it into f16 V_hi / V_lo and write both in the 128-byte-swizzled row layout the
//               MMA reads (two buffers, so the next block's split overlaps this block's MMAs).
// Every mbarrier wait is bounded (~2 s of %globaltimer): on timeout the CTA records kErrTimeout, drains its own
// copies and MMAs, frees TMEM and returns.  No cluster multicast (loads read this GPU's memory only).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "device.hpp"
#include "tc_common.cuh"

namespace ptowsp::dev {

namespace {

using namespace tc;

constexpr int AT_THREADS = 320;
constexpr int AT_ROWS = 128;   // query rows of a task
constexpr int AT_D = 128;      // head dim
constexpr int AT_BN = 64;      // keys per block (softmax, V split, P.V)
constexpr int AT_SN = 128;     // keys per S block: two key blocks in one N = 128 MMA chain
constexpr int BOX = 8192;      // one TMA box / one V chunk: 64 x 64 16-bit elements, 128-byte rows
constexpr int Q_BYTES = AT_ROWS * AT_D * 2;   // 32 KB
constexpr int K_BYTES = AT_D * AT_BN * 2;     // 16 KB: the K^T of one key block
constexpr int KS_BYTES = 2 * K_BYTES;         // 32 KB per stage: one S block's two key blocks, 16 KB apart
constexpr int V_BYTES = AT_BN * AT_D * 2;     // 16 KB: one f16 part of a V block (two 64-dim chunks)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int KST = 2;                        // K^T stages (S blocks of 128 keys)
constexpr int NVB = 4;                        // V buffers: the splitters run up to four blocks ahead of the MMAs
constexpr int OFF_VSP = OFF_K + KST * KS_BYTES;  // NVB buffers of [V_hi | V_lo]
constexpr int VSP_BYTES = 2 * V_BYTES;
constexpr int OFF_BAR = OFF_VSP + NVB * VSP_BYTES;  // 224 KB
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;  // + barriers / flags / V scales + 1024-byte alignment slack
static_assert(SMEM_BYTES <= 232448, "attention tile exceeds the 227 KB of shared memory per CTA");
// TMEM columns: three S/P buffers of 128 (S block J, key blocks 2J and 2J+1, in buffer J % 3; key block j's S in
// the 64 columns at 64 (j % 2), and P_j, [P_hi | P_lo] with two f16 keys per column, over them once S_j has been
// read), O 384-511
constexpr int SPB = 3;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_SP = 128;  // columns per S/P buffer
constexpr uint32_t TMEM_O = 384;
constexpr float kRescaleLog2 = 8.f;  // a row's reference max moves when its max grows by more than this
constexpr int kPScaleLog2 = 7;       // P (at most 2^8) enters the MMA as P * 2^7 (< 2^15, inside f16's range)
constexpr int kVScaleMax = 100;      // V's scale 2^k keeps |k| <= 100 (all-zero or non-finite blocks included)

// One S block, S_J = Q . K^T_J over the 128 head dims: eight kind::f16 MMAs (M = 128, N = 128 -- two key blocks --
// or 64 for a last lone key block, from `idesc`, K = 16) in one asm block, so that the single issuing thread
// spends one add per operand per MMA.  `a` is the descriptor of Q's first 16 dims (K-major, 128-byte swizzle: +32 B
// per 16 dims inside a 64-dim box, +16 KB per box), `b` that of the K^T stage's first 16 dims (MN-major: +2 KB per
// 16 dims, +8 KB per box, the second key block 16 KB on as the descriptor's leading offset); descriptor address
// fields count 16-byte units.  The first MMA overwrites D (`accum` = 0), the rest accumulate.
__device__ __forceinline__ void mma_s_block(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .b64 bd;\n\t"
        ".reg .b64 ad;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.b32 q, %4, %4;\n\t"
        "add.s64 ad, %1, 0;\n\tadd.s64 bd, %2, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, p;\n\t"
        "add.s64 ad, %1, 2;\n\tadd.s64 bd, %2, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 4;\n\tadd.s64 bd, %2, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 6;\n\tadd.s64 bd, %2, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 1024;\n\tadd.s64 bd, %2, 512;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 1026;\n\tadd.s64 bd, %2, 640;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 1028;\n\tadd.s64 bd, %2, 768;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;\n\t"
        "add.s64 ad, %1, 1030;\n\tadd.s64 bd, %2, 896;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, q;}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

// O += P_j . V_j over the block's 64 keys as three terms, P_lo.V_hi + P_hi.V_lo + P_hi.V_hi, each four kind::f16
// MMAs (M = N = 128, K = 16) on f16 operands: A from TMEM (`p_tmem`: P_hi in columns 0-31, P_lo in 32-63, two
// keys per column, 8 columns per MMA), B from shared memory (`vh` / `vl`: the V_hi / V_lo descriptors, MN-major,
// 128-byte swizzle, 64-dim chunks 8 KB apart, +2 KB per 16 keys).  The first MMA accumulates only if `accum` is set.
__device__ __forceinline__ void mma_pv_block(uint32_t d_tmem, uint32_t p_tmem, uint64_t vh, uint64_t vl, uint32_t idesc,
                                             uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .b64 bd;\n\t"
        ".reg .b32 ta;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 q, %5, %5;\n\t"
        "add.u32 ta, %1, 32;\n\tadd.s64 bd, %2, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, p;\n\t"
        "add.u32 ta, %1, 40;\n\tadd.s64 bd, %2, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 48;\n\tadd.s64 bd, %2, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 56;\n\tadd.s64 bd, %2, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 0;\n\tadd.s64 bd, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 8;\n\tadd.s64 bd, %3, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 16;\n\tadd.s64 bd, %3, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 24;\n\tadd.s64 bd, %3, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 0;\n\tadd.s64 bd, %2, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 8;\n\tadd.s64 bd, %2, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 16;\n\tadd.s64 bd, %2, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;\n\t"
        "add.u32 ta, %1, 24;\n\tadd.s64 bd, %2, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %4, q;}"
        ::"r"(d_tmem), "r"(p_tmem), "l"(vh), "l"(vl), "r"(idesc), "r"(accum)
        : "memory");
}

// Two f32 values rounded to f16 and packed into one 32-bit word, `lo` in the low half (the lower key / dim).
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// x with its low 13 mantissa bits cleared: 11 significant bits, exactly an f16 value inside f16's normal range.  The
// split x = hi + (x - hi) then needs no conversion back from f16: hi packs exactly, and x - hi (exact in f32,
// below 2^-10 |x|) loses only bits under 2^-21 |x| when it is rounded to f16.
__device__ __forceinline__ float f16_hi_part(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error ~2^-22, results below 2^-126 flush to
// zero).  The probabilities it makes stay far inside the contraction's 2e-3 bar, and it is a quarter of the cost
// of exp2f(), which dominated the softmax warps' time per key block.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^e as an f32 for -126 <= e <= 127 (exact; no exp2 evaluation).
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// tcgen05.st of 16 columns of this warp's 32 TMEM lanes (one register per lane and column).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// V's scale exponent for a largest |V| whose f32 bits are `mbits` (a non-negative float; NaN sorts above inf): the
// k with |V| 2^k < 2^15, clamped to [-kVScaleMax, kVScaleMax].
__device__ __forceinline__ int v_scale_log2(uint32_t mbits) {
    const int be = static_cast<int>(min(mbits, 0x7f800000u) >> 23);  // |V| < 2^(be - 126)
    return max(-kVScaleMax, min(kVScaleMax, 141 - be));
}

struct AttnArgs {
    const int64_t* rec;
    int64_t ntasks;
    int stride;
    int q_p, kt_p, v_p, o_p;      // tensor param positions in the records
    int64_t q_pitch, kt_pitch, v_pitch;
    const float* v;               // V base (the splitters read it directly)
    float* out;
    int64_t o_pitch;
    int nblocks;                  // L / 64
    int scale_mode;               // 0 none, 1 constant, 2 f32 bits in the record at scale_pos
    int scale_pos;
    float scale_const;
    int* err;
};

__global__ void __launch_bounds__(AT_THREADS, 1)
    attention_tcgen05_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mkt,
                             AttnArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = q_full + 1;          // [KST]
    uint64_t* k_empty = k_full + KST;       // [KST]
    uint64_t* vsp_full = k_empty + KST;     // [NVB] V_hi / V_lo written
    uint64_t* vsp_empty = vsp_full + NVB;   // [NVB] the MMAs read them
    uint64_t* s_full = vsp_empty + NVB;     // [3] S block J in buffer J % 3
    uint64_t* p_full = s_full + SPB;        // [6] P_j written over S_j (key block j: j % 6)
    uint64_t* pv_done = p_full + 2 * SPB;   // [2] O holds block j's contribution
    uint64_t* o_full = pv_done + 2;
    uint64_t* drain = o_full + 1;
    uint64_t* vmax_ready = drain + 1;       // [2] the four splitter warps posted their parts of a block's largest |V|
    volatile int* abort_flag = reinterpret_cast<volatile int*>(vmax_ready + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(vmax_ready + 3);
    volatile int* v_log2 = reinterpret_cast<volatile int*>(vmax_ready + 4);         // [NVB] V's scale exponent of buffer b
    uint32_t* v_part = reinterpret_cast<uint32_t*>(vmax_ready + 4 + (NVB + 1) / 2);  // [2][4] splitter warps' largest |V| bits
    static_assert((1 + 2 * KST + 2 * NVB + 3 * SPB + 8 + (NVB + 1) / 2 + 4) * 8 <= 512, "barrier block exceeds its 512 bytes");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t task = blockIdx.x;
    if (task >= args.ntasks) return;  // whole CTA: nothing initialised yet
    const int64_t* rec = args.rec + task * args.stride;
    const int nb = args.nblocks;
    const int ns = (nb + 1) / 2;  // S blocks

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(q_full), 1);
        for (int s = 0; s < KST; ++s) {
            mbar_init(smem_u32(&k_full[s]), 1);
            mbar_init(smem_u32(&k_empty[s]), 1);
        }
        for (int s = 0; s < SPB; ++s) mbar_init(smem_u32(&s_full[s]), 1);
        for (int s = 0; s < 2 * SPB; ++s) mbar_init(smem_u32(&p_full[s]), 128);
        for (int s = 0; s < NVB; ++s) {
            mbar_init(smem_u32(&vsp_full[s]), 128);
            mbar_init(smem_u32(&vsp_empty[s]), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&pv_done[s]), 1);
        }
        mbar_init(smem_u32(o_full), 1);
        for (int s = 0; s < 2; ++s) mbar_init(smem_u32(&vmax_ready[s]), 4);
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mq)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mkt)) : "memory");
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
    const uint32_t sQ = smem_u32(smem + OFF_Q), sK = smem_u32(smem + OFF_K);
    const uint32_t sVsp = smem_u32(smem + OFF_VSP);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            const int64_t oq = rec[args.q_p], okt = rec[args.kt_p];
            const int32_t qx = static_cast<int32_t>(oq % args.q_pitch), qy = static_cast<int32_t>(oq / args.q_pitch);
            const int32_t kx = static_cast<int32_t>(okt % args.kt_pitch), ky = static_cast<int32_t>(okt / args.kt_pitch);
            mbar_expect_tx(smem_u32(q_full), Q_BYTES);
            tma_load_2d(sQ, &mq, qx, qy, smem_u32(q_full));
            tma_load_2d(sQ + 16384, &mq, qx + 64, qy, smem_u32(q_full));
            int last_k[KST];  // the S block last loaded into each stage
            for (int st = 0; st < KST; ++st) last_k[st] = -1;
            for (int jp = 0; jp < ns && !*abort_flag; ++jp) {
                const int st = jp % KST;
                if (jp >= KST && !mbar_wait(smem_u32(&k_empty[st]), ((jp / KST) & 1) ^ 1u, abort_flag, args.err)) break;
                const int nk = min(2, nb - 2 * jp);  // key blocks in this S block
                mbar_expect_tx(smem_u32(&k_full[st]), nk * K_BYTES);
                for (int h = 0; h < nk; ++h)
                    for (int kc = 0; kc < 2; ++kc)  // head-dim rows of K^T, 64 keys per box
                        tma_load_2d(sK + st * KS_BYTES + h * K_BYTES + kc * BOX, &mkt, kx + (2 * jp + h) * AT_BN,
                                    ky + kc * 64, smem_u32(&k_full[st]));
                last_k[st] = jp;
            }
            // drain: every copy issued has landed before shared memory goes away (S block J completes phase
            // J / KST of its stage's barrier)
            const uint64_t start = globaltimer();
            auto settle = [&](uint32_t bar, uint32_t parity) {
                while (!mbar_try_wait(bar, parity))
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        return;
                    }
            };
            settle(smem_u32(q_full), 0);
            for (int st = 0; st < KST; ++st)
                if (last_k[st] >= 0) settle(smem_u32(&k_full[st]), (last_k[st] / KST) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc_s = idesc_f16(AT_ROWS, AT_SN, 1);  // A K-major, B MN-major, M = 128, N = 128
            constexpr uint32_t idesc_s1 = idesc_f16(AT_ROWS, AT_BN, 1); // N = 64: a last S block of one key block
            constexpr uint32_t idesc_o = idesc_f16(AT_ROWS, AT_D, 1);  // A from TMEM (K-major), B MN-major, M = N = 128
            bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, args.err);
            bool issued = false;
            // descriptors of the operands' first steps; the MMA blocks add constant offsets
            // K^T: MN-major, a stage's two key blocks (64-key atoms of the N dimension) 16 KB apart
            const uint64_t q_desc = smem_desc(sQ, 16, 1024), k_desc = smem_desc(sK, K_BYTES, 1024);
            const uint64_t v_desc = smem_desc(sVsp, BOX, 1024);  // MN-major: 64-dim chunks 8 KB apart
            auto sblock = [&](int jp) -> bool {  // S block J = Q . K^T of key blocks 2J, 2J+1 into buffer J % 3
                const int kst = jp % KST;
                if (!mbar_wait(smem_u32(&k_full[kst]), (jp / KST) & 1, abort_flag, args.err)) return false;
                tc_fence_after();
                mma_s_block(tmem_base + static_cast<uint32_t>((jp % SPB) * TMEM_SP), q_desc,
                            k_desc + static_cast<uint64_t>(kst * (KS_BYTES >> 4)), 2 * jp + 1 < nb ? idesc_s : idesc_s1,
                            0u);
                issued = true;
                mma_commit(smem_u32(&k_empty[kst]));
                mma_commit(smem_u32(&s_full[jp % SPB]));
                return true;
            };
            // PV_i's inputs: P_i written over S_i, V_i split
            auto pv_ready = [&](int i) -> bool {
                return mbar_wait(smem_u32(&p_full[i % (2 * SPB)]), (i / (2 * SPB)) & 1, abort_flag, args.err) &&
                       mbar_wait(smem_u32(&vsp_full[i % NVB]), (i / NVB) & 1, abort_flag, args.err);
            };
            auto pv = [&](int i) {  // O += P_i . V_i as P_lo.V_hi + P_hi.V_lo + P_hi.V_hi
                const int b = i % NVB;
                tc_fence_after();
                const uint64_t vh = v_desc + static_cast<uint64_t>(b * (VSP_BYTES >> 4));
                mma_pv_block(tmem_base + TMEM_O, tmem_base + static_cast<uint32_t>(((i >> 1) % SPB) * TMEM_SP + (i & 1) * AT_BN),
                             vh, vh + (V_BYTES >> 4), idesc_o, i > 0 ? 1u : 0u);
                mma_commit(smem_u32(&vsp_empty[b]));
                mma_commit(smem_u32(&pv_done[i & 1]));
            };
            // issue order (S blocks by S block, P.V by key block) S_0 S_1 S_2 | PV_0 PV_1 S_3 | PV_2 PV_3 S_4 | ...
            for (int jp = 0; ok && jp < ns && jp < SPB; ++jp) ok = sblock(jp);
            for (int j = 0; ok && j < nb; ++j) {
                ok = pv_ready(j);
                if (ok) pv(j);
                if (ok && (j & 1) && (j >> 1) + SPB < ns) ok = sblock((j >> 1) + SPB);
            }
            if (ok && !*abort_flag) mma_commit(smem_u32(o_full));
            if (issued) {  // drain: every MMA issued has completed before TMEM is freed
                mma_commit(smem_u32(drain));
                const uint64_t start = globaltimer();
                while (!mbar_try_wait(smem_u32(drain), 0))
                    if (globaltimer() - start > kTimeoutNs) {
                        atomicOr(args.err, kErrTimeout);
                        break;
                    }
            }
        }
    } else if (warp >= 6) {
        // ---------------- V splitters (warps 6..9) ----------------
        // Each V block [64 keys][128 dims] f32 is read straight from global memory, scaled by 2^k (k from the
        // largest |V| of the task so far) and split into f16 V_hi / V_lo, each written in the layout the MMA reads
        // as an MN-major B: two 64-dim chunks of 8 KB, key k's 128-byte row at k * 128, 16-byte unit u (dims
        // 8u..8u+7 of the chunk) at u ^ (k % 8).  Thread t owns the dims 8(t % 16) .. 8(t % 16)+7 of keys
        // t / 16 + 8i, i = 0..7: sixteen lanes read one key's 512-byte row, and the eight lanes of a 128-byte
        // store phase fill one swizzled row.  The next block's loads are in flight while this block is written.
        // The block maximum: once block j+1's loads have landed (after block j is handed over), every warp posts
        // its part of that block's largest |V| and arrives on vmax_ready[(j+1) % 2]; before block j+1 is split,
        // every warp reads the four parts after that barrier's phase completes.
        const int t = threadIdx.x - 6 * 32;  // 0..127
        const int sw = warp - 6;             // 0..3
        const int u = t & 15;                // dims 8u..8u+7
        const int kb = t >> 4;               // keys kb + 8i
        const int st_off = (u >> 3) * BOX + kb * 128 + (((u & 7) ^ kb) << 4);  // (kb + 8i) % 8 == kb
        const float* vbase = args.v + rec[args.v_p] + 8 * u;
        auto load = [&](int j, float4 (&x)[16]) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4* src =
                    reinterpret_cast<const float4*>(vbase + static_cast<int64_t>(j * AT_BN + kb + 8 * i) * args.v_pitch);
                x[2 * i] = __ldg(src);
                x[2 * i + 1] = __ldg(src + 1);
            }
        };
        auto post_max = [&](int j, const float4 (&x)[16]) {  // this warp's part of block j's largest |V|
            uint32_t m = 0u;  // bits of a non-negative float; NaN orders above inf
#pragma unroll
            for (int i = 0; i < 16; ++i)
                m = max(m, max(max(__float_as_uint(x[i].x) & 0x7fffffffu, __float_as_uint(x[i].y) & 0x7fffffffu),
                               max(__float_as_uint(x[i].z) & 0x7fffffffu, __float_as_uint(x[i].w) & 0x7fffffffu)));
            m = __reduce_max_sync(0xffffffffu, m);
            if (lane == 0) {
                v_part[(j & 1) * 4 + sw] = m;
                mbar_arrive(smem_u32(&vmax_ready[j & 1]));
            }
        };
        float4 cur[16], nxt[16];
        uint32_t vmax_bits = 0u;  // largest |V| of the task so far
        if (nb > 0) {
            load(0, cur);
            post_max(0, cur);
        }
        for (int j = 0; j < nb; ++j) {
            const int b = j % NVB, pb = j & 1;  // V buffer; partial-maximum slot
            if (j + 1 < nb) load(j + 1, nxt);
            // block j's four parts; the slot was last read in block j-2, which every warp finished before it
            // posted block j-1's part (the phase this warp waited for in block j-1)
            if (!mbar_wait(smem_u32(&vmax_ready[pb]), (j >> 1) & 1, abort_flag, args.err)) break;
            vmax_bits =
                max(vmax_bits, max(max(v_part[pb * 4], v_part[pb * 4 + 1]), max(v_part[pb * 4 + 2], v_part[pb * 4 + 3])));
            const int k2 = v_scale_log2(vmax_bits);
            const float vs = pow2f(k2);
            if (j >= NVB && !mbar_wait(smem_u32(&vsp_empty[b]), ((j / NVB) & 1) ^ 1u, abort_flag, args.err)) break;
            uint8_t* hi = smem + OFF_VSP + b * VSP_BYTES + st_off;
            uint8_t* lo = hi + V_BYTES;
            // one pair of dims: scaled, split, packed into `h` / `l`
            auto split2 = [vs](float a, float c, uint32_t& h, uint32_t& l) {
                const float x0 = a * vs, x1 = c * vs;
                const float h0 = f16_hi_part(x0), h1 = f16_hi_part(x1);
                h = pack_f16(h0, h1);
                l = pack_f16(x0 - h0, x1 - h1);
            };
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint4 h, l;
                split2(cur[2 * i].x, cur[2 * i].y, h.x, l.x);
                split2(cur[2 * i].z, cur[2 * i].w, h.y, l.y);
                split2(cur[2 * i + 1].x, cur[2 * i + 1].y, h.z, l.z);
                split2(cur[2 * i + 1].z, cur[2 * i + 1].w, h.w, l.w);
                *reinterpret_cast<uint4*>(hi + i * 8 * 128) = h;
                *reinterpret_cast<uint4*>(lo + i * 8 * 128) = l;
            }
            if (t == 0) v_log2[b] = k2;  // read by the softmax warps after they wait for this block
            fence_proxy_async_smem();    // V_hi / V_lo become visible to the tensor core's reads
            mbar_arrive(smem_u32(&vsp_full[b]));
            if (j + 1 < nb) post_max(j + 1, nxt);
#pragma unroll
            for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
        }
    } else {
        // ---------------- softmax + epilogue (warps 2..5, one row per thread) ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        float scale = 1.f;
        if (args.scale_mode == 1) scale = args.scale_const;
        else if (args.scale_mode == 2) scale = __uint_as_float(static_cast<uint32_t>(rec[args.scale_pos]));
        const float c2 = scale * 1.4426950408889634f;  // into the base-2 domain
        float m_ref = -INFINITY, l = 0.f;
        int k_v = 0;  // V's scale exponent in O so far
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            const int sb = (j >> 1) % SPB;  // S block j / 2's buffer (its phase is still the current one for j odd)
            if (!mbar_wait(smem_u32(&s_full[sb]), ((j >> 1) / SPB) & 1, abort_flag, args.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // the S row into registers (both 32-column loads in flight, one wait); P_j then goes over it
            const uint32_t sp_addr = tmem_base + lane_addr + static_cast<uint32_t>(sb * TMEM_SP + (j & 1) * AT_BN);
            uint32_t r[2][32];
            tmem_ld32_async(sp_addr, r[0]);
            tmem_ld32_async(sp_addr + 32, r[1]);
            tmem_wait_ld();
            reg_fence(r[0]);
            reg_fence(r[1]);
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four chains: latency, not one long one
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int i = 0; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(r[c][i]) * c2);
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            float corr = 1.f;
            const bool grow = j == 0 || mx > m_ref + kRescaleLog2;
            if (grow) {
                const float m_new = j == 0 ? mx : fmaxf(m_ref, mx);
                corr = j == 0 ? 1.f : exp2f(m_ref - m_new);
                m_ref = m_new;
            }
            l *= corr;
            // p = 2^(x - max) in f32 for the sum; p * 2^7 as f16 P_hi + P_lo (key pairs packed) into this row's TMEM
            // lane
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 2; ++c) {  // keys 32c .. 32c+31: P_hi columns 16c.., P_lo columns 32 + 16c..
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = ex2_approx(__uint_as_float(r[c][2 * i]) * c2 - m_ref);
                    const float p1 = ex2_approx(__uint_as_float(r[c][2 * i + 1]) * c2 - m_ref);
                    sum4[(2 * i) & 3] += p0;
                    sum4[(2 * i + 1) & 3] += p1;
                    const float q0 = p0 * static_cast<float>(1 << kPScaleLog2), q1 = p1 * static_cast<float>(1 << kPScaleLog2);
                    const float h0 = f16_hi_part(q0), h1 = f16_hi_part(q1);
                    ph[i] = pack_f16(h0, h1);
                    pl[i] = pack_f16(q0 - h0, q1 - h1);
                }
                tmem_st16(sp_addr + 16 * c, ph);
                tmem_st16(sp_addr + 32 + 16 * c, pl);
            }
            tmem_wait_st();
            const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
            l += sum;
            // V's scale for this block (set by the splitters before they released its buffer), read after P_j is
            // out; when it drops, O moves to the new scale together with the row-max correction, before PV_j
            // (which waits for p_full) accumulates
            if (!mbar_wait(smem_u32(&vsp_full[j % NVB]), (j / NVB) & 1, abort_flag, args.err)) {
                ok = false;
                break;
            }
            const int k_j = v_log2[j % NVB];
            const bool v_moved = j > 0 && k_j != k_v;  // the same in every thread
            const float ofac = v_moved ? corr * (k_j - k_v >= -126 ? pow2f(k_j - k_v) : 0.f) : corr;  // k only falls
            k_v = k_j;
            if (j > 0 && (v_moved || __any_sync(0xffffffffu, grow))) {
                // O holds block j-1's contribution (its MMAs are done) before it is rescaled
                if (!mbar_wait(smem_u32(&pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, abort_flag, args.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < AT_D / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32_async(tmem_base + lane_addr + TMEM_O + c * 32, r);
                    tmem_wait_ld();
                    reg_fence(r);
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * ofac);
                    tmem_st32(tmem_base + lane_addr + TMEM_O + c * 32, r);
                }
                tmem_wait_st();
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&p_full[j % (2 * SPB)]));
        }
        if (ok && mbar_wait(smem_u32(o_full), 0, abort_flag, args.err)) {
            tc_fence_after();
            const float inv = pow2f(-(kPScaleLog2 + k_v)) / l;  // the two scales and the sum
            float* orow = args.out + rec[args.o_p] + static_cast<int64_t>(row) * args.o_pitch;
#pragma unroll 1
            for (int c = 0; c < AT_D / 32; ++c) {
                float v[32];
                tmem_ld32(tmem_base + lane_addr + TMEM_O + c * 32, v);
                float4* dst = reinterpret_cast<float4*>(orow + c * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    dst[i] = make_float4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace

bool attention_tiles_supported(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L) {
    const ParamDesc &Q = b.p[q_p], &KT = b.p[kt_p], &V = b.p[v_p], &O = b.p[o_p];
    auto rows16 = [](const ParamDesc& p, int type, int eb) {
        return p.type == type && p.s4 == 1 && p.s3 > 0 && (p.s3 * eb) % 16 == 0 &&
               (reinterpret_cast<uintptr_t>(p.base) & 15) == 0;
    };
    return rows16(Q, PT_F16, 2) && rows16(KT, PT_F16, 2) && rows16(V, PT_F32, 4) && rows16(O, PT_F32, 4) &&
           Q.rows == AT_ROWS && Q.cols == AT_D && KT.rows == AT_D && KT.cols == L && V.rows == L && V.cols == AT_D &&
           O.rows == AT_ROWS && O.cols == AT_D && L >= AT_BN && L % AT_BN == 0;
}

bool attention_task_ok(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L, const int64_t* r) {
    const ParamDesc &Q = b.p[q_p], &KT = b.p[kt_p], &V = b.p[v_p], &O = b.p[o_p];
    const int64_t oq = r[q_p], ok = r[kt_p], ov = r[v_p], oo = r[o_p];
    const int64_t q_rows = (Q.numel_span + Q.s3 - 1) / Q.s3, k_rows = (KT.numel_span + KT.s3 - 1) / KT.s3;
    const int64_t v_rows = (V.numel_span + V.s3 - 1) / V.s3;
    // TMA x coordinates on 16-byte boundaries (8 f16 / 4 f32), every tile inside its tensor
    return oq >= 0 && ok >= 0 && ov >= 0 && oo >= 0 && oo % 4 == 0 && (oq % Q.s3) % 8 == 0 &&
           (ok % KT.s3) % 8 == 0 && (ov % V.s3) % 4 == 0 && (oq % Q.s3) + AT_D <= Q.s3 &&
           (oq / Q.s3) + AT_ROWS <= q_rows && (ok % KT.s3) + L <= KT.s3 && (ok / KT.s3) + AT_D <= k_rows &&
           (ov % V.s3) + AT_D <= V.s3 && (ov / V.s3) + L <= v_rows && oo + (AT_ROWS - 1) * O.s3 + AT_D <= O.numel_span;
}

cudaError_t launch_attention(const TaskBatch& b, int q_p, int kt_p, int v_p, int o_p, int L, int scale_mode,
                             int scale_pos, float scale_const, cudaStream_t s) {
    if (b.ntasks <= 0) return cudaSuccess;
    if (b.ntasks > 0x7fffffff) return cudaErrorInvalidValue;
    const ParamDesc &Q = b.p[q_p], &KT = b.p[kt_p], &V = b.p[v_p], &O = b.p[o_p];
    CUtensorMap mq, mkt;
    if (!make_map_f16(&mq, Q.base, Q.s3, (Q.numel_span + Q.s3 - 1) / Q.s3, 64, AT_ROWS)) return cudaErrorInvalidValue;
    if (!make_map_f16(&mkt, KT.base, KT.s3, (KT.numel_span + KT.s3 - 1) / KT.s3, 64, 64)) return cudaErrorInvalidValue;
    AttnArgs a;
    a.rec = b.rec;
    a.ntasks = b.ntasks;
    a.stride = b.stride;
    a.q_p = q_p;
    a.kt_p = kt_p;
    a.v_p = v_p;
    a.o_p = o_p;
    a.q_pitch = Q.s3;
    a.kt_pitch = KT.s3;
    a.v_pitch = V.s3;
    a.v = reinterpret_cast<const float*>(V.base);
    a.out = reinterpret_cast<float*>(O.base);
    a.o_pitch = O.s3;
    a.nblocks = L / AT_BN;
    a.scale_mode = scale_mode;
    a.scale_pos = scale_pos;
    a.scale_const = scale_const;
    a.err = b.err;
    cudaError_t e = cudaFuncSetAttribute(attention_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attention_tcgen05_kernel<<<static_cast<unsigned>(b.ntasks), AT_THREADS, SMEM_BYTES, s>>>(mq, mkt, a);
    return cudaGetLastError();
}

}  // namespace ptowsp::dev
