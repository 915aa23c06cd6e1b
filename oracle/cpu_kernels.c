/*
 * cpu_kernels.c -- C port of the reference CPU-sim hot loops (TEST / BASELINE
 * INFRASTRUCTURE ONLY: used by the tests and by bench.py's CPU-baseline and
 * `--impl reference` legs, never by the product path).
 *
 * Each function executes the same per-task tile-op sequence the reference
 * emitter generates for the config kernels (src/python/pto_codegen.cpp:
 * 470-1241): TLOAD the tile into a local buffer, run the tile ops one by one
 * over the whole tile (TMUL, TROWSUM, TDIVS, TRSQRT, TROWEXPAND*, TEXP,
 * TROWMAX, TMATMUL with f32 accumulation), TSTORE.  The task loop is the
 * generated P(batch) x P(tiles) nest (:2305-2360).  The CPU-sim runs tasks on
 * one thread; here tasks are split over `nthreads` pthreads so the baseline
 * can use every host core.
 *
 * The two built-in task bodies of configs 4 and 5 (paged GQA decode; indexer
 * scoring + stable top-k) follow the plain-C++ CPU bodies this target's
 * workload forms attach to those kernels (pto_wsp_b200/workloads.py) and the
 * reference top-k rule, score descending with ties to the lower index
 * (examples/deepseek_lightning_indexer/golden.py:6-25).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int kind;
    const void* a;
    const void* b;
    void* c;
    int64_t t0, t1;
    int rows, cols, k;
    int64_t lda, ldb, ldc;  /* row pitch (elements) of each operand's tile rows */
    int64_t sa, sb, sc;     /* element stride between consecutive tiles */
} job_t;

static float half_to_float(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (m == 0) f = s;
        else {
            e = 127 - 15 + 1;
            while (!(m & 0x400)) { m <<= 1; e--; }
            m &= 0x3ff;
            f = s | (e << 23) | (m << 13);
        }
    } else if (e == 31) f = s | 0x7f800000u | (m << 13);
    else f = s | ((e + 127 - 15) << 23) | (m << 13);
    float out;
    memcpy(&out, &f, 4);
    return out;
}

/* RMSNorm task: TLOAD, TMUL, TROWSUM, TDIVS(cols), TRSQRT, TROWEXPANDMUL, TSTORE. */
static void rmsnorm_task(const float* x, float* y, int R, int C, int64_t ld, float* t0, float* t1) {
    for (int r = 0; r < R; ++r) memcpy(t0 + (int64_t)r * C, x + r * ld, sizeof(float) * C);   /* TLOAD */
    for (int i = 0; i < R * C; ++i) t1[i] = t0[i] * t0[i];                                      /* TMUL */
    float red[1024];
    for (int r = 0; r < R; ++r) {                                                                /* TROWSUM */
        float s = 0.f;
        for (int c = 0; c < C; ++c) s += t1[(int64_t)r * C + c];
        red[r] = s;
    }
    for (int r = 0; r < R; ++r) red[r] = red[r] / (float)C;                                      /* TDIVS */
    for (int r = 0; r < R; ++r) red[r] = 1.0f / sqrtf(red[r]);                                   /* TRSQRT */
    for (int r = 0; r < R; ++r)                                                                  /* TROWEXPANDMUL */
        for (int c = 0; c < C; ++c) t1[(int64_t)r * C + c] = t0[(int64_t)r * C + c] * red[r];
    for (int r = 0; r < R; ++r) memcpy(y + r * ld, t1 + (int64_t)r * C, sizeof(float) * C);    /* TSTORE */
}

/* Softmax task: TLOAD, TROWMAX, TROWEXPANDSUB, TEXP, TROWSUM, TROWEXPANDDIV, TSTORE. */
static void softmax_task(const float* x, float* y, int R, int C, int64_t ld, float* t0, float* t1) {
    for (int r = 0; r < R; ++r) memcpy(t0 + (int64_t)r * C, x + r * ld, sizeof(float) * C);
    float mx[1024], sm[1024];
    for (int r = 0; r < R; ++r) {
        float m = -INFINITY;
        for (int c = 0; c < C; ++c) m = fmaxf(m, t0[(int64_t)r * C + c]);
        mx[r] = m;
    }
    for (int r = 0; r < R; ++r)
        for (int c = 0; c < C; ++c) t1[(int64_t)r * C + c] = t0[(int64_t)r * C + c] - mx[r];
    for (int i = 0; i < R * C; ++i) t0[i] = expf(t1[i]);
    for (int r = 0; r < R; ++r) {
        float s = 0.f;
        for (int c = 0; c < C; ++c) s += t0[(int64_t)r * C + c];
        sm[r] = s;
    }
    for (int r = 0; r < R; ++r)
        for (int c = 0; c < C; ++c) t1[(int64_t)r * C + c] = t0[(int64_t)r * C + c] / sm[r];
    for (int r = 0; r < R; ++r) memcpy(y + r * ld, t1 + (int64_t)r * C, sizeof(float) * C);
}

/* bgemm task: TLOAD A[M,K] (f16), TLOAD B[K,N] (f16), TMATMUL (f32 acc), TSTORE C[M,N] f32. */
static void gemm_task(const uint16_t* a, const uint16_t* b, float* c, int M, int N, int K, int64_t lda,
                      int64_t ldb, int64_t ldc, float* ta, float* tb, float* tc) {
    for (int i = 0; i < M; ++i)
        for (int kk = 0; kk < K; ++kk) ta[(int64_t)i * K + kk] = half_to_float(a[i * lda + kk]);
    for (int kk = 0; kk < K; ++kk)
        for (int j = 0; j < N; ++j) tb[(int64_t)kk * N + j] = half_to_float(b[kk * ldb + j]);
    for (int i = 0; i < M * N; ++i) tc[i] = 0.f;
    for (int i = 0; i < M; ++i)
        for (int kk = 0; kk < K; ++kk) {
            const float av = ta[(int64_t)i * K + kk];
            for (int j = 0; j < N; ++j) tc[(int64_t)i * N + j] += av * tb[(int64_t)kk * N + j];
        }
    for (int i = 0; i < M; ++i) memcpy(c + i * ldc, tc + (int64_t)i * N, sizeof(float) * N);
}

static void* worker(void* arg) {
    job_t* j = (job_t*)arg;
    if (j->kind == 0 || j->kind == 1) {
        size_t n = (size_t)j->rows * j->cols;
        float* t0 = (float*)malloc(sizeof(float) * n);
        float* t1 = (float*)malloc(sizeof(float) * n);
        for (int64_t t = j->t0; t < j->t1; ++t) {
            const float* x = (const float*)j->a + t * j->sa;
            float* y = (float*)j->c + t * j->sc;
            if (j->kind == 0) rmsnorm_task(x, y, j->rows, j->cols, j->lda, t0, t1);
            else softmax_task(x, y, j->rows, j->cols, j->lda, t0, t1);
        }
        free(t0);
        free(t1);
    } else {
        float* ta = (float*)malloc(sizeof(float) * (size_t)j->rows * j->k);
        float* tb = (float*)malloc(sizeof(float) * (size_t)j->k * j->cols);
        float* tc = (float*)malloc(sizeof(float) * (size_t)j->rows * j->cols);
        for (int64_t t = j->t0; t < j->t1; ++t) {
            /* a/b/c offsets are precomputed per task by the caller in sa/sb/sc tables */
            const int64_t* offs = (const int64_t*)j->b;
            gemm_task((const uint16_t*)j->a + offs[3 * t], (const uint16_t*)j->a + offs[3 * t + 1],
                      (float*)j->c + offs[3 * t + 2], j->rows, j->cols, j->k, j->lda, j->ldb, j->ldc, ta, tb, tc);
        }
        free(ta);
        free(tb);
        free(tc);
    }
    return NULL;
}

static void run_jobs(job_t proto, int64_t ntasks, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    job_t jobs[256];
    int64_t per = (ntasks + nthreads - 1) / nthreads;
    int used = 0;
    for (int i = 0; i < nthreads; ++i) {
        jobs[i] = proto;
        jobs[i].t0 = i * per;
        jobs[i].t1 = (i + 1) * per < ntasks ? (i + 1) * per : ntasks;
        if (jobs[i].t0 >= jobs[i].t1) break;
        pthread_create(&th[i], NULL, worker, &jobs[i]);
        used++;
    }
    for (int i = 0; i < used; ++i) pthread_join(th[i], NULL);
}

/* Row tiles of a contiguous [ntiles, rows, cols] f32 tensor: kind 0 = RMSNorm, 1 = softmax. */
void oracle_row_tiles(int kind, const float* x, float* y, int64_t ntiles, int rows, int cols, int nthreads) {
    job_t j;
    memset(&j, 0, sizeof j);
    j.kind = kind;
    j.a = x;
    j.c = y;
    j.rows = rows;
    j.cols = cols;
    j.lda = cols;
    j.sa = j.sc = (int64_t)rows * cols;
    run_jobs(j, ntiles, nthreads);
}

/* bgemm tiles: base = f16 element pointer covering A and B (offsets in f16 elements from base),
 * c = f32 base; offs[3*t + {0,1,2}] = A tile, B tile (from base) and C tile (from c) offsets. */
void oracle_gemm_tiles(const uint16_t* base, const int64_t* offs, float* c, int64_t ntasks, int M, int N, int K,
                       int64_t lda, int64_t ldb, int64_t ldc, int nthreads) {
    job_t j;
    memset(&j, 0, sizeof j);
    j.kind = 2;
    j.a = base;
    j.b = offs;
    j.c = c;
    j.rows = M;
    j.cols = N;
    j.k = K;
    j.lda = lda;
    j.ldb = ldb;
    j.ldc = ldc;
    run_jobs(j, ntasks, nthreads);
}

/* ---------------------------------------------------------------------------------------------------------- */
/* Config 4: paged GQA decode, one (request, kv head) task = online softmax over the request's tokens per query  */
/* head, f32 arithmetic, f16 out.  q [R][KVH][G][D], caches [pages][PS][KVH][D], page table [R][maxp].          */
/* ---------------------------------------------------------------------------------------------------------- */

static uint16_t float_to_half_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (ax < 0x38800000u) {                                   /* subnormal half */
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e; /* 14 + (113 - e) */
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((ax - 0x38000000u) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

typedef struct {
    const uint16_t *q, *kc, *vc;
    const int32_t *pt, *len;
    uint16_t* out;
    int R, KVH, G, D, PS, maxp;
    int64_t t0, t1;
} decode_job_t;

static void* decode_worker(void* arg) {
    decode_job_t* j = (decode_job_t*)arg;
    const int G = j->G, D = j->D, KVH = j->KVH, PS = j->PS;
    float acc[8][256], qf[8][256], m[8], l[8];
    const float scale = 1.0f / sqrtf((float)D);
    for (int64_t t = j->t0; t < j->t1; ++t) {
        const int r = (int)(t / KVH), h = (int)(t % KVH);
        const int L = j->len[r];
        for (int g = 0; g < G; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
            for (int d = 0; d < D; ++d) {
                acc[g][d] = 0.f;
                qf[g][d] = half_to_float(j->q[(((int64_t)r * KVH + h) * G + g) * D + d]);
            }
        }
        for (int tok = 0; tok < L; ++tok) {
            const int64_t page = j->pt[(int64_t)r * j->maxp + tok / PS];
            const uint16_t* kr = j->kc + ((page * PS + tok % PS) * KVH + h) * D;
            const uint16_t* vr = j->vc + ((page * PS + tok % PS) * KVH + h) * D;
            float kf[256], vf[256];
            for (int d = 0; d < D; ++d) {
                kf[d] = half_to_float(kr[d]);
                vf[d] = half_to_float(vr[d]);
            }
            for (int g = 0; g < G; ++g) {
                float s = 0.f;
                for (int d = 0; d < D; ++d) s += qf[g][d] * kf[d];
                s *= scale;
                const float mn = s > m[g] ? s : m[g], c = expf(m[g] - mn), p = expf(s - mn);
                l[g] = l[g] * c + p;
                for (int d = 0; d < D; ++d) acc[g][d] = acc[g][d] * c + p * vf[d];
                m[g] = mn;
            }
        }
        for (int g = 0; g < G; ++g)
            for (int d = 0; d < D; ++d)
                j->out[(((int64_t)r * KVH + h) * G + g) * D + d] = float_to_half_rne(L > 0 ? acc[g][d] / l[g] : 0.f);
    }
    return NULL;
}

void oracle_paged_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pt,
                         const int32_t* len, uint16_t* out, int R, int KVH, int G, int D, int PS, int maxp,
                         int nthreads) {
    if (G > 8 || D > 256) return;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    const int64_t ntasks = (int64_t)R * KVH;
    pthread_t th[256];
    decode_job_t jobs[256];
    int used = 0;
    for (int i = 0; i < nthreads; ++i) {
        decode_job_t j = {q, kc, vc, pt, len, out, R, KVH, G, D, PS, maxp, 0, 0};
        /* interleaved slices keep long and short requests spread over the threads */
        j.t0 = ntasks * i / nthreads;
        j.t1 = ntasks * (i + 1) / nthreads;
        if (j.t0 >= j.t1) continue;
        jobs[used] = j;
        pthread_create(&th[used], NULL, decode_worker, &jobs[used]);
        used++;
    }
    for (int i = 0; i < used; ++i) pthread_join(th[i], NULL);
}

/* ---------------------------------------------------------------------------------------------------------- */
/* Config 5: lightning indexer.  score[b][q][t] = sum_h w[b][q][h] * relu(q[b][q*H+h] . k[b][t]) (f32, heads in  */
/* order), then per (b, q) row the indices of the top K scores, score descending, ties -> lower index.          */
/* ---------------------------------------------------------------------------------------------------------- */

typedef struct {
    const uint16_t *q, *k;
    const float* w;
    float* s;
    int32_t* idx;
    int B, Q, H, D, T, K;
    int64_t t0, t1;  /* rows (b, q) */
} indexer_job_t;

static int cmp_desc_u64(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

static void* indexer_worker(void* arg) {
    indexer_job_t* j = (indexer_job_t*)arg;
    const int H = j->H, D = j->D, T = j->T;
    float* qf = (float*)malloc(sizeof(float) * (size_t)H * D);
    float* kf = (float*)malloc(sizeof(float) * (size_t)D * 64);
    uint64_t* comp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)T);
    for (int64_t row = j->t0; row < j->t1; ++row) {
        const int b = (int)(row / j->Q), qi = (int)(row % j->Q);
        for (int h = 0; h < H; ++h)
            for (int d = 0; d < D; ++d)
                qf[h * D + d] = half_to_float(j->q[(((int64_t)b * j->Q + qi) * H + h) * D + d]);
        const float* w = j->w + ((int64_t)b * j->Q + qi) * H;
        float* srow = j->s + ((int64_t)b * j->Q + qi) * T;
        for (int t0 = 0; t0 < T; t0 += 64) {
            const int nt = T - t0 < 64 ? T - t0 : 64;
            for (int t = 0; t < nt; ++t)
                for (int d = 0; d < D; ++d) kf[t * D + d] = half_to_float(j->k[((int64_t)b * T + t0 + t) * D + d]);
            for (int t = 0; t < nt; ++t) {
                float acc = 0.f;
                for (int h = 0; h < H; ++h) {
                    float dot = 0.f;
                    for (int d = 0; d < D; ++d) dot += qf[h * D + d] * kf[t * D + d];
                    acc += w[h] * (dot > 0.f ? dot : 0.f);
                }
                srow[t0 + t] = acc;
            }
        }
        for (int t = 0; t < T; ++t) {
            uint32_t bits;
            memcpy(&bits, &srow[t], 4);
            uint32_t key = (bits >> 31) ? ~bits : (bits | 0x80000000u);
            if (srow[t] == 0.f) key = 0x80000000u;
            comp[t] = ((uint64_t)key << 32) | (uint64_t)(0xffffffffu - (uint32_t)t);
        }
        qsort(comp, (size_t)T, sizeof(uint64_t), cmp_desc_u64);
        int32_t* out = j->idx + ((int64_t)b * j->Q + qi) * j->K;
        for (int i = 0; i < j->K && i < T; ++i) out[i] = (int32_t)(0xffffffffu - (uint32_t)(comp[i] & 0xffffffffu));
    }
    free(qf);
    free(kf);
    free(comp);
    return NULL;
}

void oracle_indexer(const uint16_t* q, const uint16_t* k, const float* w, float* s, int32_t* idx, int B, int Q, int H,
                    int D, int T, int K, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    const int64_t rows = (int64_t)B * Q;
    pthread_t th[256];
    indexer_job_t jobs[256];
    int used = 0;
    for (int i = 0; i < nthreads; ++i) {
        indexer_job_t j = {q, k, w, s, idx, B, Q, H, D, T, K, rows * i / nthreads, rows * (i + 1) / nthreads};
        if (j.t0 >= j.t1) continue;
        jobs[used] = j;
        pthread_create(&th[used], NULL, indexer_worker, &jobs[used]);
        used++;
    }
    for (int i = 0; i < used; ++i) pthread_join(th[i], NULL);
}
