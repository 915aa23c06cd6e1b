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
