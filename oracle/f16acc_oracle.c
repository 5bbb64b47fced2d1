/*
 * f16acc_oracle.c -- CPU restatement of f16acc's chunked FP16-accumulate GEMM.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the parity tests,
 * the smoke check and bench.py's CPU-baseline leg compare the CUDA kernels
 * against.  It is never linked into the product library and no product code
 * path calls it.
 *
 * What it restates (reference = steppergg/f16acc, file:line within that project):
 *   - f16acc/kernel.py:37-54  `_loop`: C = sum over 32-long K chunks, each chunk
 *     a dot product accumulated in FP16 (`tl.dot(..., out_dtype=fp16)`) and
 *     then converted to FP32 and added into an FP32 accumulator; chunks start
 *     at absolute K offsets 0, 32, 64, ...; the K tail is zero padded.
 *   - f16acc/kernel.py:50-51  the `CHUNKED=False` mode: plain FP32 accumulation.
 *   - f16acc/kernel.py:70-71  the per-tile flag: set when any accumulator in
 *     the tile is not finite (|acc| < inf is false for inf and NaN).
 *   - f16acc/kernel.py:75-81  `_redo`: flagged tiles are recomputed with FP32
 *     accumulation and overwrite the tile.
 *   - f16acc/kernel.py:57-60  `_store`: the FP32 accumulator cast to C's dtype.
 *   - tests/test_f16acc.py:11-12  `rel()`: max|x - ref| / max|ref|.
 *
 * How a chunk is rounded.  Where the FP16 rounding happens inside one
 * tensor-core dot is hardware defined; the reference leaves it to Triton.
 * `round_every` selects the emulation:
 *   32 -> the exact chunk sum is rounded to FP16 once (what Triton's CPU
 *         interpreter does for the reference kernel: FP32 dot, then a cast);
 *   16 -> the two 16-long halves are rounded separately: the second half is
 *         added to the rounded first half and rounded again (the shape of two
 *         K=16 MMA instructions sharing an FP16 accumulator).
 * Products of two FP16 values are exact in FP32.  Partial sums are formed in
 * double and rounded to FP16 by one correctly rounded conversion (_Float16).
 *
 * Matrices are FP16 bit patterns (uint16_t) with arbitrary element strides,
 * exactly like the operands `mm()` accepts.  Operands are widened once per
 * call into contiguous float copies (A as [M][K], B as [K][N]) through a
 * 65536-entry table, so the inner loops are plain float/double arithmetic.
 */
#include <math.h>
#include <omp.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float g_h2f[65536];
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void build_table(void) {
    for (uint32_t h = 0; h < 65536u; ++h) {
        _Float16 v;
        uint16_t b = (uint16_t)h;
        memcpy(&v, &b, 2);
        g_h2f[h] = (float)v;
    }
}

static inline uint16_t f2h(double x) {
    _Float16 v = (_Float16)x;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static float *widen_a(const uint16_t *A, int64_t sAm, int64_t sAk, int64_t M, int64_t K) {
    float *a = (float *)malloc(sizeof(float) * (size_t)(M * K > 0 ? M * K : 1));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i)
        for (int64_t k = 0; k < K; ++k) a[i * K + k] = g_h2f[A[i * sAm + k * sAk]];
    return a;
}

static float *widen_b(const uint16_t *B, int64_t sBk, int64_t sBn, int64_t K, int64_t N) {
    float *b = (float *)malloc(sizeof(float) * (size_t)(K * N > 0 ? K * N : 1));
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < K; ++k)
        for (int64_t j = 0; j < N; ++j) b[k * N + j] = g_h2f[B[k * sBk + j * sBn]];
    return b;
}

/* FP64 product: the accuracy reference (tests/test_f16acc.py:22-24, :29). */
void oracle_gemm_f64(const uint16_t *A, int64_t sAm, int64_t sAk,
                     const uint16_t *B, int64_t sBk, int64_t sBn,
                     double *C, int64_t M, int64_t N, int64_t K) {
    pthread_once(&g_once, build_table);
    float *a = widen_a(A, sAm, sAk, M, K);
    float *b = widen_b(B, sBk, sBn, K, N);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        double *row = C + i * N;
        for (int64_t j = 0; j < N; ++j) row[j] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            double av = a[i * K + k];
            if (av == 0.0) continue;
            const float *bk = b + k * N;
            for (int64_t j = 0; j < N; ++j) row[j] += av * (double)bk[j];
        }
    }
    free(a);
    free(b);
}

/* Plain FP32 accumulation over the whole K range (kernel.py:50-51).  The sum
 * is formed in double and rounded to FP32 once, which is within FP32 rounding
 * of any tensor-core accumulation order. */
void oracle_gemm_f32acc(const uint16_t *A, int64_t sAm, int64_t sAk,
                        const uint16_t *B, int64_t sBk, int64_t sBn,
                        float *C, int64_t M, int64_t N, int64_t K) {
    pthread_once(&g_once, build_table);
    float *a = widen_a(A, sAm, sAk, M, K);
    float *b = widen_b(B, sBk, sBn, K, N);
#pragma omp parallel
    {
        double *acc = (double *)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
        for (int64_t i = 0; i < M; ++i) {
            for (int64_t j = 0; j < N; ++j) acc[j] = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                double av = a[i * K + k];
                const float *bk = b + k * N;
                for (int64_t j = 0; j < N; ++j) acc[j] += av * (double)bk[j];
            }
            for (int64_t j = 0; j < N; ++j) C[i * N + j] = (float)acc[j];
        }
        free(acc);
    }
    free(a);
    free(b);
}

/* Chunked FP16-accumulate GEMM (kernel.py:44-49): FP32 result before the
 * final cast.  chunk = 32 in the reference (kernel.py:17).  Optional tile
 * flags (kernel.py:70-71) and redo (kernel.py:75-81) for bm x bn tiles laid
 * out row-major over the tile grid: tile (tm, tn) -> flags[tm * cdiv(N,bn) + tn].
 * Rows [row0, row1) only are computed when row1 > row0 (a bounded sample for
 * timing); C is then indexed by absolute row. */
void oracle_gemm_chunked_rows(const uint16_t *A, int64_t sAm, int64_t sAk,
                              const uint16_t *B, int64_t sBk, int64_t sBn,
                              float *C, int64_t M, int64_t N, int64_t K,
                              int chunk, int round_every, int64_t row0, int64_t row1) {
    pthread_once(&g_once, build_table);
    if (chunk <= 0) chunk = 32;
    if (round_every <= 0 || round_every > chunk) round_every = chunk;
    if (row1 <= row0) { row0 = 0; row1 = M; }
    int64_t rows = row1 - row0;
    float *a = widen_a(A + row0 * sAm, sAm, sAk, rows, K);
    float *b = widen_b(B, sBk, sBn, K, N);
#pragma omp parallel
    {
        size_t n_alloc = (size_t)(N > 0 ? N : 1);
        double *part = (double *)malloc(sizeof(double) * n_alloc);
        float *half_acc = (float *)malloc(sizeof(float) * n_alloc);
        float *acc = (float *)malloc(sizeof(float) * n_alloc);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const float *ar = a + r * K;
            for (int64_t j = 0; j < N; ++j) acc[j] = 0.0f;
            for (int64_t k0 = 0; k0 < K; k0 += chunk) {
                int64_t k1 = k0 + chunk < K ? k0 + chunk : K;
                /* the FP16 accumulator of this chunk */
                for (int64_t j = 0; j < N; ++j) half_acc[j] = 0.0f;
                for (int64_t s0 = k0; s0 < k1; s0 += round_every) {
                    int64_t s1 = s0 + round_every < k1 ? s0 + round_every : k1;
                    for (int64_t j = 0; j < N; ++j) part[j] = 0.0;
                    for (int64_t k = s0; k < s1; ++k) {
                        double av = ar[k];
                        const float *bk = b + k * N;
                        for (int64_t j = 0; j < N; ++j) part[j] += av * (double)bk[j];
                    }
                    for (int64_t j = 0; j < N; ++j)
                        half_acc[j] = g_h2f[f2h((double)half_acc[j] + part[j])];
                }
                for (int64_t j = 0; j < N; ++j) acc[j] += half_acc[j];
            }
            for (int64_t j = 0; j < N; ++j) C[(row0 + r) * N + j] = acc[j];
        }
        free(part);
        free(half_acc);
        free(acc);
    }
    free(a);
    free(b);
}

void oracle_gemm_chunked(const uint16_t *A, int64_t sAm, int64_t sAk,
                         const uint16_t *B, int64_t sBk, int64_t sBn,
                         float *C, int64_t M, int64_t N, int64_t K,
                         int chunk, int round_every,
                         int64_t bm, int64_t bn, uint8_t *flags, int redo) {
    oracle_gemm_chunked_rows(A, sAm, sAk, B, sBk, sBn, C, M, N, K, chunk, round_every, 0, M);
    if (flags == NULL || bm <= 0 || bn <= 0) return;
    int64_t tm_n = (M + bm - 1) / bm, tn_n = (N + bn - 1) / bn;
    for (int64_t tm = 0; tm < tm_n; ++tm) {
        for (int64_t tn = 0; tn < tn_n; ++tn) {
            int bad = 0;
            int64_t i1 = (tm + 1) * bm < M ? (tm + 1) * bm : M;
            int64_t j1 = (tn + 1) * bn < N ? (tn + 1) * bn : N;
            for (int64_t i = tm * bm; i < i1 && !bad; ++i)
                for (int64_t j = tn * bn; j < j1; ++j)
                    if (!(fabsf(C[i * N + j]) < INFINITY)) { bad = 1; break; }
            flags[tm * tn_n + tn] = (uint8_t)bad;
            if (!bad || !redo) continue;
            for (int64_t i = tm * bm; i < i1; ++i)
                for (int64_t j = tn * bn; j < j1; ++j) {
                    double s = 0.0;
                    for (int64_t k = 0; k < K; ++k)
                        s += (double)g_h2f[A[i * sAm + k * sAk]] * (double)g_h2f[B[k * sBk + j * sBn]];
                    C[i * N + j] = (float)s;
                }
        }
    }
}

/* FP32 -> FP16 round-to-nearest-even (the `acc.to(fp16)` of kernel.py:59). */
void oracle_round_f16(const float *in, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f2h((double)in[i]);
}

/* OpenMP threads the oracle uses (set / query); a launcher such as torchrun
 * may have pinned OMP_NUM_THREADS to 1 for the process. */
void oracle_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
int oracle_threads(void) { return omp_get_max_threads(); }

/* rel() of tests/test_f16acc.py:11-12 for an FP32 candidate; NaN propagates. */
double oracle_rel(const float *x, const double *ref, int64_t n) {
    double num = 0.0, den = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double d = fabs((double)x[i] - ref[i]);
        if (!(d <= num)) num = d;
        double r = fabs(ref[i]);
        if (r > den) den = r;
    }
    return num / den;
}
