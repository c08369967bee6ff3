/*
 * sdtw_oracle.c -- CPU restatement of the reference Soft-DTW dynamic programme.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under sdtw-cuda-torch_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and the cpu_baseline / reference arm of bench.py may load it.  The product
 * never links or calls it.
 *
 * It restates, in plain C with OpenMP over the batch (the reference uses a
 * Numba prange over the batch), the reference's CPU implementation:
 *
 *   forward   softdtw_cuda/cuda/launcher.py:307-324  (_softdtw_forward_cpu_np)
 *   backward  softdtw_cuda/cuda/launcher.py:327-353  (_softdtw_backward_cpu_np)
 *   wrappers  softdtw_cuda/cuda/launcher.py:356-368  (R and E stored in D's dtype)
 *
 * Arithmetic follows the reference's dtype rules exactly, because the
 * reference's gradients are sensitive to them:
 *
 *   * forward: the R table is float64 inside Numba (np.ones(float32) * np.inf is
 *     typed float64 there), so the whole recurrence runs in double with the
 *     float32 cost promoted; the wrapper then rounds R to the input dtype.
 *   * backward, float32 inputs: R and the zero-padded D are float32 arrays, so
 *     (R[succ] - R[cell] - D[succ]) is evaluated in float32 and only the
 *     division by gamma promotes to double; E is a float32 array, so every
 *     E cell is rounded to float32 when stored.
 *   * backward, float64 inputs: everything in double.
 *
 * Bandwidth: a cell (i, j) (1-based, padded coordinates) is skipped when
 * 0 < bandwidth < |i - j|, as in launcher.py:315 and :345.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define IDX(b, i, j) (((size_t)(b) * (size_t)(N + 2) + (size_t)(i)) * (size_t)(M + 2) + (size_t)(j))

static inline double dmax(double a, double b) { return a > b ? a : b; }

/* launcher.py:307-324.  D: (B,N,M) as double (exact copy of the caller's
 * float32 or float64 values).  R64: (B,N+2,M+2) output, double. */
static void forward_core(const double *D, int B, int N, int M, double gamma,
                         double bandwidth, double *R) {
    size_t total = (size_t)B * (size_t)(N + 2) * (size_t)(M + 2);
    for (size_t t = 0; t < total; ++t) R[t] = INFINITY;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        R[IDX(b, 0, 0)] = 0.0;
        for (int j = 1; j <= M; ++j) {
            for (int i = 1; i <= N; ++i) {
                if (0.0 < bandwidth && bandwidth < fabs((double)(i - j))) continue;
                double r0 = -R[IDX(b, i - 1, j - 1)] / gamma;
                double r1 = -R[IDX(b, i - 1, j)] / gamma;
                double r2 = -R[IDX(b, i, j - 1)] / gamma;
                double rmax = dmax(dmax(r0, r1), r2);
                double rsum = exp(r0 - rmax) + exp(r1 - rmax) + exp(r2 - rmax);
                double softmin = -gamma * (log(rsum) + rmax);
                R[IDX(b, i, j)] = D[((size_t)b * N + (i - 1)) * M + (j - 1)] + softmin;
            }
        }
    }
}

void oracle_forward_f32(const float *D32, int B, int N, int M, double gamma,
                        double bandwidth, double *R64, float *R32) {
    size_t nd = (size_t)B * N * M;
    double *D = (double *)malloc(nd * sizeof(double));
    for (size_t t = 0; t < nd; ++t) D[t] = (double)D32[t];
    forward_core(D, B, N, M, gamma, bandwidth, R64);
    free(D);
    if (R32) {
        size_t total = (size_t)B * (size_t)(N + 2) * (size_t)(M + 2);
        for (size_t t = 0; t < total; ++t) R32[t] = (float)R64[t];
    }
}

void oracle_forward_f64(const double *D, int B, int N, int M, double gamma,
                        double bandwidth, double *R64) {
    forward_core(D, B, N, M, gamma, bandwidth, R64);
}

/* launcher.py:327-353 with float32 arrays.  R32_in is the (B,N+2,M+2) float32
 * table from the forward; it is copied (launcher.py:366 copies before the
 * in-place boundary edits).  E: (B,N,M) float32 output. */
void oracle_backward_f32(const float *D32, const float *R32_in, int B, int N, int M,
                         double gamma, double bandwidth, float *E_out) {
    size_t total = (size_t)B * (size_t)(N + 2) * (size_t)(M + 2);
    float *R = (float *)malloc(total * sizeof(float));
    float *Dp = (float *)calloc(total, sizeof(float));
    float *E = (float *)calloc(total, sizeof(float));
    memcpy(R, R32_in, total * sizeof(float));
    for (int b = 0; b < B; ++b) {
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < M; ++j)
                Dp[IDX(b, i + 1, j + 1)] = D32[((size_t)b * N + i) * M + j];
        E[IDX(b, N + 1, M + 1)] = 1.0f;
        for (int i = 0; i < N + 2; ++i) R[IDX(b, i, M + 1)] = -INFINITY;
        for (int j = 0; j < M + 2; ++j) R[IDX(b, N + 1, j)] = -INFINITY;
        R[IDX(b, N + 1, M + 1)] = R[IDX(b, N, M)];
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        for (int j = M; j >= 1; --j) {
            for (int i = N; i >= 1; --i) {
                if (isinf(R[IDX(b, i, j)])) R[IDX(b, i, j)] = -INFINITY;
                if (0.0 < bandwidth && bandwidth < fabs((double)(i - j))) continue;
                float rc = R[IDX(b, i, j)];
                /* float32 subtraction chain, then promotion by the division. */
                float fa = (R[IDX(b, i + 1, j)] - rc) - Dp[IDX(b, i + 1, j)];
                float fb = (R[IDX(b, i, j + 1)] - rc) - Dp[IDX(b, i, j + 1)];
                float fc = (R[IDX(b, i + 1, j + 1)] - rc) - Dp[IDX(b, i + 1, j + 1)];
                double a = exp((double)fa / gamma);
                double bb = exp((double)fb / gamma);
                double c = exp((double)fc / gamma);
                double e = (double)E[IDX(b, i + 1, j)] * a + (double)E[IDX(b, i, j + 1)] * bb +
                           (double)E[IDX(b, i + 1, j + 1)] * c;
                E[IDX(b, i, j)] = (float)e;
            }
        }
    }
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < M; ++j)
                E_out[((size_t)b * N + i) * M + j] = E[IDX(b, i + 1, j + 1)];
    free(R);
    free(Dp);
    free(E);
}

/* launcher.py:327-353 with float64 arrays (the whole pipeline in double). */
void oracle_backward_f64(const double *D64, const double *R64_in, int B, int N, int M,
                         double gamma, double bandwidth, double *E_out) {
    size_t total = (size_t)B * (size_t)(N + 2) * (size_t)(M + 2);
    double *R = (double *)malloc(total * sizeof(double));
    double *Dp = (double *)calloc(total, sizeof(double));
    double *E = (double *)calloc(total, sizeof(double));
    memcpy(R, R64_in, total * sizeof(double));
    for (int b = 0; b < B; ++b) {
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < M; ++j)
                Dp[IDX(b, i + 1, j + 1)] = D64[((size_t)b * N + i) * M + j];
        E[IDX(b, N + 1, M + 1)] = 1.0;
        for (int i = 0; i < N + 2; ++i) R[IDX(b, i, M + 1)] = -INFINITY;
        for (int j = 0; j < M + 2; ++j) R[IDX(b, N + 1, j)] = -INFINITY;
        R[IDX(b, N + 1, M + 1)] = R[IDX(b, N, M)];
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        for (int j = M; j >= 1; --j) {
            for (int i = N; i >= 1; --i) {
                if (isinf(R[IDX(b, i, j)])) R[IDX(b, i, j)] = -INFINITY;
                if (0.0 < bandwidth && bandwidth < fabs((double)(i - j))) continue;
                double rc = R[IDX(b, i, j)];
                double a = exp((R[IDX(b, i + 1, j)] - rc - Dp[IDX(b, i + 1, j)]) / gamma);
                double bb = exp((R[IDX(b, i, j + 1)] - rc - Dp[IDX(b, i, j + 1)]) / gamma);
                double c = exp((R[IDX(b, i + 1, j + 1)] - rc - Dp[IDX(b, i + 1, j + 1)]) / gamma);
                E[IDX(b, i, j)] = E[IDX(b, i + 1, j)] * a + E[IDX(b, i, j + 1)] * bb +
                                  E[IDX(b, i + 1, j + 1)] * c;
            }
        }
    }
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < M; ++j)
                E_out[((size_t)b * N + i) * M + j] = E[IDX(b, i + 1, j + 1)];
    free(R);
    free(Dp);
    free(E);
}

/* Fused-mode cost, softdtw_cuda/cuda/kernels.py:27-31: a direct difference
 * accumulated in double (Numba types the accumulator `cost = 0.0` as float64).
 * x: (B,N,Dim), y: (B,M,Dim) float32 -> D: (B,N,M) double. */
void oracle_cost_direct_f32(const float *x, const float *y, int B, int N, int M, int Dim,
                            double *D) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < N; ++i) {
            const float *xi = x + ((size_t)b * N + i) * Dim;
            for (int j = 0; j < M; ++j) {
                const float *yj = y + ((size_t)b * M + j) * Dim;
                double cost = 0.0;
                for (int k = 0; k < Dim; ++k) {
                    /* diff and diff*diff are float32 expressions (both
                     * operands float32); only the accumulation is double. */
                    float diff = xi[k] - yj[k];
                    float sq = diff * diff;
                    cost += (double)sq;
                }
                D[((size_t)b * N + i) * M + j] = cost;
            }
        }
}

/* Thread count of the oracle's parallel regions (the bench's reference arm uses
 * every host core even where the launcher set OMP_NUM_THREADS=1). */
void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    extern void omp_set_num_threads(int);
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}
