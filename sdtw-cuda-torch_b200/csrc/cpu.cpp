// cpu.cpp -- Soft-DTW on the host, for CPU tensors (OpenMP over the batch).
//
// Same recurrences as the device kernels, evaluated in double precision:
//   forward   R[i,j] = D[i-1,j-1] + softmin_gamma(R[i-1,j-1], R[i-1,j], R[i,j-1])
//             (softdtw_cuda/cuda/launcher.py:307-324 semantics: R[0,0] = 0,
//             other borders +inf, cells with 0 < bandwidth < |i-j| stay +inf)
//   backward  E[p] = sum_c E[c] * w(c <- p), where w(c <- p) is the softmax
//             weight of predecessor p among c's three predecessors; this equals
//             exp((R[c] - D[c] - R[p]) / gamma) of launcher.py:327-353.
// The (B, N+2, M+2) R table uses the reference layout.  Rows are swept i-major
// so the inner loop walks memory contiguously.
#include <cmath>
#include <cstddef>
#include <limits>
#include <vector>

#include "../../include/sdtw_b200.h"

namespace {

inline bool pruned(double bw, int i, int j) { return bw > 0.0 && std::fabs(static_cast<double>(i - j)) > bw; }

}  // namespace

extern "C" {

int sdtw_cpu_forward_f64(const double* D, double* R, double* out, int B, int N, int M, double gamma,
                         double bandwidth) {
    if (B <= 0 || N <= 0 || M <= 0 || !(gamma > 0.0) || !std::isfinite(gamma) || !D || !R || !out)
        return SDTW_ERR_INVALID_ARGUMENT;
    const double inf = std::numeric_limits<double>::infinity();
    const size_t W = static_cast<size_t>(M) + 2;
    const size_t plane = (static_cast<size_t>(N) + 2) * W;
    const double ig = 1.0 / gamma;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        double* Rb = R + static_cast<size_t>(b) * plane;
        const double* Db = D + static_cast<size_t>(b) * N * M;
        for (size_t t = 0; t < plane; ++t) Rb[t] = inf;
        Rb[0] = 0.0;
        for (int i = 1; i <= N; ++i) {
            const double* up = Rb + static_cast<size_t>(i - 1) * W;
            double* cur = Rb + static_cast<size_t>(i) * W;
            for (int j = 1; j <= M; ++j) {
                if (pruned(bandwidth, i, j)) continue;
                const double a = -up[j - 1] * ig, u = -up[j] * ig, l = -cur[j - 1] * ig;
                const double m = std::fmax(std::fmax(a, u), l);
                double v;
                if (m == -inf) {
                    v = inf;
                } else {
                    const double s = std::exp(a - m) + std::exp(u - m) + std::exp(l - m);
                    v = Db[static_cast<size_t>(i - 1) * M + (j - 1)] - gamma * (std::log(s) + m);
                }
                cur[j] = v;
            }
        }
        out[b] = Rb[static_cast<size_t>(N) * W + M];
    }
    return SDTW_OK;
}

int sdtw_cpu_backward_f64(const double* R, const double* grad_out, double* E, int B, int N, int M, double gamma,
                          double bandwidth) {
    if (B <= 0 || N <= 0 || M <= 0 || !(gamma > 0.0) || !std::isfinite(gamma) || !R || !E)
        return SDTW_ERR_INVALID_ARGUMENT;
    const size_t W = static_cast<size_t>(M) + 2;
    const size_t plane = (static_cast<size_t>(N) + 2) * W;
    const double ig = 1.0 / gamma;
#pragma omp parallel
    {
        // Per-thread rows of pending contributions: row i+1's messages to row i.
        std::vector<double> below_u(static_cast<size_t>(M) + 2), below_d(static_cast<size_t>(M) + 2);
        std::vector<double> cur_u(static_cast<size_t>(M) + 2), cur_d(static_cast<size_t>(M) + 2);
#pragma omp for schedule(dynamic, 1)
        for (int b = 0; b < B; ++b) {
            const double* Rb = R + static_cast<size_t>(b) * plane;
            double* Eb = E + static_cast<size_t>(b) * N * M;
            const double g = grad_out ? grad_out[b] : 1.0;
            std::fill(below_u.begin(), below_u.end(), 0.0);
            std::fill(below_d.begin(), below_d.end(), 0.0);
            for (int i = N; i >= 1; --i) {
                double left_in = 0.0;  // contribution from (i, j+1) to (i, j)
                std::fill(cur_u.begin(), cur_u.end(), 0.0);
                std::fill(cur_d.begin(), cur_d.end(), 0.0);
                for (int j = M; j >= 1; --j) {
                    double e = 0.0;
                    if (!pruned(bandwidth, i, j)) {
                        e = left_in + below_u[j] + below_d[j + 1];
                        if (i == N && j == M) e = g;
                    }
                    Eb[static_cast<size_t>(i - 1) * M + (j - 1)] = e;
                    double wd = 0.0, wu = 0.0, wl = 0.0;
                    if (e != 0.0) {
                        const double td = -Rb[static_cast<size_t>(i - 1) * W + j - 1] * ig;
                        const double tu = -Rb[static_cast<size_t>(i - 1) * W + j] * ig;
                        const double tl = -Rb[static_cast<size_t>(i) * W + j - 1] * ig;
                        const double m = std::fmax(std::fmax(td, tu), tl);
                        if (std::isfinite(m)) {
                            const double ed = std::exp(td - m), eu = std::exp(tu - m), el = std::exp(tl - m);
                            const double inv = 1.0 / (ed + eu + el);
                            wd = ed * inv;
                            wu = eu * inv;
                            wl = el * inv;
                        }
                    }
                    left_in = e * wl;    // to (i, j-1)
                    cur_u[j] = e * wu;   // to (i-1, j)
                    cur_d[j] = e * wd;   // to (i-1, j-1), read by row i-1 as below_d[(j-1)+1]
                }
                below_u.swap(cur_u);
                below_d.swap(cur_d);
            }
        }
    }
    return SDTW_OK;
}

}  // extern "C"
