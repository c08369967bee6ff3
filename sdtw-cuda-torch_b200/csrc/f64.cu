// f64.cu -- the float64 CUDA path.
//
// The reference runs float64 tensors on the GPU with its float64 arithmetic
// (kernels.py computes in double), and its CPU path keeps the whole pipeline in
// double for float64 inputs (launcher.py:307-353).  These kernels restate that
// pipeline on the device, in double, with the reference's (B, N+2, M+2) R
// layout, so that float64 CUDA tensors (gradcheck on the device, for one) get
// results that agree with the float64 reference to rounding.  They are a
// correctness path, not a fast one: one CTA per problem sweeps the
// anti-diagonals with a block barrier per diagonal.
//
//   fwd_f64_kernel   launcher.py:307-324  R[i,j] = D + softmin(R[i-1,j-1], R[i-1,j], R[i,j-1])
//   bwd_f64_kernel   launcher.py:327-353  E[i,j] = sum over successors of E[s] * exp((R[s] - R[i,j] - D[s]) / gamma),
//                                          then grad_D = grad_out[b] * E (autograd.py:46-47)
//   cost_f64_kernel  kernels.py:27-31     D[i,j] = sum_k (x_ik - y_jk)^2 (the fused cost, direct form)
//   grad_f64_kernel  autograd_xy.py:41-49 grad_x = 2 (x rowsum(G) - G y), grad_y = 2 (y colsum(G) - G^T x),
//                                          the sums over the other sequence in double, in index order
#include <cmath>
#include <cstdint>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int kF64Threads = 512;

// Cell (i, j), 1-based, is skipped when 0 < bandwidth < |i - j| (launcher.py:315, :345).
__device__ __forceinline__ bool f64_skip(double bw, int i, int j) {
    return 0.0 < bw && bw < fabs(static_cast<double>(i - j));
}

__global__ void __launch_bounds__(kF64Threads) fwd_f64_kernel(const double* __restrict__ D, double* __restrict__ R,
                                                              double* __restrict__ out, int N, int M, double gamma,
                                                              double bw) {
    const int b = blockIdx.x;
    const size_t W = static_cast<size_t>(M) + 2;
    double* Rb = R + static_cast<size_t>(b) * (N + 2) * W;
    const double* Db = D + static_cast<size_t>(b) * N * M;
    const size_t total = static_cast<size_t>(N + 2) * W;
    for (size_t e = threadIdx.x; e < total; e += blockDim.x) Rb[e] = e == 0 ? 0.0 : INFINITY;
    __syncthreads();
    // Anti-diagonal s = i + j (1-based cells), s = 2 .. N + M.
    for (int s = 2; s <= N + M; ++s) {
        const int i_lo = max(1, s - M), i_hi = min(N, s - 1);
        for (int i = i_lo + static_cast<int>(threadIdx.x); i <= i_hi; i += blockDim.x) {
            const int j = s - i;
            if (f64_skip(bw, i, j)) continue;
            const double r0 = -Rb[(i - 1) * W + (j - 1)] / gamma;
            const double r1 = -Rb[(i - 1) * W + j] / gamma;
            const double r2 = -Rb[i * W + (j - 1)] / gamma;
            const double rmax = fmax(fmax(r0, r1), r2);
            const double rsum = exp(r0 - rmax) + exp(r1 - rmax) + exp(r2 - rmax);
            const double softmin = -gamma * (log(rsum) + rmax);
            Rb[i * W + j] = Db[static_cast<size_t>(i - 1) * M + (j - 1)] + softmin;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) out[b] = Rb[N * W + M];
}

// The reference's backward edits a copy of R (launcher.py:337-342) and pads D
// with zeros; both are applied here on the fly, reading the forward's R as is:
//   R'(i, j) = -inf on row N+1 and column M+1, R(N, M) at (N+1, M+1), and -inf
//   where R is infinite (the loop's first statement, applied to every cell);
//   D'(i, j) = D(i-1, j-1) inside the table, 0 on the padding;
//   E(N+1, M+1) = 1, 0 elsewhere on the padding.
__global__ void __launch_bounds__(kF64Threads) bwd_f64_kernel(const double* __restrict__ D,
                                                              const double* __restrict__ R,
                                                              const double* __restrict__ grad_out,
                                                              double* __restrict__ E, int N, int M, double gamma,
                                                              double bw) {
    const int b = blockIdx.x;
    const size_t W = static_cast<size_t>(M) + 2;
    const double* Rb = R + static_cast<size_t>(b) * (N + 2) * W;
    const double* Db = D + static_cast<size_t>(b) * N * M;
    double* Eb = E + static_cast<size_t>(b) * N * M;
    const double NEG = -INFINITY;
    auto rp = [&](int i, int j) -> double {
        if (i == N + 1 && j == M + 1) {
            const double v = Rb[N * W + M];
            return isinf(v) ? NEG : v;
        }
        if (i == N + 1 || j == M + 1) return NEG;
        const double v = Rb[i * W + j];
        return isinf(v) ? NEG : v;
    };
    auto dp = [&](int i, int j) -> double {
        return (i <= N && j <= M) ? Db[static_cast<size_t>(i - 1) * M + (j - 1)] : 0.0;
    };
    auto ev = [&](int i, int j) -> double {
        if (i == N + 1 && j == M + 1) return 1.0;
        if (i == N + 1 || j == M + 1) return 0.0;
        return Eb[static_cast<size_t>(i - 1) * M + (j - 1)];
    };
    for (size_t e = threadIdx.x; e < static_cast<size_t>(N) * M; e += blockDim.x) Eb[e] = 0.0;
    __syncthreads();
    for (int s = N + M; s >= 2; --s) {
        const int i_lo = max(1, s - M), i_hi = min(N, s - 1);
        for (int i = i_lo + static_cast<int>(threadIdx.x); i <= i_hi; i += blockDim.x) {
            const int j = s - i;
            if (f64_skip(bw, i, j)) continue;
            const double rc = rp(i, j);
            const double a = exp(((rp(i + 1, j) - rc) - dp(i + 1, j)) / gamma);
            const double bb = exp(((rp(i, j + 1) - rc) - dp(i, j + 1)) / gamma);
            const double c = exp(((rp(i + 1, j + 1) - rc) - dp(i + 1, j + 1)) / gamma);
            Eb[static_cast<size_t>(i - 1) * M + (j - 1)] = ev(i + 1, j) * a + ev(i, j + 1) * bb + ev(i + 1, j + 1) * c;
        }
        __syncthreads();
    }
    if (grad_out) {
        const double g = grad_out[b];
        for (size_t e = threadIdx.x; e < static_cast<size_t>(N) * M; e += blockDim.x) Eb[e] *= g;
    }
}

// One thread per cell; the features are summed in order.
__global__ void __launch_bounds__(256) cost_f64_kernel(const double* __restrict__ x, const double* __restrict__ y,
                                                       double* __restrict__ D, int N, int M, int dim) {
    const int b = blockIdx.z;
    const int i = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= M) return;
    const double* xr = x + (static_cast<size_t>(b) * N + i) * dim;
    const double* yr = y + (static_cast<size_t>(b) * M + j) * dim;
    double acc = 0.0;
    for (int k = 0; k < dim; ++k) {
        const double d = xr[k] - yr[k];
        acc += d * d;
    }
    D[(static_cast<size_t>(b) * N + i) * M + j] = acc;
}

cudaError_t launch_forward_f64(const double* D, double* R, double* out, int B, int N, int M, double gamma, double bw,
                               cudaStream_t stream) {
    fwd_f64_kernel<<<B, kF64Threads, 0, stream>>>(D, R, out, N, M, gamma, bw);
    return cudaGetLastError();
}

cudaError_t launch_backward_f64(const double* D, const double* R, const double* grad_out, double* E, int B, int N,
                                int M, double gamma, double bw, cudaStream_t stream) {
    bwd_f64_kernel<<<B, kF64Threads, 0, stream>>>(D, R, grad_out, E, N, M, gamma, bw);
    return cudaGetLastError();
}

cudaError_t launch_cost_f64(const double* x, const double* y, double* D, int B, int N, int M, int dim,
                            cudaStream_t stream) {
    const dim3 grid((M + 255) / 256, N, B);
    cost_f64_kernel<<<grid, 256, 0, stream>>>(x, y, D, N, M, dim);
    return cudaGetLastError();
}

// One thread per (row r of the own sequence, feature f): lanes take 32
// consecutive features of one row (the G element is a broadcast, the other
// sequence's row a coalesced load); 8 rows per block.  COL = false: grad_x,
// own = x (rows N), G row r; COL = true: grad_y, own = y (rows M), G column r.
template <bool COL>
__global__ void __launch_bounds__(256) grad_f64_kernel(const double* __restrict__ G, const double* __restrict__ own,
                                                       const double* __restrict__ other, double* __restrict__ g,
                                                       int N, int M, int dim) {
    const int b = blockIdx.z;
    const int r = blockIdx.x * 8 + threadIdx.y;
    const int f = blockIdx.y * 32 + threadIdx.x;
    const int rows = COL ? M : N, cols = COL ? N : M;
    if (r >= rows || f >= dim) return;
    const double* Gb = G + static_cast<size_t>(b) * N * M;
    const double* ob = other + static_cast<size_t>(b) * cols * dim;
    double s = 0.0, t = 0.0;
    for (int c = 0; c < cols; ++c) {
        const double w = COL ? Gb[static_cast<size_t>(c) * M + r] : Gb[static_cast<size_t>(r) * M + c];
        s += w;
        t = fma(w, ob[static_cast<size_t>(c) * dim + f], t);
    }
    const size_t o = (static_cast<size_t>(b) * rows + r) * dim + f;
    g[o] = 2.0 * (own[o] * s - t);
}

cudaError_t launch_grad_f64(const double* G, const double* x, const double* y, double* gx, double* gy, int B, int N,
                            int M, int dim, cudaStream_t stream) {
    const dim3 block(32, 8);
    if (gx) {
        grad_f64_kernel<false><<<dim3((N + 7) / 8, (dim + 31) / 32, B), block, 0, stream>>>(G, x, y, gx, N, M, dim);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (gy) grad_f64_kernel<true><<<dim3((M + 7) / 8, (dim + 31) / 32, B), block, 0, stream>>>(G, y, x, gy, N, M, dim);
    return cudaGetLastError();
}

}  // namespace sdtw
