// layout.cu -- the wavefront ("WL") layout of per-cell tables and the kernels
// that produce or convert them.
//
// A (B,N,M) table in WL layout is stored stripe by stripe (32*K rows), each
// stripe by local anti-diagonal t in [0, n_diag), n_diag = M + 32K - 1, and
// within an anti-diagonal by position p = k*32 + l for the cell
// (row = s*32K + l*K + k, col = t - l*K - k):
//     wl[((b*n_stripes + s)*n_diag + t)*32K + p]
// The wavefront kernels touch one such anti-diagonal row per step, so every
// per-step load or store of D, E or the scores is one coalesced transaction.
//
//   cost_wl_kernel    D in WL layout straight from x, y:
//                     <false> clamp(||x||^2 + ||y||^2 - 2 x.y, 0)   (distances.py:6-28)
//                     <true>  sum_k (x_k - y_k)^2                     (kernels.py:27-31)
//   rm_to_wl_kernel   row-major (B,N,M) -> WL (caller-supplied cost matrices)
//   wl_to_rm_kernel   WL -> row-major, optionally multiplied by (D_wl > 0),
//                     the clamp mask of the unfused cost's chain rule
#include <algorithm>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int kTB = 32;   // anti-diagonals per tile

__device__ __forceinline__ size_t wl_row_base(const WavePlan& P, int b, int s, int t) {
    return ((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + t) * (32 * P.K);
}

// One CTA per (anti-diagonal block of kTB, stripe, problem).  The block covers
// the parallelogram of cells (q, t - q), q in [0, 32K), t in [t0, t0 + kTB):
// x rows R0 .. R0+32K-1 and y rows t0-32K+1 .. t0+kTB-1, staged in shared
// memory feature chunk by feature chunk.
template <int K, bool DIRECT, int kFC>
__global__ void __launch_bounds__(256) cost_wl_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                      float* __restrict__ Dw, WavePlan P, int dim) {
    constexpr int SR = 32 * K;
    constexpr int YR = SR + kTB - 1;  // y rows touched by the block
    constexpr int CELLS = SR * kTB / 256;
    __shared__ float xs[SR][kFC + 1];     // indexed by stripe position p
    __shared__ float ys[YR][kFC + 1];
    __shared__ float xn[SR], yn[YR];
    const int t0 = blockIdx.x * kTB;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int R0 = s * SR;
    const int j0 = t0 - SR + 1;  // first y row of the block
    const float* xb = x + static_cast<size_t>(b) * P.N * dim;
    const float* yb = y + static_cast<size_t>(b) * P.M * dim;

    float acc[CELLS];
#pragma unroll
    for (int c = 0; c < CELLS; ++c) acc[c] = 0.f;
    if (!DIRECT) {
        for (int i = threadIdx.x; i < SR; i += 256) xn[i] = 0.f;
        for (int i = threadIdx.x; i < YR; i += 256) yn[i] = 0.f;
    }
    for (int f0 = 0; f0 < dim; f0 += kFC) {
        __syncthreads();
        for (int e = threadIdx.x; e < SR * kFC; e += 256) {
            const int p = e / kFC, f = e % kFC;
            const int q = (p % 32) * K + p / 32;
            const int row = R0 + q;
            xs[p][f] = (row < P.N && f0 + f < dim) ? __ldg(xb + static_cast<size_t>(row) * dim + f0 + f) : 0.f;
        }
        for (int e = threadIdx.x; e < YR * kFC; e += 256) {
            const int r = e / kFC, f = e % kFC;
            const int j = j0 + r;
            ys[r][f] = (j >= 0 && j < P.M && f0 + f < dim) ? __ldg(yb + static_cast<size_t>(j) * dim + f0 + f) : 0.f;
        }
        __syncthreads();
        if (!DIRECT) {
            for (int i = threadIdx.x; i < SR; i += 256) {
                float a = xn[i];
#pragma unroll 8
                for (int f = 0; f < kFC; ++f) a = fmaf(xs[i][f], xs[i][f], a);
                xn[i] = a;
            }
            for (int i = threadIdx.x; i < YR; i += 256) {
                float a = yn[i];
#pragma unroll 8
                for (int f = 0; f < kFC; ++f) a = fmaf(ys[i][f], ys[i][f], a);
                yn[i] = a;
            }
        }
#pragma unroll
        for (int c = 0; c < CELLS; ++c) {
            const int idx = threadIdx.x + c * 256;
            const int p = idx % SR;
            const int tt = idx / SR;
            const int q = (p % 32) * K + p / 32;
            const int r = tt + (SR - 1) - q;  // y row of cell (q, t0 + tt - q), relative to j0
            float a = acc[c];
#pragma unroll 8
            for (int f = 0; f < kFC; ++f) {
                if (DIRECT) {
                    const float df = xs[p][f] - ys[r][f];
                    a = fmaf(df, df, a);
                } else {
                    a = fmaf(xs[p][f], ys[r][f], a);
                }
            }
            acc[c] = a;
        }
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < CELLS; ++c) {
        const int idx = threadIdx.x + c * 256;
        const int p = idx % SR;
        const int tt = idx / SR;
        const int t = t0 + tt;
        if (t >= P.n_diag) continue;
        const int q = (p % 32) * K + p / 32;
        const int col = t - q;
        if (R0 + q >= P.N || col < 0 || col >= P.M) continue;
        float v = acc[c];
        if (!DIRECT) v = fmaxf((xn[p] + yn[tt + (SR - 1) - q]) - 2.f * v, 0.f);
        Dw[wl_row_base(P, b, s, t) + p] = v;
    }
}

// Row-major <-> WL through a shared-memory tile of 32K rows x kTB anti-diagonals.
template <int K>
__global__ void __launch_bounds__(256) rm_to_wl_kernel(const float* __restrict__ A, float* __restrict__ Aw, WavePlan P) {
    constexpr int SR = 32 * K;
    __shared__ float tile[SR][kTB + 1];
    const int t0 = blockIdx.x * kTB;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int R0 = s * SR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Rows q: cells (q, t0 + lane - q) are 32 consecutive columns of row-major A.
    for (int q = warp; q < SR; q += 8) {
        const int row = R0 + q;
        const int col = t0 + lane - q;
        float v = 0.f;
        if (row < P.N && col >= 0 && col < P.M) v = __ldg(A + (static_cast<size_t>(b) * P.N + row) * P.M + col);
        tile[q][lane] = v;
    }
    __syncthreads();
    for (int tt = warp; tt < kTB; tt += 8) {
        const int t = t0 + tt;
        if (t >= P.n_diag) break;
        float* dst = Aw + wl_row_base(P, b, s, t);
#pragma unroll
        for (int k = 0; k < K; ++k) dst[k * 32 + lane] = tile[lane * K + k][tt];
    }
}

template <int K>
__global__ void __launch_bounds__(256) wl_to_rm_kernel(const float* __restrict__ Aw, const float* __restrict__ maskw,
                                                       float* __restrict__ A, WavePlan P) {
    constexpr int SR = 32 * K;
    __shared__ float tile[SR][kTB + 1];
    const int t0 = blockIdx.x * kTB;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int R0 = s * SR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int tt = warp; tt < kTB; tt += 8) {
        const int t = t0 + tt;
        if (t >= P.n_diag) break;
        const size_t base = wl_row_base(P, b, s, t);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float v = __ldg(Aw + base + k * 32 + lane);
            if (maskw && !(__ldg(maskw + base + k * 32 + lane) > 0.f)) v = 0.f;
            tile[lane * K + k][tt] = v;
        }
    }
    __syncthreads();
    for (int q = warp; q < SR; q += 8) {
        const int row = R0 + q;
        const int col = t0 + lane - q;
        if (row < P.N && col >= 0 && col < P.M && t0 + lane < P.n_diag)
            A[(static_cast<size_t>(b) * P.N + row) * P.M + col] = tile[q][lane];
    }
}

static dim3 wl_grid(const WavePlan& P) {
    return dim3((P.n_diag + kTB - 1) / kTB, P.n_stripes, P.B);
}

template <int K, int FC>
static void cost_wl_launch(const float* x, const float* y, float* Dw, const WavePlan& P, int dim, bool direct,
                           cudaStream_t stream) {
    const dim3 g = wl_grid(P);
    if (direct) cost_wl_kernel<K, true, FC><<<g, 256, 0, stream>>>(x, y, Dw, P, dim);
    else cost_wl_kernel<K, false, FC><<<g, 256, 0, stream>>>(x, y, Dw, P, dim);
}

template <int K>
static void cost_wl_by_dim(const float* x, const float* y, float* Dw, const WavePlan& P, int dim, bool direct,
                           cudaStream_t stream) {
    // Feature chunk sized to the feature count: no padded work for small dims.
    if (dim <= 8) cost_wl_launch<K, 8>(x, y, Dw, P, dim, direct, stream);
    else if (dim <= 16) cost_wl_launch<K, 16>(x, y, Dw, P, dim, direct, stream);
    else cost_wl_launch<K, 32>(x, y, Dw, P, dim, direct, stream);
}

cudaError_t launch_cost_wl(const float* x, const float* y, float* Dw, const WavePlan& P, int dim, bool direct,
                           cudaStream_t stream) {
    switch (P.K) {
        case 1: cost_wl_by_dim<1>(x, y, Dw, P, dim, direct, stream); break;
        case 2: cost_wl_by_dim<2>(x, y, Dw, P, dim, direct, stream); break;
        case 4: cost_wl_by_dim<4>(x, y, Dw, P, dim, direct, stream); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_rm_to_wl(const float* A, float* Aw, const WavePlan& P, cudaStream_t stream) {
    const dim3 g = wl_grid(P);
    switch (P.K) {
        case 1: rm_to_wl_kernel<1><<<g, 256, 0, stream>>>(A, Aw, P); break;
        case 2: rm_to_wl_kernel<2><<<g, 256, 0, stream>>>(A, Aw, P); break;
        case 4: rm_to_wl_kernel<4><<<g, 256, 0, stream>>>(A, Aw, P); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_wl_to_rm(const float* Aw, const float* maskw, float* A, const WavePlan& P, cudaStream_t stream) {
    const dim3 g = wl_grid(P);
    switch (P.K) {
        case 1: wl_to_rm_kernel<1><<<g, 256, 0, stream>>>(Aw, maskw, A, P); break;
        case 2: wl_to_rm_kernel<2><<<g, 256, 0, stream>>>(Aw, maskw, A, P); break;
        case 4: wl_to_rm_kernel<4><<<g, 256, 0, stream>>>(Aw, maskw, A, P); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sdtw
