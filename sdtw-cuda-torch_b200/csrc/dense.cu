// dense.cu -- cost matrix and the chain rule of the squared-Euclidean cost.
//
//   cost_kernel<false>  D = clamp(||x_i||^2 + ||y_j||^2 - 2 x_i.y_j, 0)
//                       softdtw_cuda/distances.py:6-28 (unfused cost)
//   cost_kernel<true>   D = sum_k (x_ik - y_jk)^2
//                       softdtw_cuda/cuda/kernels.py:27-31 (fused-mode cost)
//   grad_x / grad_y     G = E (optionally masked where the clamp was active);
//                       gx_i = 2 (x_i sum_j G_ij - sum_j G_ij y_j)
//                       gy_j = 2 (y_j sum_i G_ij - sum_i G_ij x_i)
//                       softdtw_cuda/autograd_xy.py:41-49 and the autograd of
//                       distances.py:20-28.
// fp32 SIMT tiles.
#include <algorithm>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int CT = 64;   // cost tile
constexpr int CF = 16;   // feature chunk

template <bool DIRECT>
__global__ void __launch_bounds__(256) cost_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                   float* __restrict__ D, int N, int M, int dim) {
    __shared__ float xs[CF][CT + 4];
    __shared__ float ys[CF][CT + 4];
    const int b = blockIdx.z;
    const int i0 = blockIdx.y * CT;
    const int j0 = blockIdx.x * CT;
    const int tx = threadIdx.x & 15;
    const int ty = threadIdx.x >> 4;
    const float* xb = x + static_cast<size_t>(b) * N * dim;
    const float* yb = y + static_cast<size_t>(b) * M * dim;
    float acc[4][4];
    float xn[4], yn[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        xn[r] = yn[r] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
    }
    for (int f0 = 0; f0 < dim; f0 += CF) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int e = threadIdx.x + r * 256;
            const int i = e / CF;
            const int f = e % CF;
            xs[f][i] = (i0 + i < N && f0 + f < dim) ? __ldg(xb + static_cast<size_t>(i0 + i) * dim + f0 + f) : 0.f;
            ys[f][i] = (j0 + i < M && f0 + f < dim) ? __ldg(yb + static_cast<size_t>(j0 + i) * dim + f0 + f) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int f = 0; f < CF; ++f) {
            float xv[4], yv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                xv[r] = xs[f][ty * 4 + r];
                yv[r] = ys[f][tx * 4 + r];
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (!DIRECT) {
                    xn[r] = fmaf(xv[r], xv[r], xn[r]);
                    yn[r] = fmaf(yv[r], yv[r], yn[r]);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (DIRECT) {
                        const float df = xv[r] - yv[c];
                        acc[r][c] = fmaf(df, df, acc[r][c]);
                    } else {
                        acc[r][c] = fmaf(xv[r], yv[c], acc[r][c]);
                    }
                }
            }
        }
        __syncthreads();
    }
    float* Db = D + static_cast<size_t>(b) * N * M;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int i = i0 + ty * 4 + r;
        if (i >= N) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int j = j0 + tx * 4 + c;
            if (j >= M) continue;
            float v;
            if (DIRECT) v = acc[r][c];
            else v = fmaxf((xn[r] + yn[c]) - 2.f * acc[r][c], 0.f);
            Db[static_cast<size_t>(i) * M + j] = v;
        }
    }
}

cudaError_t launch_cost(const float* x, const float* y, float* D, int B, int N, int M, int dim, bool direct,
                        cudaStream_t stream) {
    dim3 grid((M + CT - 1) / CT, (N + CT - 1) / CT, B);
    if (direct) cost_kernel<true><<<grid, 256, 0, stream>>>(x, y, D, N, M, dim);
    else cost_kernel<false><<<grid, 256, 0, stream>>>(x, y, D, N, M, dim);
    return cudaGetLastError();
}

constexpr int GT = 32;   // rows (or columns) per CTA

// gx[b, i0:i0+32, :] from G rows i0..i0+31 and all of y[b].  GF = feature
// chunk (8, 16, 32 or 64, chosen from the feature count).
template <int GF>
__global__ void __launch_bounds__(256) grad_x_kernel(const float* __restrict__ G, const float* __restrict__ mask,
                                                     const float* __restrict__ x, const float* __restrict__ y,
                                                     float* __restrict__ gx, int N, int M, int dim) {
    __shared__ float Gs[GT][GT + 1];
    __shared__ float Ys[GT][GF + 1];
    const int b = blockIdx.y;
    const int i0 = blockIdx.x * GT;
    const int tx = threadIdx.x & 7;
    const int ty = threadIdx.x >> 3;
    const float* Gb = G + static_cast<size_t>(b) * N * M;
    const float* Mb = mask ? mask + static_cast<size_t>(b) * N * M : nullptr;
    const float* yb = y + static_cast<size_t>(b) * M * dim;
    for (int fc = 0; fc < dim; fc += GF) {
        float acc[GF / 8];
#pragma unroll
        for (int u = 0; u < GF / 8; ++u) acc[u] = 0.f;
        float rs = 0.f;
        for (int j0 = 0; j0 < M; j0 += GT) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int e = threadIdx.x + r * 256;
                const int ii = e / GT, jj = e % GT;
                float gv = 0.f;
                if (i0 + ii < N && j0 + jj < M) {
                    const size_t off = static_cast<size_t>(i0 + ii) * M + j0 + jj;
                    gv = __ldg(Gb + off);
                    if (Mb && !(__ldg(Mb + off) > 0.f)) gv = 0.f;
                }
                Gs[ii][jj] = gv;
            }
#pragma unroll
            for (int r = 0; r < GF / 8; ++r) {
                const int e = threadIdx.x + r * 256;
                const int jj = e / GF, ff = e % GF;
                Ys[jj][ff] = (j0 + jj < M && fc + ff < dim) ? __ldg(yb + static_cast<size_t>(j0 + jj) * dim + fc + ff) : 0.f;
            }
            __syncthreads();
#pragma unroll 8
            for (int jj = 0; jj < GT; ++jj) {
                const float gv = Gs[ty][jj];
                rs += gv;
#pragma unroll
                for (int u = 0; u < GF / 8; ++u) acc[u] = fmaf(gv, Ys[jj][tx + 8 * u], acc[u]);
            }
            __syncthreads();
        }
        const int i = i0 + ty;
        if (i < N) {
#pragma unroll
            for (int u = 0; u < GF / 8; ++u) {
                const int f = fc + tx + 8 * u;
                if (f < dim) {
                    const size_t o = (static_cast<size_t>(b) * N + i) * dim + f;
                    gx[o] = 2.f * (__ldg(x + o) * rs - acc[u]);
                }
            }
        }
    }
}

// gy[b, j0:j0+32, :] from G columns j0..j0+31 and all of x[b].
template <int GF>
__global__ void __launch_bounds__(256) grad_y_kernel(const float* __restrict__ G, const float* __restrict__ mask,
                                                     const float* __restrict__ x, const float* __restrict__ y,
                                                     float* __restrict__ gy, int N, int M, int dim) {
    __shared__ float Gs[GT][GT + 1];
    __shared__ float Xs[GT][GF + 1];
    const int b = blockIdx.y;
    const int j0 = blockIdx.x * GT;
    const int tx = threadIdx.x & 7;
    const int ty = threadIdx.x >> 3;
    const float* Gb = G + static_cast<size_t>(b) * N * M;
    const float* Mb = mask ? mask + static_cast<size_t>(b) * N * M : nullptr;
    const float* xb = x + static_cast<size_t>(b) * N * dim;
    for (int fc = 0; fc < dim; fc += GF) {
        float acc[GF / 8];
#pragma unroll
        for (int u = 0; u < GF / 8; ++u) acc[u] = 0.f;
        float cs = 0.f;
        for (int i0 = 0; i0 < N; i0 += GT) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int e = threadIdx.x + r * 256;
                const int ii = e / GT, jj = e % GT;
                float gv = 0.f;
                if (i0 + ii < N && j0 + jj < M) {
                    const size_t off = static_cast<size_t>(i0 + ii) * M + j0 + jj;
                    gv = __ldg(Gb + off);
                    if (Mb && !(__ldg(Mb + off) > 0.f)) gv = 0.f;
                }
                Gs[ii][jj] = gv;
            }
#pragma unroll
            for (int r = 0; r < GF / 8; ++r) {
                const int e = threadIdx.x + r * 256;
                const int ii = e / GF, ff = e % GF;
                Xs[ii][ff] = (i0 + ii < N && fc + ff < dim) ? __ldg(xb + static_cast<size_t>(i0 + ii) * dim + fc + ff) : 0.f;
            }
            __syncthreads();
#pragma unroll 8
            for (int ii = 0; ii < GT; ++ii) {
                const float gv = Gs[ii][ty];
                cs += gv;
#pragma unroll
                for (int u = 0; u < GF / 8; ++u) acc[u] = fmaf(gv, Xs[ii][tx + 8 * u], acc[u]);
            }
            __syncthreads();
        }
        const int j = j0 + ty;
        if (j < M) {
#pragma unroll
            for (int u = 0; u < GF / 8; ++u) {
                const int f = fc + tx + 8 * u;
                if (f < dim) {
                    const size_t o = (static_cast<size_t>(b) * M + j) * dim + f;
                    gy[o] = 2.f * (__ldg(y + o) * cs - acc[u]);
                }
            }
        }
    }
}

template <int GF>
static void grad_launch(const float* G, const float* mask, const float* x, const float* y, float* gx, float* gy, int B,
                        int N, int M, int dim, cudaStream_t stream) {
    if (gx) grad_x_kernel<GF><<<dim3((N + GT - 1) / GT, B), 256, 0, stream>>>(G, mask, x, y, gx, N, M, dim);
    if (gy) grad_y_kernel<GF><<<dim3((M + GT - 1) / GT, B), 256, 0, stream>>>(G, mask, x, y, gy, N, M, dim);
}

cudaError_t launch_grad_xy(const float* G, const float* mask, const float* x, const float* y, float* gx,
                           float* gy, int B, int N, int M, int dim, cudaStream_t stream) {
    if (dim <= 8) grad_launch<8>(G, mask, x, y, gx, gy, B, N, M, dim, stream);
    else if (dim <= 16) grad_launch<16>(G, mask, x, y, gx, gy, B, N, M, dim, stream);
    else if (dim <= 32) grad_launch<32>(G, mask, x, y, gx, gy, B, N, M, dim, stream);
    else grad_launch<64>(G, mask, x, y, gx, gy, B, N, M, dim, stream);
    return cudaGetLastError();
}

}  // namespace sdtw
