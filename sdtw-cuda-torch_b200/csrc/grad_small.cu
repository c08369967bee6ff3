// grad_small.cu -- dL/dx and dL/dy of the squared-Euclidean chain rule for
// few features (dim <= 16), on the FP32 pipes, reading E straight from the
// wavefront layout (one row per lane).
//
//   grad_x[b,i,:] = 2 (x_i * sum_j G_ij - sum_j G_ij y_j)
//   grad_y[b,j,:] = 2 (y_j * sum_i G_ij - sum_i G_ij x_i)
//
// with G = E (fused cost, autograd_xy.py:41-49), or E where the unfused
// cost is positive (the clamp mask of distances.py:20-28).  With few features
// the contraction is a handful of multiply-adds per cell and the kernel is
// bound by the one read of E; the tensor-core kernels (tcgemm.cu) need tiles of
// 16+ features to pay their operand preparation.
//
// One warp per stripe, up to 8 stripes (a split) per CTA.  For every block of
// 32 columns the warp stages the 32 x 32 cells of its stripe -- anti-diagonal
// rows t in [j0, j0 + 63), cell (l, j) at row j - j0 + l, lane l -- in shared
// memory (pitch 33 floats) and makes two passes over them:
//   row pass     lane l: row l over the 32 columns, y rows broadcast; the row
//                sums stay in registers across all blocks (grad_x at the end)
//   column pass  lane c: column c over the 32 rows, x rows broadcast; the
//                split's warps' column sums are added in warp order and stored
//                to the split's slice of the partial buffer (no atomics)
// grad_small_finalize_kernel sums the splits' column partials into grad_y.
#include <algorithm>
#include <cstdint>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int kSmallTile = 63;   // anti-diagonal rows of a (stripe, 32-column block)
constexpr int kSmallPitch = 33;  // floats per staged row: the column pass hits 32 banks
constexpr int kSmallWarps = 8;   // stripes per CTA

template <int DP>
struct SmallSmem {
    static constexpr int E = (kSmallTile * kSmallPitch + 3) / 4 * 4;  // per warp (16-byte multiple)
    static constexpr int X = 32 * DP;                   // per warp: its stripe's x rows
    static constexpr int RED = 32 * (DP + 1);           // per warp: column sums of a block
    static constexpr int Y = 32 * DP;                   // the block's y rows
    static constexpr int floats(int warps) { return warps * (E + X + RED) + Y; }
};

template <int DP, bool MASKED>
__global__ void __launch_bounds__(32 * kSmallWarps) grad_small_kernel(const float* __restrict__ Ew,
                                                                      const float* __restrict__ Mw,
                                                                      const float* __restrict__ x,
                                                                      const float* __restrict__ y,
                                                                      float* __restrict__ gx,
                                                                      float* __restrict__ part, WavePlan P, int dim,
                                                                      int n_split, size_t xbs) {
    extern __shared__ __align__(16) float sm[];
    pdl_trigger();
    pdl_wait();
    const int warps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* Et = sm + warp * SmallSmem<DP>::E;
    float* Xt = sm + warps * SmallSmem<DP>::E + warp * SmallSmem<DP>::X;
    float* red = sm + warps * (SmallSmem<DP>::E + SmallSmem<DP>::X);
    float* Yt = red + warps * SmallSmem<DP>::RED;
    const int N = P.N, M = P.M;
    const int b = blockIdx.y, split = blockIdx.x;  // problem, split of 8 stripes
    const int s = split * warps + warp;
    const bool live = s < P.n_stripes;  // warp-uniform
    const int R0 = s * 32;
    const bool need_x = gx != nullptr, need_y = part != nullptr;
    const size_t base = (static_cast<size_t>(b) * P.n_stripes + (live ? s : 0)) * P.n_diag * 32 + lane;

    // The stripe's x rows (zeros past N and past dim).
#pragma unroll
    for (int d = 0; d < DP; ++d)
        Xt[lane * DP + d] =
            (live && R0 + lane < N && d < dim) ? __ldg(x + b * xbs + static_cast<size_t>(R0 + lane) * dim + d) : 0.f;
    float racc[DP + 1];  // row R0 + lane: sum_j G y_j (DP), sum_j G
#pragma unroll
    for (int d = 0; d <= DP; ++d) racc[d] = 0.f;

    for (int j0 = 0; j0 < M; j0 += 32) {
        __syncthreads();  // Yt and red of the previous block are consumed
        for (int i = threadIdx.x; i < 32 * DP; i += blockDim.x) {
            const int jj = i / DP, d = i % DP;
            Yt[i] = (j0 + jj < M && d < dim) ? __ldg(y + (static_cast<size_t>(b) * M + j0 + jj) * dim + d) : 0.f;
        }
        if (live) {
            // All 63 loads in flight at once, then the stores (one round trip
            // of latency per block).
            float v[kSmallTile];
            const int rows = min(kSmallTile, P.n_diag - j0);
#pragma unroll
            for (int r = 0; r < kSmallTile; ++r) {
                v[r] = 0.f;
                if (r < rows) {
                    v[r] = __ldg(Ew + base + static_cast<size_t>(j0 + r) * 32);
                    if (MASKED && !(__ldg(Mw + base + static_cast<size_t>(j0 + r) * 32) > 0.f)) v[r] = 0.f;
                }
            }
#pragma unroll
            for (int r = 0; r < kSmallTile; ++r) Et[r * kSmallPitch + lane] = v[r];
        }
        __syncthreads();
        float cacc[DP + 1];
#pragma unroll
        for (int d = 0; d <= DP; ++d) cacc[d] = 0.f;
        if (live) {
            if (need_x) {
#pragma unroll 4
                for (int jj = 0; jj < 32; ++jj) {
                    const float g = Et[(jj + lane) * kSmallPitch + lane];
                    const float4* y4 = reinterpret_cast<const float4*>(Yt + jj * DP);
                    racc[DP] += g;
#pragma unroll
                    for (int q = 0; q < DP / 4; ++q) {
                        const float4 v = y4[q];
                        racc[4 * q + 0] = fmaf(g, v.x, racc[4 * q + 0]);
                        racc[4 * q + 1] = fmaf(g, v.y, racc[4 * q + 1]);
                        racc[4 * q + 2] = fmaf(g, v.z, racc[4 * q + 2]);
                        racc[4 * q + 3] = fmaf(g, v.w, racc[4 * q + 3]);
                    }
                }
            }
            if (need_y) {
#pragma unroll 4
                for (int l = 0; l < 32; ++l) {
                    const float g = Et[(lane + l) * kSmallPitch + l];
                    const float4* x4 = reinterpret_cast<const float4*>(Xt + l * DP);
                    cacc[DP] += g;
#pragma unroll
                    for (int q = 0; q < DP / 4; ++q) {
                        const float4 v = x4[q];
                        cacc[4 * q + 0] = fmaf(g, v.x, cacc[4 * q + 0]);
                        cacc[4 * q + 1] = fmaf(g, v.y, cacc[4 * q + 1]);
                        cacc[4 * q + 2] = fmaf(g, v.z, cacc[4 * q + 2]);
                        cacc[4 * q + 3] = fmaf(g, v.w, cacc[4 * q + 3]);
                    }
                }
            }
        }
        if (need_y) {
#pragma unroll
            for (int d = 0; d <= DP; ++d) red[(warp * 32 + lane) * (DP + 1) + d] = cacc[d];
            __syncthreads();
            float* pp = part + ((static_cast<size_t>(b) * n_split + split) * M + j0) * (DP + 1);
            for (int i = threadIdx.x; i < 32 * (DP + 1); i += blockDim.x) {
                if (j0 + i / (DP + 1) >= M) continue;
                float v = 0.f;
                for (int w = 0; w < warps; ++w) v += red[w * SmallSmem<DP>::RED + i];
                pp[i] = v;
            }
        }
    }
    if (need_x && live && R0 + lane < N) {
        const size_t o = (static_cast<size_t>(b) * N + R0 + lane) * dim;
#pragma unroll
        for (int d = 0; d < DP; ++d)
            if (d < dim) gx[o + d] = 2.f * (Xt[lane * DP + d] * racc[DP] - racc[d]);
    }
}

// grad_y from the splits' column partials, summed in split order.
template <int DP>
__global__ void __launch_bounds__(256) grad_small_finalize_kernel(const float* __restrict__ part,
                                                                  const float* __restrict__ y,
                                                                  float* __restrict__ gy, int B, int M, int dim,
                                                                  int n_split) {
    pdl_trigger();
    pdl_wait();
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(B) * M * dim) return;
    const int d = static_cast<int>(i % dim);
    const size_t bj = i / dim;
    const int j = static_cast<int>(bj % M), b = static_cast<int>(bj / M);
    float s = 0.f, t = 0.f;
    for (int k = 0; k < n_split; ++k) {
        const float* pp = part + ((static_cast<size_t>(b) * n_split + k) * M + j) * (DP + 1);
        s += __ldg(pp + DP);
        t += __ldg(pp + d);
    }
    gy[i] = 2.f * (__ldg(y + i) * s - t);
}

static int small_dp(int dim) { return dim <= 4 ? 4 : dim <= 8 ? 8 : 16; }

static int small_warps(const WavePlan& P) { return std::min(kSmallWarps, P.n_stripes); }
int grad_small_splits(const WavePlan& P) { return (P.n_stripes + kSmallWarps - 1) / kSmallWarps; }

bool grad_small_supported(const WavePlan& P, int dim) { return P.K == 1 && dim >= 1 && dim <= 16; }

size_t grad_small_part_bytes(const WavePlan& P, int dim) {
    return static_cast<size_t>(P.B) * grad_small_splits(P) * P.M * (small_dp(dim) + 1) * sizeof(float);
}

template <int DP>
static cudaError_t go_small(const float* Ew, const float* Mw, const float* x, const float* y, float* gx, float* gy,
                            float* part, const WavePlan& P, int dim, cudaStream_t st, size_t xbs) {
    const int n_split = grad_small_splits(P);
    const int warps = small_warps(P);
    const size_t smem = static_cast<size_t>(SmallSmem<DP>::floats(warps)) * sizeof(float);
    const void* fn = Mw ? (const void*)grad_small_kernel<DP, true> : (const void*)grad_small_kernel<DP, false>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const dim3 grid(n_split, P.B);
    float* pp = gy ? part : nullptr;
    if (Mw)
        e = launch_pdl(false, grad_small_kernel<DP, true>, grid, dim3(32 * warps), smem, st, Ew, Mw, x, y, gx, pp, P, dim,
                       n_split, xbs);
    else
        e = launch_pdl(false, grad_small_kernel<DP, false>, grid, dim3(32 * warps), smem, st, Ew, Mw, x, y, gx, pp, P, dim,
                       n_split, xbs);
    if (e != cudaSuccess || !gy) return e;
    const size_t n = static_cast<size_t>(P.B) * P.M * dim;
    return launch_pdl(false, grad_small_finalize_kernel<DP>, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st,
                      part, y, gy, P.B, P.M, dim, n_split);
}

cudaError_t launch_grad_small(const float* Ew, const float* Mw, const float* x, const float* y, float* gx, float* gy,
                              float* part, const WavePlan& P, int dim, cudaStream_t st, size_t xbs) {
    if (!grad_small_supported(P, dim)) return cudaErrorInvalidValue;
    if (!gx && !gy) return cudaSuccess;
    switch (small_dp(dim)) {
        case 4: return go_small<4>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
        case 8: return go_small<8>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
        default: return go_small<16>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
    }
}

}  // namespace sdtw
