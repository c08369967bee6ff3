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
// One warp per stripe, up to 8 stripes (a split) per CTA, and the columns cut
// into ranges (column splits) so that the launch has CTAs for every SM.  For
// every block of 32 columns the warp loads the 32 x 32 cells of its stripe --
// anti-diagonal rows t in [j0, j0 + 63), cell (l, j) at row j - j0 + l, lane l
// -- stores them in shared memory by (column, row) with an XOR swizzle, and
// makes two passes over them:
//   row pass     lane l: row l over the 32 columns, y rows broadcast; the row
//                sums stay in registers across the range's blocks (grad_x at
//                the end, or a partial per column split)
//   column pass  lane c: column c over the 32 rows, x rows broadcast; the
//                split's warps' column sums are added in warp order and stored
//                to the split's slice of the partial buffer (no atomics)
// grad_small_finalize_kernel sums the splits' column partials into grad_y,
// grad_small_finalize_x_kernel the column splits' row partials into grad_x.
#include <algorithm>
#include <cstdint>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int kSmallTile = 63;   // anti-diagonal rows of a (stripe, 32-column block)
constexpr int kSmallWarps = 8;   // stripes per CTA
// CTAs a launch aims at (column splits multiply the stripe splits up to it):
// measured at C3 (256 stripe-split CTAs), 2 / 3 / 4 / 6 column splits took
// 0.663 / 0.717 / 0.607 / 0.626 ms.
constexpr int kSmallCtas = 1024;
constexpr int kSmallMinBlocks = 8;   // 32-column blocks per column split, at least

template <int DP>
struct SmallSmem {
    static constexpr int E = (32 * 33 + 3) / 4 * 4;  // per warp: the block's cells
    static constexpr int X = 32 * DP;          // per warp: its stripe's x rows
    static constexpr int RED = 32 * (DP + 1);  // per warp: column sums of a block
    static constexpr int Y = 32 * DP;          // the block's y rows
    static constexpr int floats(int warps) { return warps * (E + X + RED) + Y; }
};
// Cell (row l, column c) of a warp's block sits at c * 33 + row_slot(l), where
// row_slot (0, 2, .., 30, 1, 3, .., 31) permutes the rows: the row pass (lanes
// = rows, one column: banks c + row_slot(l)) and the column pass (lanes =
// columns, one row: banks c + row_slot(l)) read 32 distinct banks, and the
// anti-diagonal stores (lane l, column r - l: banks r + row_slot(l) - l) as
// well but for one pair of lanes in one store of the 63.  Every address is a
// per-lane base plus a constant offset (33 r), so the stores need no address
// arithmetic.
__device__ __forceinline__ int row_slot(int l) { return ((l & 15) << 1) | (l >> 4); }

template <int DP, bool MASKED>
__global__ void __launch_bounds__(32 * kSmallWarps) grad_small_kernel(const float* __restrict__ Ew,
                                                                      const float* __restrict__ Mw,
                                                                      const SeqIn x_s, const SeqIn y_s,
                                                                      const SeqOut gx_s,
                                                                      float* __restrict__ part,
                                                                      float* __restrict__ part_x, WavePlan P, int dim,
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
    const int cs = blockIdx.z, n_cs = gridDim.z;   // column split: blocks [blk0, blk1)
    const int nblk = (M + 31) / 32;
    const int blk0 = static_cast<int>(static_cast<long long>(nblk) * cs / n_cs);
    const int blk1 = static_cast<int>(static_cast<long long>(nblk) * (cs + 1) / n_cs);
    const int s = split * warps + warp;
    const bool live = s < P.n_stripes;  // warp-uniform
    const int R0 = s * 32;
    const bool need_x = !gx_s.null(), need_y = part != nullptr;
    const float* __restrict__ x = x_s.at(b, xbs);
    const size_t base = (static_cast<size_t>(b) * P.n_stripes + (live ? s : 0)) * P.n_diag * 32 + lane;

    // The stripe's x rows (zeros past N and past dim).
#pragma unroll
    for (int d = 0; d < DP; ++d)
        Xt[lane * DP + d] =
            (live && R0 + lane < N && d < dim) ? __ldg(x + static_cast<size_t>(R0 + lane) * dim + d) : 0.f;
    const int rs = row_slot(lane);
    float racc[DP + 1];  // row R0 + lane: sum_j G y_j (DP), sum_j G
#pragma unroll
    for (int d = 0; d <= DP; ++d) racc[d] = 0.f;

    for (int j0 = blk0 * 32; j0 < blk1 * 32; j0 += 32) {
        __syncthreads();  // Yt and red of the previous block are consumed
        const float* __restrict__ y = y_s.at(b, static_cast<size_t>(M) * dim);
        for (int i = threadIdx.x; i < 32 * DP; i += blockDim.x) {
            const int jj = i / DP, d = i % DP;
            Yt[i] = (j0 + jj < M && d < dim) ? __ldg(y + static_cast<size_t>(j0 + jj) * dim + d) : 0.f;
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
            const int sbase = row_slot(lane) - 33 * lane;  // cell (row lane, column r - lane) at sbase + 33 r
#pragma unroll
            for (int r = 0; r < kSmallTile; ++r)
                if (static_cast<unsigned>(r - lane) < 32u) Et[sbase + 33 * r] = v[r];
        }
        __syncthreads();
        float cacc[DP + 1];
#pragma unroll
        for (int d = 0; d <= DP; ++d) cacc[d] = 0.f;
        if (live) {
            if (need_x) {
#pragma unroll 4
                for (int jj = 0; jj < 32; ++jj) {
                    const float g = Et[jj * 33 + rs];  // cell (row lane, column jj)
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
                    const float g = Et[lane * 33 + row_slot(l)];  // cell (row l, column lane)
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
        if (n_cs == 1) {
            float* gx = gx_s.at(b, static_cast<size_t>(N) * dim) + static_cast<size_t>(R0 + lane) * dim;
#pragma unroll
            for (int d = 0; d < DP; ++d)
                if (d < dim) gx[d] = 2.f * (Xt[lane * DP + d] * racc[DP] - racc[d]);
        } else {
            // This column split's row sums; grad_small_finalize_x_kernel adds them up.
            float* px = part_x + ((static_cast<size_t>(b) * n_cs + cs) * N + R0 + lane) * (DP + 1);
#pragma unroll
            for (int d = 0; d <= DP; ++d) px[d] = racc[d];
        }
    }
}

// grad_x from the column splits' row partials, summed in split order.
template <int DP>
__global__ void __launch_bounds__(256) grad_small_finalize_x_kernel(const float* __restrict__ part_x,
                                                                    const SeqIn x, const SeqOut gx, int B, int N,
                                                                    int dim, int n_cs, size_t xbs) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(B) * N * dim) return;
    const int d = static_cast<int>(i % dim);
    const size_t bi = i / dim;
    const int r = static_cast<int>(bi % N), b = static_cast<int>(bi / N);
    float s = 0.f, t = 0.f;
    for (int k = 0; k < n_cs; ++k) {
        const float* px = part_x + ((static_cast<size_t>(b) * n_cs + k) * N + r) * (DP + 1);
        s += __ldg(px + DP);
        t += __ldg(px + d);
    }
    const size_t o = static_cast<size_t>(r) * dim + d;
    gx.at(b, static_cast<size_t>(N) * dim)[o] = 2.f * (__ldg(x.at(b, xbs) + o) * s - t);
}

// grad_y from the splits' column partials, summed in split order.
template <int DP>
__global__ void __launch_bounds__(256) grad_small_finalize_kernel(const float* __restrict__ part,
                                                                  const SeqIn y, const SeqOut gy, int B, int M,
                                                                  int dim, int n_split) {
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
    const size_t o = static_cast<size_t>(j) * dim + d, stride = static_cast<size_t>(M) * dim;
    gy.at(b, stride)[o] = 2.f * (__ldg(y.at(b, stride) + o) * s - t);
}

static int small_dp(int dim) { return dim <= 4 ? 4 : dim <= 8 ? 8 : 16; }

static int small_warps(const WavePlan& P) { return std::min(kSmallWarps, P.n_stripes); }
int grad_small_splits(const WavePlan& P) { return (P.n_stripes + kSmallWarps - 1) / kSmallWarps; }

bool grad_small_supported(const WavePlan& P, int dim) { return P.K == 1 && dim >= 1 && dim <= 16; }

// Column splits: about kSmallCtas CTAs, with at least kSmallMinBlocks blocks
// of 32 columns each (C3, 16 x 4096^2 x 8: 4 splits, 1024 CTAs).
static int small_colsplits(const WavePlan& P) {
    const int nblk = (P.M + 31) / 32;
    const int ctas = grad_small_splits(P) * P.B;
    const int want = (kSmallCtas + ctas - 1) / ctas;
    return std::max(1, std::min(want, nblk / kSmallMinBlocks));
}

static size_t part_y_floats(const WavePlan& P, int dim) {
    return static_cast<size_t>(P.B) * grad_small_splits(P) * P.M * (small_dp(dim) + 1);
}

// The splits' column partials of grad_y, then (more than one column split)
// the column splits' row partials of grad_x.
size_t grad_small_part_bytes(const WavePlan& P, int dim) {
    const int n_cs = small_colsplits(P);
    const size_t px = n_cs > 1 ? static_cast<size_t>(P.B) * n_cs * P.N * (small_dp(dim) + 1) : 0;
    return (part_y_floats(P, dim) + px) * sizeof(float);
}

template <int DP>
static cudaError_t go_small(const float* Ew, const float* Mw, const SeqIn& x, const SeqIn& y, const SeqOut& gx,
                            const SeqOut& gy, float* part, const WavePlan& P, int dim, cudaStream_t st, size_t xbs) {
    const int n_split = grad_small_splits(P);
    const int warps = small_warps(P);
    const size_t smem = static_cast<size_t>(SmallSmem<DP>::floats(warps)) * sizeof(float);
    const void* fn = Mw ? (const void*)grad_small_kernel<DP, true> : (const void*)grad_small_kernel<DP, false>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int n_cs = small_colsplits(P);
    const dim3 grid(n_split, P.B, n_cs);
    float* pp = gy.null() ? nullptr : part;
    float* px = part + part_y_floats(P, dim);
    if (Mw)
        e = launch_pdl(false, grad_small_kernel<DP, true>, grid, dim3(32 * warps), smem, st, Ew, Mw, x, y, gx, pp, px, P,
                       dim, n_split, xbs);
    else
        e = launch_pdl(false, grad_small_kernel<DP, false>, grid, dim3(32 * warps), smem, st, Ew, Mw, x, y, gx, pp, px, P,
                       dim, n_split, xbs);
    if (e != cudaSuccess) return e;
    if (!gx.null() && n_cs > 1) {
        const size_t nx = static_cast<size_t>(P.B) * P.N * dim;
        grad_small_finalize_x_kernel<DP><<<static_cast<unsigned>((nx + 255) / 256), 256, 0, st>>>(px, x, gx, P.B, P.N,
                                                                                                 dim, n_cs, xbs);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (gy.null()) return cudaSuccess;
    const size_t n = static_cast<size_t>(P.B) * P.M * dim;
    return launch_pdl(false, grad_small_finalize_kernel<DP>, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st,
                      part, y, gy, P.B, P.M, dim, n_split);
}

cudaError_t launch_grad_small(const float* Ew, const float* Mw, const SeqIn& x, const SeqIn& y, const SeqOut& gx,
                              const SeqOut& gy, float* part, const WavePlan& P, int dim, cudaStream_t st, size_t xbs) {
    if (!grad_small_supported(P, dim)) return cudaErrorInvalidValue;
    if (gx.null() && gy.null()) return cudaSuccess;
    switch (small_dp(dim)) {
        case 4: return go_small<4>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
        case 8: return go_small<8>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
        default: return go_small<16>(Ew, Mw, x, y, gx, gy, part, P, dim, st, xbs);
    }
}

}  // namespace sdtw
