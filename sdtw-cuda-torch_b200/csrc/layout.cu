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
//   cost_wl_kernel    D in WL layout straight from x, y (register-tiled FP32):
//                     <false> clamp(||x||^2 + ||y||^2 - 2 x.y, 0)   (distances.py:6-28)
//                     <true>  sum_k (x_k - y_k)^2                     (kernels.py:27-31)
//   rm_to_wl_kernel   row-major (B,N,M) -> WL (caller-supplied cost matrices)
//   wl_to_rm_kernel   WL -> row-major, optionally multiplied by (D_wl > 0),
//                     the clamp mask of the unfused cost's chain rule
//   wl_to_rm_cm_kernel  the same, writing the table and its transpose
//   transpose_kernel  (B,R,C) -> (B,C,R) (feature-major copies of x and y)
#include <algorithm>
#include <cstdint>

#include "sdtw_kernels.h"

namespace sdtw {

constexpr int kTB = 32;   // anti-diagonals per tile


__device__ __forceinline__ size_t wl_row_base(const WavePlan& P, int b, int s, int t) {
    return ((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + t) * (32 * P.K);
}

// Cost tiles.  One CTA (256 threads) per (block of CJ = 4096 / (32K) columns,
// stripe, problem): the rectangle of cells q in [0, 32K) x j in [j0, j0+CJ),
// with x rows R0 .. R0+32K-1 and y rows j0 .. j0+CJ-1 staged in shared
// memory FC features at a time.  Each thread owns 16 cells: 4 consecutive rows
// q = 4a+i times the 4 columns j = j0 + jb + (CJ/4) c.  Per group of 4
// features it reads 4 x rows (the same for the whole warp: broadcasts) and 4
// y rows (consecutive across lanes) as float4, 8 shared loads for 64
// cell-features, so the kernel is bound by the FP32 pipe rather than by
// shared-memory bandwidth.  Rows are padded to a multiple of 4 floats whose
// quotient by 4 is odd, so the 8 lanes of a 128-bit load phase hit distinct
// banks.  The cells go through a shared-memory tile indexed by anti-diagonal
// to stores of anti-diagonal rows; cells of the table's padding are not
// written.
template <int FC>
struct CostPitch {
    static constexpr int v = ((FC + 4) / 4) % 2 ? FC + 4 : FC + 8;
};

template <int K, bool DIRECT, int FC, bool VEC>
__global__ void __launch_bounds__(256, 3) cost_wl_kernel(const SeqIn x, const SeqIn y,
                                                         float* __restrict__ Dw, WavePlan P, int dim) {
    constexpr int SR = 32 * K;
    constexpr int CJ = 4096 / SR;        // columns per tile
    constexpr int CG = CJ / 4;           // column stride of a thread's cells
    constexpr int PITCH = CostPitch<FC>::v;
    constexpr int NOFF = (SR + CJ + 3) / 4 * 4;  // norms region, rounded to 16 bytes
    extern __shared__ __align__(16) float cs[];
    pdl_trigger();
    pdl_wait();
    float* xn = cs;                      // [SR]
    float* yn = xn + SR;                 // [CJ]
    float* xs0 = cs + NOFF;                  // [SR + CJ][PITCH]: x rows then y rows
    float* xs1 = xs0 + (SR + CJ) * PITCH;    // second buffer (16-byte async copies)
    const int j0 = blockIdx.x * CJ;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int R0 = s * SR;
    const int jb = threadIdx.x % CG;  // columns j0 + jb + CG c
    const int ag = threadIdx.x / CG;  // rows 4ag .. 4ag+3

    float acc[4][4];
    unsigned long long acc2[4][4];  // DIRECT: packed (even, odd) partial sums
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            acc[i][c] = 0.f;
            acc2[i][c] = 0ull;
        }
    if (!DIRECT) {
        for (int i = threadIdx.x; i < SR + CJ; i += 256) xn[i] = 0.f;  // xn and yn are adjacent
    }
    // VEC (dim % 4 == 0, 16-byte aligned rows): feature chunks staged with
    // 16-byte cp.async into two buffers, the next chunk's copies in flight
    // while this one is computed.
    auto stage_async = [&](float* dstb, int f0) {
        const float* __restrict__ xb = x.at(b, static_cast<size_t>(P.N) * dim);
        const float* __restrict__ yb = y.at(b, static_cast<size_t>(P.M) * dim);
        for (int e = threadIdx.x; e < (SR + CJ) * (FC / 4); e += 256) {
            const int r = e / (FC / 4), f = (e % (FC / 4)) * 4;
            const bool isx = r < SR;
            const int row = isx ? R0 + r : j0 + r - SR;
            const bool in = (isx ? row < P.N : row < P.M) && f0 + f < dim;
            float* dst = dstb + r * PITCH + f;
            if (in)
                cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dst)),
                           (isx ? xb : yb) + static_cast<size_t>(row) * dim + f0 + f);
            else
                *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_commit();
    };
    const int n_chunks = (dim + FC - 1) / FC;
    if (VEC) stage_async(xs0, 0);
    for (int ci = 0; ci < n_chunks; ++ci) {
        const int f0 = ci * FC;
        float* const xs = (VEC && (ci & 1)) ? xs1 : xs0;
        float* const ys = xs + SR * PITCH;
        if (VEC) {
            if (ci + 1 < n_chunks) {
                stage_async((ci & 1) ? xs0 : xs1, f0 + FC);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
        } else {
            __syncthreads();
            const float* __restrict__ xb = x.at(b, static_cast<size_t>(P.N) * dim);
            const float* __restrict__ yb = y.at(b, static_cast<size_t>(P.M) * dim);
            for (int e = threadIdx.x; e < (SR + CJ) * FC; e += 256) {
                const int r = e / FC, f = e % FC;
                const bool isx = r < SR;
                const int row = isx ? R0 + r : j0 + r - SR;
                const bool in = (isx ? row < P.N : row < P.M) && f0 + f < dim;
                xs[r * PITCH + f] = in ? __ldg((isx ? xb : yb) + static_cast<size_t>(row) * dim + f0 + f) : 0.f;
            }
            __syncthreads();
        }
        if (!DIRECT) {
            for (int i = threadIdx.x; i < SR + CJ; i += 256) {
                const float* row = xs + i * PITCH;
                float a = 0.f;
#pragma unroll
                for (int f = 0; f < FC; ++f) a = fmaf(row[f], row[f], a);
                xn[i] += a;  // xn[SR + r] is yn[r]
            }
        }
        const float* xrow = xs + (4 * ag) * PITCH;
        const float* yrow = ys + jb * PITCH;
        if (DIRECT) {
            // Packed pairs of features (f32x2): one subtract and one FMA per two
            // cell-features; acc2 holds the even- and odd-feature partial sums.
#pragma unroll
            for (int f = 0; f < FC; f += 4) {
                ulonglong2 xv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const ulonglong2*>(xrow + i * PITCH + f);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const ulonglong2 yv = *reinterpret_cast<const ulonglong2*>(yrow + c * CG * PITCH + f);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const unsigned long long d01 = sub_f32x2(xv[i].x, yv.x);
                        const unsigned long long d23 = sub_f32x2(xv[i].y, yv.y);
                        acc2[i][c] = fma_f32x2(d01, d01, acc2[i][c]);
                        acc2[i][c] = fma_f32x2(d23, d23, acc2[i][c]);
                    }
                }
            }
        } else {
#pragma unroll
            for (int f = 0; f < FC; f += 4) {
                float4 xv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(xrow + i * PITCH + f);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 yv = *reinterpret_cast<const float4*>(yrow + c * CG * PITCH + f);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 a = xv[i];
                        float r = acc[i][c];
                        r = fmaf(a.x, yv.x, r);
                        r = fmaf(a.y, yv.y, r);
                        r = fmaf(a.z, yv.z, r);
                        r = fmaf(a.w, yv.w, r);
                        acc[i][c] = r;
                    }
                }
            }
        }
        // The next iteration's copies overwrite the buffer read above.
        if (VEC) __syncthreads();
    }
    __syncthreads();
    // Stage by local anti-diagonal tl = q + (j - j0) in [0, SR + CJ - 1), row
    // pitch SR + 1 (aliases the staging buffers, not the norms), then store.
    float* stg = xs0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = 4 * ag + i;
        const int p = (q % K) * 32 + q / K;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int jl = jb + CG * c;
            float v;
            if (DIRECT) v = lo_f32x2(acc2[i][c]) + hi_f32x2(acc2[i][c]);
            else v = fmaxf((xn[q] + yn[jl]) - 2.f * acc[i][c], 0.f);
            stg[(q + jl) * (SR + 1) + p] = v;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < (SR + CJ - 1) * SR; e += 256) {
        const int tl = e / SR, p = e % SR;
        const int q = (p % 32) * K + p / 32;
        const int jl = tl - q;
        const int j = j0 + jl;
        if (jl >= 0 && jl < CJ && j < P.M && R0 + q < P.N)
            Dw[wl_row_base(P, b, s, j0 + tl) + p] = stg[tl * (SR + 1) + p];
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

// Both row-major A (B,N,lda) and AT (B,M,ldt) from the WL table, by rectangles
// of 32K rows x CB = 4096 / (32K) columns: the WL rows t in [j0, j0 + CB +
// 32K - 1) of the stripe hold the rectangle, each row read once by one warp
// (the neighbouring rectangles read the overlap, mostly from L2).  Both stores
// are then aligned runs: 128-byte runs of A's rows and 32K-float runs of AT's
// rows.  The padding columns (M .. lda of A, N .. ldt of AT) are written as
// zeros.  The tile pitch CB + 2 keeps the skewed writes (cell (q, t - q)) on
// distinct banks for K = 1.
template <int K>
__global__ void __launch_bounds__(256) wl_to_rm_cm_kernel(const float* __restrict__ Aw, const float* __restrict__ maskw,
                                                          float* __restrict__ A, int lda, float* __restrict__ AT,
                                                          int ldt, WavePlan P) {
    constexpr int SR = 32 * K, CB = 4096 / SR, PITCH = CB + 2;
    __shared__ float tile[SR * PITCH];
    const int j0 = blockIdx.x * CB;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int R0 = s * SR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t_end = min(j0 + CB, P.M) + SR - 1;
#pragma unroll 4
    for (int t = j0 + warp; t < t_end; t += 8) {
        const size_t base = wl_row_base(P, b, s, t);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float v = __ldg(Aw + base + k * 32 + lane);
            if (maskw && !(__ldg(maskw + base + k * 32 + lane) > 0.f)) v = 0.f;
            const int q = lane * K + k;
            const int c = t - q - j0;
            if (c >= 0 && c < CB) tile[q * PITCH + c] = v;
        }
    }
    __syncthreads();
    if (A) {
        for (int q = warp; q < SR; q += 8) {
            const int row = R0 + q;
            if (row >= P.N) break;
            float* dst = A + (static_cast<size_t>(b) * P.N + row) * lda;
#pragma unroll
            for (int c = lane; c < CB; c += 32) {
                const int col = j0 + c;
                if (col < P.M) dst[col] = tile[q * PITCH + c];
                else if (col < lda) dst[col] = 0.f;
            }
        }
    }
    if (AT) {
        for (int c = warp; c < CB; c += 8) {
            const int col = j0 + c;
            if (col >= P.M) break;
            float* dst = AT + (static_cast<size_t>(b) * P.M + col) * ldt;
#pragma unroll
            for (int q = lane; q < SR; q += 32) {
                const int row = R0 + q;
                if (row < P.N) dst[row] = tile[q * PITCH + c];
                else if (row < ldt) dst[row] = 0.f;
            }
        }
    }
}

// 32 x 32 tiles through shared memory; grid (ceil(C/32), ceil(ldo/32), B).
// Output columns R .. ldo are written as zeros.
__global__ void __launch_bounds__(256) transpose_kernel(const SeqIn in_s, float* __restrict__ out, int R, int C,
                                                        int ldo) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const float* __restrict__ in = in_s.at(blockIdx.z, static_cast<size_t>(R) * C);
    const size_t out_off = static_cast<size_t>(blockIdx.z) * C * ldo;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = warp; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + lane;
        if (r < R && c < C) tile[i][lane] = __ldg(in + static_cast<size_t>(r) * C + c);
    }
    __syncthreads();
    for (int i = warp; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + lane;
        if (r < ldo && c < C) out[out_off + static_cast<size_t>(c) * ldo + r] = r < R ? tile[lane][i] : 0.f;
    }
}

// 32 sequence positions x up to kTransTiles * 32 features per block through
// shared memory, every tile's loads issued before the first store; grid
// (ceil(max(R0, R1)/32), ceil(C/(32 kTransTiles)), 2B): z < B transposes in0
// (rows R0), the rest in1 (rows R1); either may be null.  Output rows are 36
// floats: 32 positions and 4 zeros.  (One 32 x 32 tile per block measured
// 12.8 us for C2's x and y, 1.4 TB/s.)
constexpr int kTransTiles = 4;
__global__ void __launch_bounds__(256) transpose_chunked_kernel(const SeqIn in0, float* __restrict__ out0, int R0,
                                                                const SeqIn in1, float* __restrict__ out1, int R1,
                                                                int B, int C) {
    __shared__ float tile[kTransTiles][32][33];
    pdl_trigger();
    pdl_wait();
    const bool second = static_cast<int>(blockIdx.z) >= B;
    float* __restrict__ out = second ? out1 : out0;
    const int R = second ? R1 : R0;
    const int b = second ? blockIdx.z - B : blockIdx.z;
    const int c = blockIdx.x, f0 = blockIdx.y * 32 * kTransTiles;
    const int n_chunks = (R + 31) / 32;
    if ((second ? in1.null() : in0.null()) || c >= n_chunks) return;  // block-uniform
    const size_t rc = static_cast<size_t>(R) * C;
    const float* __restrict__ in = second ? in1.at(b, rc) : in0.at(b, rc);
    const size_t out_off = (static_cast<size_t>(b) * n_chunks + c) * C * 36;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = min(kTransTiles, (C - f0 + 31) / 32);  // block-uniform
#pragma unroll
    for (int t = 0; t < kTransTiles; ++t) {
        if (t < tiles) {
#pragma unroll
            for (int i = warp; i < 32; i += 8) {
                const int r = 32 * c + i, f = f0 + 32 * t + lane;
                tile[t][i][lane] = (r < R && f < C) ? __ldg(in + static_cast<size_t>(r) * C + f) : 0.f;
            }
        }
    }
    __syncthreads();
    for (int t = 0; t < tiles; ++t) {
        for (int i = warp; i < 32; i += 8) {
            const int f = f0 + 32 * t + i;
            if (f < C) {
                float* row = out + out_off + static_cast<size_t>(f) * 36;
                row[lane] = tile[t][lane][i];
                if (lane < 4) row[32 + lane] = 0.f;
            }
        }
    }
}

// g += a + b, four floats per thread (n4 = n / 4 units of 16 bytes) and the
// tail one by one: normalize folds its triple's other gradients into x's / y's.
__global__ void __launch_bounds__(256) add2_kernel(float* __restrict__ g, const float* __restrict__ a,
                                                   const float* __restrict__ b, size_t n, int vec) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    size_t done = 0;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t u = i; u < n4; u += stride) {
            float4 v = reinterpret_cast<float4*>(g)[u];
            const float4 p = __ldg(reinterpret_cast<const float4*>(a) + u);
            const float4 q = __ldg(reinterpret_cast<const float4*>(b) + u);
            v.x += p.x + q.x;
            v.y += p.y + q.y;
            v.z += p.z + q.z;
            v.w += p.w + q.w;
            reinterpret_cast<float4*>(g)[u] = v;
        }
        done = n4 * 4;
    }
    for (size_t k = done + i; k < n; k += stride) g[k] += __ldg(a + k) + __ldg(b + k);
}

static dim3 wl_grid(const WavePlan& P) {
    return dim3((P.n_diag + kTB - 1) / kTB, P.n_stripes, P.B);
}

template <int K, int FC>
static size_t cost_wl_smem() {
    constexpr int SR = 32 * K, CJ = 4096 / SR;
    constexpr int NOFF = (SR + CJ + 3) / 4 * 4;
    const size_t in = 2 * static_cast<size_t>(SR + CJ) * CostPitch<FC>::v;  // two buffers
    const size_t stage = static_cast<size_t>(SR + CJ - 1) * (SR + 1);
    return (NOFF + (in > stage ? in : stage)) * sizeof(float);
}

template <int K, int FC>
static cudaError_t cost_wl_launch(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, bool direct,
                                  cudaStream_t stream) {
    constexpr int CJ = 4096 / (32 * K);
    const dim3 g((P.M + CJ - 1) / CJ, P.n_stripes, P.B);
    const size_t smem = cost_wl_smem<K, FC>();
    const bool vec = (dim % 4 == 0) && x.aligned16() && y.aligned16();
    auto fn = direct ? (vec ? cost_wl_kernel<K, true, FC, true> : cost_wl_kernel<K, true, FC, false>)
                     : (vec ? cost_wl_kernel<K, false, FC, true> : cost_wl_kernel<K, false, FC, false>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_pdl(false, fn, g, dim3(256), smem, stream, x, y, Dw, P, dim);  // first of its call
}

template <int K>
static cudaError_t cost_wl_by_dim(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, bool direct,
                                  cudaStream_t stream) {
    // Feature chunk sized to the feature count: no padded work for small dims.
    if (dim <= 4) return cost_wl_launch<K, 4>(x, y, Dw, P, dim, direct, stream);
    if (dim <= 8) return cost_wl_launch<K, 8>(x, y, Dw, P, dim, direct, stream);
    if (dim <= 16) return cost_wl_launch<K, 16>(x, y, Dw, P, dim, direct, stream);
    return cost_wl_launch<K, 32>(x, y, Dw, P, dim, direct, stream);
}

cudaError_t launch_cost_wl(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, bool direct,
                           cudaStream_t stream) {
    switch (P.K) {
        case 1: return cost_wl_by_dim<1>(x, y, Dw, P, dim, direct, stream);
        case 2: return cost_wl_by_dim<2>(x, y, Dw, P, dim, direct, stream);
        case 4: return cost_wl_by_dim<4>(x, y, Dw, P, dim, direct, stream);
        default: return cudaErrorInvalidValue;
    }
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

cudaError_t launch_wl_to_rm_cm(const float* Aw, const float* maskw, float* A, int lda, float* AT, int ldt,
                               const WavePlan& P, cudaStream_t stream) {
    if (lda < P.M || ldt < P.N) return cudaErrorInvalidValue;
    const int cb = 4096 / (32 * P.K);
    const dim3 g((P.M + cb - 1) / cb, P.n_stripes, P.B);
    switch (P.K) {
        case 1: wl_to_rm_cm_kernel<1><<<g, 256, 0, stream>>>(Aw, maskw, A, lda, AT, ldt, P); break;
        case 2: wl_to_rm_cm_kernel<2><<<g, 256, 0, stream>>>(Aw, maskw, A, lda, AT, ldt, P); break;
        case 4: wl_to_rm_cm_kernel<4><<<g, 256, 0, stream>>>(Aw, maskw, A, lda, AT, ldt, P); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_transpose_chunked(const SeqIn& in0, float* out0, int R0, const SeqIn& in1, float* out1, int R1,
                                     int B, int C, cudaStream_t stream) {
    if (B <= 0 || C <= 0 || (in0.null() && in1.null())) return cudaSuccess;
    const int rows = std::max(in0.null() ? 0 : R0, in1.null() ? 0 : R1);
    const dim3 g((rows + 31) / 32, (C + 32 * kTransTiles - 1) / (32 * kTransTiles), 2 * B);
    return launch_pdl(false, transpose_chunked_kernel, g, dim3(256), 0, stream, in0, out0, R0, in1, out1, R1, B, C);
}

cudaError_t launch_add2(float* g, const float* a, const float* b, size_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int vec = ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) &
                     15u) == 0;
    const size_t units = vec ? n / 4 + 1 : n;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((units + 255) / 256, 148 * 16));
    add2_kernel<<<blocks, 256, 0, stream>>>(g, a, b, n, vec);
    return cudaGetLastError();
}

cudaError_t launch_transpose_brc(const SeqIn& in, float* out, int B, int R, int C, int ldo, cudaStream_t stream) {
    if (B <= 0 || R <= 0 || C <= 0) return cudaSuccess;
    const dim3 g((C + 31) / 32, (ldo + 31) / 32, B);
    transpose_kernel<<<g, 256, 0, stream>>>(in, out, R, C, ldo);
    return cudaGetLastError();
}

}  // namespace sdtw
