// wavefront.cu -- Soft-DTW forward (score table) and reverse (E table)
// anti-diagonal wavefronts for sm_100a.
//
// Semantics follow the reference recurrences:
//   forward   softdtw_cuda/cuda/kernels.py:126-187 and launcher.py:307-324
//             R[i,j] = D[i-1,j-1] + softmin_gamma(R[i-1,j-1], R[i-1,j], R[i,j-1]),
//             R[0,0] = 0, other borders +inf, band-pruned cells +inf.
//   backward  softdtw_cuda/cuda/kernels.py:216-307 and launcher.py:327-353
//             E[i,j] = sum over successors c of E[c] * exp((R[c] - D[c] - R[i,j]) / gamma),
//             E[N,M] = 1 (here: grad_out[b], which autograd.py:46-47 multiplies in).
//
// Formulation (B200 design, not a translation):
//   * scores T = -R * log2(e) / gamma in base 2, so one softmin is
//     T = m + (lg2(sum_k ex2(T_k - m)) - D * log2(e)/gamma) with m = max_k T_k:
//     three MUFU ex2 and one MUFU lg2 per cell, no division.
//   * the backward weight exp((R[c] - D[c] - R[p]) / gamma) equals the softmax
//     weight of predecessor p among c's three predecessors, so the reverse pass
//     recomputes it from the stored scores of c's predecessors, normalised to
//     sum to one.  It needs no cost values and no log-space E table.
//   * one warp per stripe of 32*K rows, three live anti-diagonals in registers,
//     neighbour rows exchanged with one warp shuffle per step, stripe-to-stripe
//     rows handed over through tagged u64 ring slots in the consumer's shared
//     memory (DSMEM stores across the CTAs of a cluster), bounded waits only.
#include "sdtw_device.cuh"
#include "sdtw_kernels.h"
#include "sdtw_plan.h"

namespace sdtw {

constexpr int kRing = 128;  // ring slots per warp (power of two)

__device__ __forceinline__ uint32_t wrap_tag(uint32_t seq, int band) {
    return (seq << 12) | (static_cast<uint32_t>(band) & 0xfffu);
}

// ============================================================== forward
template <int K>
__global__ void __launch_bounds__(512) fwd_kernel(const FwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    constexpr int SR = 32 * K;
    const int N = P.N, M = P.M;

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);                // [wpc][kRing]
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * kRing);  // [wpc]
    for (int i = threadIdx.x; i < wpc * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    cluster_sync_all();

    const uint32_t my_ring = smem_addr(ring + warp * kRing);
    const uint32_t my_consumed = smem_addr(consumed + warp);
    uint32_t next_ring = 0, prev_consumed = 0;
    if (g + 1 < P.G) next_ring = mapa_shared(smem_addr(ring + ((g + 1) % wpc) * kRing), (g + 1) / wpc);
    if (g > 0) prev_consumed = mapa_shared(smem_addr(consumed + (g - 1) % wpc), (g - 1) / wpc);

    const float kk = a.kk;
    const float NEG = neg_inf();
    bool ok = true;          // false once a wait of this lane failed
    bool quit = false;       // warp-uniform
    uint32_t cons_seen = 0;  // lane 31: consumer progress last observed

    for (int band = 0; band < P.n_bands && !quit; ++band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) break;
        const int R0 = s * SR;
        const bool has_next = (s + 1 < P.n_stripes);
        const bool next_wrap = (g == P.G - 1);
        const bool prev_wrap = (g == 0);
        const bool withhold = (s == a.debug_stall);
        const uint32_t band_base = static_cast<uint32_t>(band) * static_cast<uint32_t>(M);
        float* Ts = a.score + (static_cast<size_t>(b) * P.n_stripes + s) * static_cast<size_t>(P.n_diag) * SR;
        const float* Db = a.D + static_cast<size_t>(b) * N * M;

        float cur[K], old[K];
#pragma unroll
        for (int k = 0; k < K; ++k) cur[k] = old[k] = NEG;
        float up_prev = (R0 == 0) ? 0.f : NEG;  // T(R0-1, -1)
        const int n_steps = M + SR - 1;

        for (int t = 0; t < n_steps; ++t) {
            float up = __shfl_up_sync(SDTW_FULL_MASK, cur[K - 1], 1);
            if (lane == 0) {
                up = NEG;
                if (R0 > 0 && t < M) {
                    float v = NEG;
                    if (ok) {
                        if (prev_wrap)
                            ok = wait_gmem_tag(a.wrap + static_cast<size_t>(b) * M + t, wrap_tag(a.seq, band - 1), v, a.wait);
                        else
                            ok = wait_smem_tag(my_ring + ((band_base + t) % kRing) * 8u, band_base + t, v, a.wait);
                    }
                    up = v;
                    if (!prev_wrap && (((t + 1) % (kRing / 4)) == 0 || t == M - 1))
                        st_release_cluster_u32(prev_consumed, band_base + t + 1);
                }
            }
            const float dg_top = up_prev;
            up_prev = up;
            float nw[K];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int q = lane * K + k;
                const int col = t - q;
                const int row = R0 + q;
                const float left = cur[k];
                const float u = (k == 0) ? up : cur[k > 0 ? k - 1 : 0];
                const float d = (k == 0) ? dg_top : old[k > 0 ? k - 1 : 0];
                const bool inr = (col >= 0) && (col < M) && (row < N);
                const float c = inr ? __ldg(Db + static_cast<size_t>(row) * M + col) : 0.f;
                const float m = max3f(d, u, left);
                const float sm = ex2f(d - m) + ex2f(u - m) + ex2f(left - m);
                float v = m + (lg2f(sm) - c * kk);
                const bool pruned = (a.bw > 0.f) && (fabsf(static_cast<float>(row - col)) > a.bw);
                v = (inr && !pruned && m != NEG) ? v : NEG;
                nw[k] = v;
                if (inr) Ts[static_cast<size_t>(t) * SR + k * 32 + lane] = v;
                if (row == N - 1 && col == M - 1) a.out[b] = -v * a.inv_k;
            }
            if (lane == 31 && has_next && !withhold) {
                const int col = t - (SR - 1);
                if (col >= 0 && col < M) {
                    if (next_wrap) {
                        st_gpu_u64(a.wrap + static_cast<size_t>(b) * M + col, pack_tagged(nw[K - 1], wrap_tag(a.seq, band)));
                    } else {
                        const uint32_t gc = band_base + static_cast<uint32_t>(col);
                        if (gc >= static_cast<uint32_t>(kRing) && ok &&
                            static_cast<int32_t>(cons_seen - (gc - kRing + 1)) < 0)
                            ok = wait_counter_ge(my_consumed, gc - kRing + 1, cons_seen, a.wait);
                        st_cluster_u64(next_ring + (gc % kRing) * 8u, pack_tagged(nw[K - 1], gc));
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < K; ++k) {
                old[k] = cur[k];
                cur[k] = nw[k];
            }
            if ((t & 63) == 63 && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
    }
    // No CTA may leave while a peer can still write into its shared memory.
    cluster_sync_all();
}

// ============================================================== backward
template <int K>
__device__ __forceinline__ float load_score(const float* __restrict__ S, const WavePlan& P, int b, int row, int col) {
    constexpr int SR = 32 * K;
    if (row < 0) return (col < 0) ? 0.f : neg_inf();
    if (col < 0) return neg_inf();
    const int s = row / SR;
    const int q = row - s * SR;
    const int l = q / K;
    const int k = q - l * K;
    const size_t idx = ((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + (q + col)) * SR + k * 32 + l;
    return __ldg(S + idx);
}

template <int K>
__global__ void __launch_bounds__(512) bwd_kernel(const BwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    constexpr int SR = 32 * K;
    const int N = P.N, M = P.M;

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * kRing);
    for (int i = threadIdx.x; i < wpc * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    cluster_sync_all();

    // Messages flow upward: the producer of this warp's input is warp g+1 (the
    // stripe below); this warp's output goes to warp g-1.
    const uint32_t my_ring = smem_addr(ring + warp * kRing);
    const uint32_t my_consumed = smem_addr(consumed + warp);
    uint32_t up_ring = 0, below_consumed = 0;
    if (g > 0) up_ring = mapa_shared(smem_addr(ring + ((g - 1) % wpc) * kRing), (g - 1) / wpc);
    if (g + 1 < P.G) below_consumed = mapa_shared(smem_addr(consumed + (g + 1) % wpc), (g + 1) / wpc);

    const float gb = a.grad_out ? __ldg(a.grad_out + b) : 1.f;
    bool ok = true;
    bool quit = false;
    uint32_t cons_seen = 0;  // lane 0: progress of the consumer above

    for (int band = P.n_bands - 1; band >= 0 && !quit; --band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) continue;
        const int R0 = s * SR;
        const bool has_up = (s > 0);
        const bool up_wrap = (g == 0);
        const bool has_below = (s + 1 < P.n_stripes);
        const bool below_wrap = (g == P.G - 1);
        const bool withhold = (s == a.debug_stall);
        const uint32_t band_base = static_cast<uint32_t>(P.n_bands - 1 - band) * static_cast<uint32_t>(M);
        float* Eb = a.E + static_cast<size_t>(b) * N * M;

        float accl[K], msg[K], dprev[K];
#pragma unroll
        for (int k = 0; k < K; ++k) accl[k] = msg[k] = dprev[k] = 0.f;
        const int n_steps = M + SR - 1;

        for (int t = n_steps - 1; t >= 0; --t) {
            float below = __shfl_down_sync(SDTW_FULL_MASK, msg[0], 1);
            if (lane == 31) {
                below = 0.f;
                const int col = t - (SR - 1);
                if (has_below && col >= 0 && col < M) {
                    const uint32_t gc = band_base + static_cast<uint32_t>(M - 1 - col);
                    float v = 0.f;
                    if (ok) {
                        if (below_wrap)
                            ok = wait_gmem_tag(a.wrap + static_cast<size_t>(b) * M + col, wrap_tag(a.seq, band + 1), v, a.wait);
                        else
                            ok = wait_smem_tag(my_ring + (gc % kRing) * 8u, gc, v, a.wait);
                    }
                    below = v;
                    if (!below_wrap && (((gc + 1) % (kRing / 4)) == 0 || col == 0))
                        st_release_cluster_u32(below_consumed, gc + 1);
                }
            }
            float nmsg[K];
#pragma unroll
            for (int k = K - 1; k >= 0; --k) {
                const int q = lane * K + k;
                const int col = t - q;
                const int row = R0 + q;
                const float in_below = (k == K - 1) ? below : msg[k < K - 1 ? k + 1 : 0];
                const bool inr = (col >= 0) && (col < M) && (row < N);
                const bool pruned = (a.bw > 0.f) && (fabsf(static_cast<float>(row - col)) > a.bw);
                const bool live = inr && !pruned;
                float e = accl[k] + in_below;
                if (row == N - 1 && col == M - 1) e = gb;
                e = live ? e : 0.f;
                if (inr) Eb[static_cast<size_t>(row) * M + col] = e;
                float wd = 0.f, wu = 0.f, wl = 0.f;
                if (live) {
                    const float td = load_score<K>(a.score, P, b, row - 1, col - 1);
                    const float tu = load_score<K>(a.score, P, b, row - 1, col);
                    const float tl = load_score<K>(a.score, P, b, row, col - 1);
                    const float m = max3f(td, tu, tl);
                    const float ed = ex2f(td - m), eu = ex2f(tu - m), el = ex2f(tl - m);
                    const float inv = rcpf(ed + eu + el);
                    wd = ed * inv;
                    wu = eu * inv;
                    wl = el * inv;
                }
                accl[k] = e * wl;
                nmsg[k] = e * wu + dprev[k];
                dprev[k] = e * wd;
            }
            if (lane == 0 && has_up && !withhold) {
                const int col = t;  // q = 0
                if (col >= 0 && col < M) {
                    if (up_wrap) {
                        st_gpu_u64(a.wrap + static_cast<size_t>(b) * M + col, pack_tagged(nmsg[0], wrap_tag(a.seq, band)));
                    } else {
                        const uint32_t gc = band_base + static_cast<uint32_t>(M - 1 - col);
                        if (gc >= static_cast<uint32_t>(kRing) && ok &&
                            static_cast<int32_t>(cons_seen - (gc - kRing + 1)) < 0)
                            ok = wait_counter_ge(my_consumed, gc - kRing + 1, cons_seen, a.wait);
                        st_cluster_u64(up_ring + (gc % kRing) * 8u, pack_tagged(nmsg[0], gc));
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < K; ++k) msg[k] = nmsg[k];
            if ((t & 63) == 0 && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
    }
    cluster_sync_all();
}

// ============================================================== score <-> padded R
// R (B, N+2, M+2) in the reference launcher layout (launcher.py:55-56, 177-178):
// R[:,0,0] = 0, other borders +inf, interior R = -T * gamma * ln 2.
template <int K>
__global__ void score_to_R_kernel(const float* __restrict__ S, float* __restrict__ R, WavePlan P, float inv_k) {
    const size_t total = static_cast<size_t>(P.B) * (P.N + 2) * (P.M + 2);
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(idx % (P.M + 2));
        const int i = static_cast<int>((idx / (P.M + 2)) % (P.N + 2));
        const int b = static_cast<int>(idx / (static_cast<size_t>(P.M + 2) * (P.N + 2)));
        float v;
        if (i == 0 && j == 0) v = 0.f;
        else if (i == 0 || j == 0 || i == P.N + 1 || j == P.M + 1) v = pos_inf();
        else v = -load_score<K>(S, P, b, i - 1, j - 1) * inv_k;
        R[idx] = v;
    }
}

template <int K>
__global__ void R_to_score_kernel(const float* __restrict__ R, float* __restrict__ S, WavePlan P, float kk) {
    constexpr int SR = 32 * K;
    const size_t total = static_cast<size_t>(P.B) * P.N * P.M;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(idx % P.M);
        const int row = static_cast<int>((idx / P.M) % P.N);
        const int b = static_cast<int>(idx / (static_cast<size_t>(P.M) * P.N));
        const float r = R[(static_cast<size_t>(b) * (P.N + 2) + row + 1) * (P.M + 2) + col + 1];
        const int s = row / SR;
        const int q = row - s * SR;
        const int l = q / K;
        const int k = q - l * K;
        S[((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + (q + col)) * SR + k * 32 + l] = -r * kk;
    }
}

// ============================================================== launchers
static cudaError_t launch_cluster(const void* fn, dim3 grid, dim3 block, size_t smem, int csize,
                                  cudaStream_t stream, void** args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

static size_t ring_smem_bytes(const WavePlan& P) {
    return static_cast<size_t>(P.wpc) * kRing * 8u + static_cast<size_t>(P.wpc) * 4u;
}

cudaError_t launch_forward(const FwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    dim3 grid(P.B * P.csize), block(P.wpc * 32);
    void* kargs[] = {const_cast<FwdArgs*>(&args)};
    switch (P.K) {
        case 1: return launch_cluster((const void*)fwd_kernel<1>, grid, block, ring_smem_bytes(P), P.csize, stream, kargs);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_backward(const BwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    dim3 grid(P.B * P.csize), block(P.wpc * 32);
    void* kargs[] = {const_cast<BwdArgs*>(&args)};
    switch (P.K) {
        case 1: return launch_cluster((const void*)bwd_kernel<1>, grid, block, ring_smem_bytes(P), P.csize, stream, kargs);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_score_to_R(const float* S, float* R, const WavePlan& P, float inv_k, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(P.B) * (P.N + 2) * (P.M + 2);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<size_t>((total + threads - 1) / threads, 148u * 16u));
    switch (P.K) {
        case 1: score_to_R_kernel<1><<<blocks, threads, 0, stream>>>(S, R, P, inv_k); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_R_to_score(const float* R, float* S, const WavePlan& P, float kk, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(P.B) * P.N * P.M;
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<size_t>((total + threads - 1) / threads, 148u * 16u));
    switch (P.K) {
        case 1: R_to_score_kernel<1><<<blocks, threads, 0, stream>>>(R, S, P, kk); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sdtw
