// barycenter.cu -- the device side of one Soft-DTW barycenter iteration
// around the wavefronts (softdtw_cuda/barycenters.py:114-137 of the
// reference):
//
//   barycenter_batch = barycenter.unsqueeze(0).expand(B, -1, -1)   (122)
//   loss = (weights * SoftDTW(barycenter_batch, X)).sum()           (125-128)
//   loss.backward()                                                 (131)
//   clip_grad_norm_([barycenter], max_norm=1.0)                     (134)
//   optimizer.step()  (Adam), scheduler.step() (cosine annealing)   (136-137)
//
// The wavefronts and the gradient kernels read the barycenter once for every
// problem (x batch stride 0), and their per-problem results are reduced here:
//   bary_reduce   grad_loss[v] = sum_b gx[b, v] for v < n (the expand's
//                 backward) and grad_loss[n] = sum_b w[b] * out[b] (the loss),
//                 in a fixed order: slices of problems to partials, then the
//                 partials in slice order -- deterministic, no atomics;
//   bary_adam     one CTA: the gradient's 2-norm, the clip factor
//                 min(1, max_norm / (norm + 1e-6)), and Adam (Kingma & Ba,
//                 2015) with torch's update form: m <- lerp(m, g, 1 - beta1),
//                 v <- beta2 v + (1 - beta2) g^2, p <- p - lr / (1 - beta1^t)
//                 * m / (sqrt(v) / sqrt(1 - beta2^t) + eps), t = step + 1, lr =
//                 lr_table[step] (the cosine schedule, precomputed); then the
//                 loss and the new barycenter are recorded at index step and
//                 step is incremented.  Everything the iteration needs stays on
//                 the device, so the iteration can be captured in a CUDA graph.
#include <algorithm>
#include <cmath>

#include "sdtw_kernels.h"

namespace sdtw {

namespace {
constexpr int kReduceThreads = 256;
constexpr int kReduceSlices = 64;  // problem slices of the first reduction stage
constexpr int kAdamThreads = 512;

int reduce_slices(int B) { return B < kReduceSlices ? B : kReduceSlices; }
}  // namespace

__global__ void bary_broadcast_kernel(const float* __restrict__ bary, float* __restrict__ xb, int B, size_t n) {
    const size_t total = static_cast<size_t>(B) * n;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        xb[i] = __ldg(bary + i % n);
}

// Stage 1: slice s of the problems, values v = blockIdx.x * 256 + thread (v ==
// n is the weighted loss).
__global__ void __launch_bounds__(kReduceThreads) bary_reduce_part_kernel(const float* __restrict__ gx,
                                                                         const float* __restrict__ w,
                                                                         const float* __restrict__ out,
                                                                         float* __restrict__ part, int B, size_t n) {
    pdl_trigger();
    pdl_wait();
    const size_t v = static_cast<size_t>(blockIdx.x) * kReduceThreads + threadIdx.x;
    if (v > n) return;
    const int S = gridDim.y, s = blockIdx.y;
    const int b0 = static_cast<int>(static_cast<long long>(B) * s / S);
    const int b1 = static_cast<int>(static_cast<long long>(B) * (s + 1) / S);
    float acc = 0.f;
    if (v < n) {
#pragma unroll 8
        for (int b = b0; b < b1; ++b) acc += __ldg(gx + static_cast<size_t>(b) * n + v);
    } else {
#pragma unroll 8
        for (int b = b0; b < b1; ++b) acc = fmaf(__ldg(w + b), __ldg(out + b), acc);
    }
    part[static_cast<size_t>(s) * (n + 1) + v] = acc;
}

// Stage 2: the slices' partials in slice order.
__global__ void __launch_bounds__(kReduceThreads) bary_reduce_final_kernel(const float* __restrict__ part,
                                                                          float* __restrict__ grad_loss, int S,
                                                                          size_t n) {
    pdl_trigger();
    pdl_wait();
    const size_t v = static_cast<size_t>(blockIdx.x) * kReduceThreads + threadIdx.x;
    if (v > n) return;
    float acc = 0.f;
#pragma unroll 8
    for (int s = 0; s < S; ++s) acc += __ldg(part + static_cast<size_t>(s) * (n + 1) + v);  // loads in flight together
    grad_loss[v] = acc;
}

// Block-wide sum in a fixed order (per-thread partials, then a tree).
__device__ float block_sum(float v, float* red) {
    red[threadIdx.x] = v;
    __syncthreads();
    for (int h = blockDim.x / 2; h > 0; h >>= 1) {
        if (threadIdx.x < h) red[threadIdx.x] += red[threadIdx.x + h];
        __syncthreads();
    }
    const float r = red[0];
    __syncthreads();
    return r;
}

// Clip to max_norm given the gradient's 2-norm, one Adam step at iteration it
// with learning rate lr, and the loss and new barycenter recorded at index it
// (the caller advances the step counter after a barrier).
__device__ void adam_update(float* __restrict__ bary, float* __restrict__ m, float* __restrict__ v,
                            const float* __restrict__ grad_loss, size_t n, float lr, int it,
                            float* __restrict__ loss_hist, float* __restrict__ bary_hist, float beta1, float beta2,
                            float eps, float max_norm, float norm) {
    const float clip = fminf(max_norm / (norm + 1e-6f), 1.f);
    const double t = static_cast<double>(it) + 1.0;
    const float bc1 = static_cast<float>(1.0 - pow(static_cast<double>(beta1), t));
    const float bc2_sqrt = sqrtf(static_cast<float>(1.0 - pow(static_cast<double>(beta2), t)));
    const float step_size = lr / bc1;
    float* hist = bary_hist + static_cast<size_t>(it) * n;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float g = grad_loss[i] * clip;
        float mi = m[i], vi = v[i];
        mi = fmaf(1.f - beta1, g - mi, mi);
        vi = fmaf(1.f - beta2, g * g, vi * beta2);
        const float p = bary[i] - step_size * (mi / (sqrtf(vi) / bc2_sqrt + eps));
        m[i] = mi;
        v[i] = vi;
        bary[i] = p;
        hist[i] = p;
    }
    if (threadIdx.x == 0) loss_hist[it] = grad_loss[n];
}

__global__ void __launch_bounds__(kAdamThreads) bary_adam_kernel(float* __restrict__ bary, float* __restrict__ m,
                                                                float* __restrict__ v,
                                                                const float* __restrict__ grad_loss, size_t n,
                                                                const float* __restrict__ lr_table, int max_iter,
                                                                int* __restrict__ step, float* __restrict__ loss_hist,
                                                                float* __restrict__ bary_hist, float beta1, float beta2,
                                                                float eps, float max_norm) {
    __shared__ float red[kAdamThreads];
    pdl_trigger();
    pdl_wait();
    const int it = *step;
    if (it < 0 || it >= max_iter) return;  // more replays than iterations: nothing to do
    float sq = 0.f;
    for (size_t i = threadIdx.x; i < n; i += kAdamThreads) {
        const float g = grad_loss[i];
        sq = fmaf(g, g, sq);
    }
    adam_update(bary, m, v, grad_loss, n, lr_table[it], it, loss_hist, bary_hist, beta1, beta2, eps, max_norm,
                sqrtf(block_sum(sq, red)));
    __syncthreads();
    if (threadIdx.x == 0) *step = it + 1;
}

// ---------------------------------------------------------------- multi-GPU
// The sum over ranks of [grad | loss] and the Adam step in one kernel, over
// peer memory (one CTA per GPU; replaces an all-reduce and the Adam launch).
// Every rank's exchange buffer (same layout on every rank, all of them mapped
// into every rank's address space) holds data [2][world][n + 1] floats, then
// flags [world] u64.  Iteration e (a device counter, the same on every rank:
// each kernel advances it by one) writes this rank's [grad | loss] into slot
// (e & 1, rank) of every rank's buffer with plain stores over NVLink, then sets
// flag `rank` of every rank's buffer to e (release, system scope); it then waits
// until all `world` flags of its own buffer reach e (acquire), and sums the
// slots in rank order, so every rank gets the same bits.  A rank can run at
// most one iteration ahead of another (iteration e + 1 needs everybody's
// e + 1 data), so the two parities never collide.  A wait that runs out of time
// records status 3 and skips the update.
__host__ __device__ inline size_t sync_flag_offset(size_t n, int world) {
    return (2 * static_cast<size_t>(world) * (n + 1) * sizeof(float) + 7) / 8 * 8;
}
size_t bary_sync_bytes(size_t n, int world) { return sync_flag_offset(n, world) + static_cast<size_t>(world) * 8; }

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kAdamThreads) bary_sync_adam_kernel(
    float* __restrict__ grad_loss, size_t n, const unsigned long long* __restrict__ peers, int world, int rank,
    unsigned long long* __restrict__ epoch, float* __restrict__ bary, float* __restrict__ m, float* __restrict__ v,
    const float* __restrict__ lr_table, int max_iter, int* __restrict__ step, float* __restrict__ loss_hist,
    float* __restrict__ bary_hist, float beta1, float beta2, float eps, float max_norm, WaitCtx wc) {
    __shared__ float red[kAdamThreads];
    __shared__ int ok_s;
    pdl_trigger();
    pdl_wait();
    const size_t n1 = n + 1;
    const unsigned long long e = *epoch + 1;
    const size_t par = static_cast<size_t>(e & 1ull);
    const size_t foff = sync_flag_offset(n, world);
    // This rank's [grad | loss] into its slot of every rank's buffer.
    for (int r = 0; r < world; ++r) {
        float* dst = reinterpret_cast<float*>(peers[r]) + (par * world + rank) * n1;
        for (size_t i = threadIdx.x; i < n1; i += kAdamThreads) dst[i] = grad_loss[i];
    }
    if (threadIdx.x == 0) ok_s = 1;
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < world) {
        __threadfence_system();
        st_release_sys_u64(reinterpret_cast<unsigned long long*>(peers[threadIdx.x] + foff) + rank, e);
        const unsigned long long* f = reinterpret_cast<const unsigned long long*>(peers[rank] + foff) + threadIdx.x;
        uint64_t t0 = 0;
        for (uint32_t it = 1;; ++it) {
            const unsigned long long s = ld_acquire_sys_u64(f);
            if (s >= e) break;
            const int r = backoff(it, t0, wc);
            if (r) {
                record_giveup(wc, r, 7, static_cast<uint32_t>(e), static_cast<uint32_t>(s));
                ok_s = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!ok_s) return;
    // The sum over ranks, in rank order, replaces this rank's [grad | loss].
    const float* mine = reinterpret_cast<const float*>(peers[rank]) + par * world * n1;
    float sq = 0.f;
    for (size_t i = threadIdx.x; i < n1; i += kAdamThreads) {
        float g = 0.f;
        for (int r = 0; r < world; ++r) g += __ldcg(mine + r * n1 + i);  // L2: peers wrote it over NVLink
        grad_loss[i] = g;
        if (i < n) sq = fmaf(g, g, sq);
    }
    __syncthreads();
    if (threadIdx.x == 0) *epoch = e;
    const int it = *step;
    if (it < 0 || it >= max_iter) return;
    adam_update(bary, m, v, grad_loss, n, lr_table[it], it, loss_hist, bary_hist, beta1, beta2, eps, max_norm,
                sqrtf(block_sum(sq, red)));
    __syncthreads();
    if (threadIdx.x == 0) *step = it + 1;
}

cudaError_t launch_bary_sync_adam(float* grad_loss, size_t n, const unsigned long long* peers, int world, int rank,
                                  unsigned long long* epoch, float* bary, float* exp_avg, float* exp_avg_sq,
                                  const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                                  float beta1, float beta2, float eps, float max_norm, const WaitCtx& wc,
                                  cudaStream_t st) {
    WaitCtx w = wc;
    w.kernel = 7;
    w.problem = rank;
    return launch_pdl(true, bary_sync_adam_kernel, dim3(1), dim3(kAdamThreads), 0, st, grad_loss, n, peers, world, rank,
                      epoch, bary, exp_avg, exp_avg_sq, lr_table, max_iter, step, loss_hist, bary_hist, beta1, beta2,
                      eps, max_norm, w);
}

cudaError_t launch_bary_broadcast(const float* bary, float* xb, int B, size_t n, cudaStream_t st) {
    const size_t total = static_cast<size_t>(B) * n;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 148 * 8));
    bary_broadcast_kernel<<<blocks, 256, 0, st>>>(bary, xb, B, n);
    return cudaGetLastError();
}

size_t bary_reduce_part_floats(int B, size_t n) { return static_cast<size_t>(reduce_slices(B)) * (n + 1); }

cudaError_t launch_bary_reduce(const float* gx, const float* w, const float* out, float* part, float* grad_loss, int B,
                               size_t n, cudaStream_t st) {
    const int S = reduce_slices(B);
    const unsigned bx = static_cast<unsigned>((n + 1 + kReduceThreads - 1) / kReduceThreads);
    cudaError_t e = launch_pdl(true, bary_reduce_part_kernel, dim3(bx, S), dim3(kReduceThreads), 0, st, gx, w, out, part, B, n);
    if (e != cudaSuccess) return e;
    return launch_pdl(true, bary_reduce_final_kernel, dim3(bx), dim3(kReduceThreads), 0, st, part, grad_loss, S, n);
}

cudaError_t launch_bary_adam(float* bary, float* exp_avg, float* exp_avg_sq, const float* grad_loss, size_t n,
                             const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                             float beta1, float beta2, float eps, float max_norm, cudaStream_t st) {
    return launch_pdl(true, bary_adam_kernel, dim3(1), dim3(kAdamThreads), 0, st, bary, exp_avg, exp_avg_sq, grad_loss, n,
                      lr_table, max_iter, step, loss_hist, bary_hist, beta1, beta2, eps, max_norm);
}

}  // namespace sdtw
