// sdtw_kernels.h -- argument blocks and launchers of the device kernels
// (internal to libsdtw_b200; the public C-ABI is include/sdtw_b200.h).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "sdtw_device.cuh"
#include "sdtw_plan.h"

namespace sdtw {

// Where the problems of a launch find their sequences.  Problem b lies in
// segment s (0 for b < per, 1 for b < 2 per, else 2) and uses row block
// b - s * per of p[s].  A plain batch is one segment (one_seq); the three
// segments (x, y), (x, x), (y, y) of B problems each are the normalized loss's
// triple, read from the caller's x and y in place (norm_x / norm_y).
template <typename T>
struct Seqs {
    T* p[3];
    int per;
    __host__ __device__ __forceinline__ T* at(int b, size_t stride) const {
        const int s = b < per ? 0 : (b - per < per ? 1 : 2);
        return (s == 0 ? p[0] : (s == 1 ? p[1] : p[2])) + static_cast<size_t>(b - s * per) * stride;
    }
    __host__ __device__ __forceinline__ bool null() const { return p[0] == nullptr; }
    bool aligned16() const {
        return ((reinterpret_cast<uintptr_t>(p[0]) | reinterpret_cast<uintptr_t>(p[1]) |
                 reinterpret_cast<uintptr_t>(p[2])) & 15u) == 0;
    }
};
using SeqIn = Seqs<const float>;
using SeqOut = Seqs<float>;
template <typename T>
inline Seqs<T> one_seq(T* p) {
    return Seqs<T>{{p, p, p}, 1 << 30};
}
// The normalized triple's first and second operands over B problems each.
inline SeqIn norm_x(const float* x, const float* y, int B) { return SeqIn{{x, x, y}, B}; }
inline SeqIn norm_y(const float* x, const float* y, int B) { return SeqIn{{y, x, y}, B}; }

struct FwdArgs {
    WavePlan P;
    const float* Dw;  // (B,N,M) cost in the wavefront layout (layout.cu)
    float2* score;    // wavefront-layout score store, (hi, lo) pairs (see sdtw_plan.h)
    float* out;       // (B,) R[N,M]
    uint64_t* wrap;   // (B*M) band-wrap ring, null when n_bands == 1
    float kk;         // log2(e) / gamma
    float inv_k;      // gamma * ln(2)
    double inv_k_d;   // gamma * ln(2) in double (the loss of the exponential-domain forward)
    float bw;         // Sakoe-Chiba bandwidth, <= 0 disables
    int ibw;          // integer band: cell (i, j) is kept when |i - j| <= ibw (floor(bw), or 2^29 when disabled)
    uint32_t seq;     // launch sequence number (tags of the global ring)
    int debug_stall;  // stripe whose output is withheld (failure-detection tests); -1 = none
    int weights;      // nonzero: store each cell's predecessor weights instead of its score (one row per lane)
    // Fused costs (wavefront_exp.cu, dp > 0): sum_k (x_ik - y_jk)^2 computed in
    // the kernel from x (B,N,dim) and y (B,M,dim); Dw is then unused.
    SeqIn x;
    SeqIn y;
    int dim;
    int dp;           // 0: costs from Dw; else the feature padding (fused_dp)
    size_t x_bstride;  // floats between problems' x (N * dim; 0 = one x for every problem)
    int wide;          // nonzero: the 128-register forward (fwdx_kernel WIDE), pass 32 + (its pass)
    int clamp_mask;    // nonzero (share store): the sign bit of a cell's diagonal share marks a cost that
                       // is not > 0 (the unfused cost's clamp), and the reverse pass stores E = 0 there
    WaitCtx wait;
};

struct BwdArgs {
    WavePlan P;
    const float2* score;
    const float* grad_out;  // (B,) upstream gradient, null = ones
    float* Ew;              // (B,N,M) output in the wavefront layout: grad_out[b] * dR[N,M]/dD[i,j]
    uint64_t* wrap;
    float bw;
    int ibw;
    uint32_t seq;
    int debug_stall;
    int weights;  // nonzero: `score` holds the forward's predecessor weights (one row per lane)
    int clamp_mask;  // nonzero: those weights carry the forward's clamp marks (FwdArgs::clamp_mask)
    // grad_x in the reverse pass (gd > 0; the fused cost, weight store, no
    // band): E is not stored; each lane accumulates its row's sum_j E y_j and
    // sum_j E and writes grad_x.
    const float* x;
    const float* y;
    int dim;
    int gd;             // features padded to 4, 8 or 16; 0 = store E
    size_t x_bstride;   // floats between problems' x (N * dim; 0 = one x for all)
    float* gx;          // (B,N,dim) grad_x
    int pdl;            // nonzero: launched with programmatic stream serialization (after the forward)
    WaitCtx wait;
};

cudaError_t launch_forward(const FwdArgs& args, cudaStream_t stream);
// wavefront_exp.cu: the one-row-per-lane forward (exponential domain) and the
// reverse pass over its stored shares; launch_forward / launch_backward route
// K = 1 to them.
cudaError_t launch_forward_x(const FwdArgs& args, cudaStream_t stream);
cudaError_t launch_backward_w(const BwdArgs& args, cudaStream_t stream);
size_t fwdx_smem(const WavePlan& P, int dp, bool wide = false);
int fwdx_threads(const WavePlan& P);
int fused_dp(int dim, const SeqIn& x, const SeqIn& y);
size_t bwdw_smem(const WavePlan& P, int gd = 0);
// cm: the variants that mark clamped costs (shares of an unfused cost table);
// seg: the fused variants for problems in several segments (SeqIn).
const void* fwdx_fn(bool banded, bool weights, int dp, bool wide = false, bool cm = false, bool seg = false);
const void* bwdw_fn(bool banded, int gd = 0, bool cm = false);
// Feature padding of the reverse pass with grad_x (4, 8, 16), or 0.
int grad_fused_gd(int dim, const float* y);
// pass: 0 forward with costs from a table, 1 reverse pass, 2 + dp the fused
// forward, 32 + those forward passes their 128-register variants, 64 + gd the
// reverse pass with grad_x.
int max_active_clusters(const WavePlan& P, int pass);
cudaError_t launch_backward(const BwdArgs& args, cudaStream_t stream);
cudaError_t launch_score_to_R(const float2* S, float* R, const WavePlan& P, float inv_k, cudaStream_t stream);
cudaError_t launch_R_to_score(const float* R, float2* S, const WavePlan& P, float kk, cudaStream_t stream);

// layout.cu
cudaError_t launch_cost_wl(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, bool direct,
                           cudaStream_t stream);
cudaError_t launch_rm_to_wl(const float* A, float* Aw, const WavePlan& P, cudaStream_t stream);
cudaError_t launch_wl_to_rm(const float* Aw, const float* maskw, float* A, const WavePlan& P, cudaStream_t stream);
// WL -> row-major A (B,N,lda) and its transpose AT (B,M,ldt), with the optional
// mask; lda >= M, ldt >= N are the row pitches (padding written as zeros).
cudaError_t launch_wl_to_rm_cm(const float* Aw, const float* maskw, float* A, int lda, float* AT, int ldt,
                               const WavePlan& P, cudaStream_t stream);
// (B,R,C) -> (B,C,ldo), ldo >= R, columns R .. ldo zero.
// (B,R,C) -> chunked (B, ceil(R/32), C, 36): out[b][c][f][kk] = in[b][32c+kk][f]
// for kk < 32, zero for 32c+kk >= R and for kk >= 32; two arrays (rows R0 and
// R1, either input may be null) in one launch.
cudaError_t launch_transpose_chunked(const SeqIn& in0, float* out0, int R0, const SeqIn& in1, float* out1, int R1,
                                     int B, int C, cudaStream_t stream);
cudaError_t launch_transpose_brc(const SeqIn& in, float* out, int B, int R, int C, int ldo, cudaStream_t stream);

// dense.cu
cudaError_t launch_cost(const float* x, const float* y, float* D, int B, int N, int M, int dim, bool direct,
                        cudaStream_t stream);
cudaError_t launch_grad_xy(const float* G, const float* mask, const float* x, const float* y, float* gx,
                           float* gy, int B, int N, int M, int dim, cudaStream_t stream);

// tcgemm.cu: grad_x / grad_y from E in the wavefront layout on the tensor cores.
struct GradTcArgs {
    // grad_wl: 2-D views (rows of 32 floats) of E and of the mask for the
    // grad_y tiles' tensor copies; filled in by launch_grad_wl.
    alignas(64) CUtensorMap tm_e;
    alignas(64) CUtensorMap tm_m;
    WavePlan P;
    const float* Ew;  // E in the wavefront layout (grad_wl)
    // grad_wl: x and y in the chunked transposed layout [b][c][f][kk] = x[b][32c+kk][f],
    // rows of 36 floats (the last 4 zero)
    const float* xTc;
    const float* yTc;
    // grad_rm operands, rows zero-padded to Np = N rounded up to 32, Mp likewise:
    const float* G;   // G = E (clamp mask applied) (B,N,Mp)
    const float* GT;  // G transposed (B,M,Np)
    const float* xT;  // x transposed (B,dim,Np)
    const float* yT;  // y transposed (B,dim,Mp)
    const float* Mw;  // unfused cost in the wavefront layout (clamp mask: G = E * (D > 0)), or null
    SeqIn x;          // (B,N,dim)
    SeqIn y;          // (B,M,dim)
    SeqOut gx;        // (B,N,dim) or null
    SeqOut gy;        // (B,M,dim) or null
    int dim;
    int fb;           // features per block
    int nt;           // fb rounded up to 16
    int n_fblk;       // feature blocks
    int tiles_x;      // 128-row tiles of grad_x per problem (0 when gx is null)
    int tiles_y;      // 128-row tiles of grad_y per problem (0 when gy is null)
    int tmem_cols;    // tensor-memory columns allocated per CTA (power of two >= nt)
    int stages;       // shared-memory pipeline depth (grad_rm)
    int stages_x;     // ring slots of the grad_x tiles (grad_wl)
    int stages_y;     // ring slots of the grad_y tiles (grad_wl)
    int ops_x;        // operand buffers of the grad_x tiles (grad_wl: 1 or 2)
    int ops_y;        // operand buffers of the grad_y tiles (grad_wl: 1 or 2)
    WaitCtx wait;
};
// From E in the wavefront layout with bulk copies (one row per lane only).
bool grad_wl_supported(const WavePlan& P);
void grad_wl_geometry(int dim, bool masked, GradTcArgs* g);
cudaError_t launch_grad_wl(const GradTcArgs& args, cudaStream_t stream);
// The same from row-major G, G^T, x^T and y^T (16-byte operand copies).
void grad_rm_geometry(int dim, int* fb, int* nt, int* n_fblk, int* tmem_cols, int* stages);
cudaError_t launch_grad_rm(const GradTcArgs& args, cudaStream_t stream);
// grad_small.cu: both gradients on the FP32 pipes for dim <= 16, from E in the
// wavefront layout (one row per lane); `part` holds grad_small_part_bytes of
// per-split column sums (needed when gy is set).
bool grad_small_supported(const WavePlan& P, int dim);
size_t grad_small_part_bytes(const WavePlan& P, int dim);
// x_bstride: floats between problems' x (N * dim; 0 = one x shared by all).
cudaError_t launch_grad_small(const float* Ew, const float* Mw, const SeqIn& x, const SeqIn& y, const SeqOut& gx,
                              const SeqOut& gy, float* part, const WavePlan& P, int dim, cudaStream_t st,
                              size_t x_bstride);

// barycenter.cu: the reductions and the optimiser step of the barycenter loop.
//   bary_broadcast: xb[b] = bary for every problem b (materialised x).
//   bary_reduce: grad_loss[v] = sum_b gx[b, v] (v < n), grad_loss[n] =
//     sum_b w[b] * out[b], in a fixed order (two kernels, `part` holds
//     bary_reduce_part_floats).
//   bary_adam: clip the gradient to norm max_norm, one Adam step with the
//     learning rate lr_table[*step], record loss and barycenter, ++*step.
cudaError_t launch_bary_broadcast(const float* bary, float* xb, int B, size_t n, cudaStream_t st);
size_t bary_reduce_part_floats(int B, size_t n);
cudaError_t launch_bary_reduce(const float* gx, const float* w, const float* out, float* part, float* grad_loss, int B,
                               size_t n, cudaStream_t st);
cudaError_t launch_bary_adam(float* bary, float* exp_avg, float* exp_avg_sq, const float* grad_loss, size_t n,
                             const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                             float beta1, float beta2, float eps, float max_norm, cudaStream_t st);
//   bary_sync_adam: the sum over `world` ranks of [grad | loss] through the
//     exchange buffers `peers` (every rank's, bary_sync_bytes each) and the
//     Adam step in one kernel; grad_loss is replaced by the sum.
size_t bary_sync_bytes(size_t n, int world);
cudaError_t launch_bary_sync_adam(float* grad_loss, size_t n, const unsigned long long* peers, int world, int rank,
                                  unsigned long long* epoch, float* bary, float* exp_avg, float* exp_avg_sq,
                                  const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                                  float beta1, float beta2, float eps, float max_norm, const WaitCtx& wc,
                                  cudaStream_t st);
// tcgemm.cu: the unfused (expanded, clamped) cost on the tensor cores, written
// in the wavefront layout.  Requires dim >= 16, dim % 4 == 0 and 16-byte
// aligned x, y (cost_tc_supported).
bool cost_tc_supported(const SeqIn& x, const SeqIn& y, int dim);
cudaError_t launch_cost_tc(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, const WaitCtx& wait,
                           cudaStream_t stream);
// The same cost row-major (B, N, M) for distances.sqeuclidean (same requirements).
cudaError_t launch_cost_tc_rm(const float* x, const float* y, float* D, int B, int N, int M, int dim,
                              const WaitCtx& wait, cudaStream_t stream);
// normalize: gx += a + b over n floats (the triple's gradients folded into x's / y's)
cudaError_t launch_add2(float* g, const float* a, const float* b, size_t n, cudaStream_t stream);

// f64.cu: the float64 pipeline (reference layout R, one CTA per problem).
cudaError_t launch_forward_f64(const double* D, double* R, double* out, int B, int N, int M, double gamma, double bw,
                               cudaStream_t stream);
cudaError_t launch_backward_f64(const double* D, const double* R, const double* grad_out, double* E, int B, int N,
                                int M, double gamma, double bw, cudaStream_t stream);
cudaError_t launch_cost_f64(const double* x, const double* y, double* D, int B, int N, int M, int dim,
                            cudaStream_t stream);
// grad_x, grad_y (either may be null) of the direct cost from G = dL/dD (B,N,M), in double.
cudaError_t launch_grad_f64(const double* G, const double* x, const double* y, double* gx, double* gy, int B, int N,
                            int M, int dim, cudaStream_t stream);

}  // namespace sdtw
