/*
 * sdtw_b200.h -- C ABI of libsdtw_b200.so, the B200 (sm_100a) Soft-DTW engine.
 *
 * Plain pointers and sizes only: every device pointer is a CUDA device
 * address of float32 data, row-major and contiguous; `stream` is a
 * cudaStream_t passed as void* (NULL = the legacy default stream).  Every entry
 * point validates its arguments, enqueues its kernels on `stream` and returns
 * without synchronising.  The library allocates no device memory: the caller
 * passes the outputs and a workspace of the size the *_workspace_bytes
 * functions report.  The only persistent allocation is one mapped pinned host
 * word used as the error status of the device-side bounded waits.
 *
 * Each entry point replaces one function of the reference package
 * (BGU-CS-VIL/sdtw-cuda-torch, softdtw_cuda/...), cited below as file:line.
 *
 * The "score" table takes the place of the reference's R table
 * (B, N+2, M+2): it holds T = -R * log2(e) / gamma for every cell, as a pair
 * of float32 (hi, lo) with T = hi + lo, in the anti-diagonal ("wavefront")
 * layout the kernels write by whole anti-diagonal rows.  It must be 16-byte aligned;
 * workspaces 256-byte aligned.  The cost table of the unfused x/y entry points
 * (sdtw_cost_elems floats) uses the same anti-diagonal layout and must be
 * 16-byte aligned.
 * sdtw_score_to_R_f32 / sdtw_R_to_score_f32 convert the table of
 * sdtw_forward_f32 to and from the reference layout.  The x/y pairs
 * (sdtw_forward_xy_f32 / sdtw_backward_xy_f32 and the sqeuclid pair) keep, in a
 * buffer of the same size, the state their backward needs: with one row per
 * lane, each cell's softmax weights of its diagonal and upper predecessors
 * instead of its score.  Pass that buffer only to the matching backward.
 */
#ifndef SDTW_B200_H
#define SDTW_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define SDTW_OK 0
#define SDTW_ERR_INVALID_ARGUMENT 1 /* bad size, pointer, gamma or workspace */
#define SDTW_ERR_CUDA 2             /* a CUDA runtime call failed (see sdtw_last_error_message) */
#define SDTW_ERR_TIMEOUT 3          /* a device-side wait ran out of time; results are invalid */
#define SDTW_ERR_RANGE 4            /* the forward's values left the float32 exponential-domain range
                                       (|R|/gamma >= 3.7e8, |cost|*log2(e)/gamma >= 4.2e6, or a NaN
                                       cost); results are invalid */

/* Library version string. */
const char *sdtw_version(void);

/* Human-readable text for a return code, and detail of the last failure on
 * the calling thread. */
const char *sdtw_error_string(int code);
const char *sdtw_last_error_message(void);

/* Reads and clears the device status word written by the kernels' bounded
 * waits (0 = no failure; on failure sdtw_last_error_message says which wait
 * gave up).  It does not synchronise: call it after the stream has been
 * synchronised to observe the kernels enqueued before.  Once the current
 * device has run sdtw_forward_noalloc_f32, it also reads that entry point's
 * device status word (a small synchronous copy). */
int sdtw_status(void);

/* Wall-clock limit of one device-side wait, in nanoseconds (default 2e9). */
void sdtw_set_wait_timeout_ns(unsigned long long ns);

/* Per-kernel device timing.  While enabled, every kernel the library launches
 * is bracketed by CUDA events on its stream.  sdtw_timing_read synchronises the
 * recorded events, and returns per kernel name (comma-separated in `names`)
 * the total milliseconds and launch count accumulated since enabling; the
 * return value is the number of entries.  Enabling clears the totals. */
void sdtw_timing_enable(int on);
int sdtw_timing_read(char *names, size_t names_len, double *total_ms, long *counts, int max_entries);

/* Failure-detection test hook: the producer of stripe `stripe` (32-row band
 * of the DP table) withholds its output so that its consumer's wait runs out.
 * -1 disables.  Never set outside tests. */
void sdtw_debug_stall_stripe(int stripe);

/* Tuning/test hook: force the stripes (chain warps) per CTA (1..8), the thread-block cluster
 * size (1..8) and the DP rows per lane (1, 2 or 4) of the wavefront launches;
 * 0 restores the automatic choice.  The score layout depends on the rows per
 * lane, so a forward and its backward must run under the same setting. */
void sdtw_set_plan_override(int warps_per_cta, int cluster_size, int rows_per_lane);

/* Diagnostic: number of kernels the library has launched since it was loaded
 * (every entry point counts the kernels it enqueues).  No counterpart in the
 * reference. */
unsigned long long sdtw_launch_count(void);

/* Diagnostic: the launch geometry chosen for a (B,N,M) problem on the
 * current device.  info[0..5] = DP rows per lane, warps per CTA, cluster size,
 * bands, stripes, clusters of that geometry that fit on the device at once
 * (-1 if unknown).  No counterpart in the reference. */
int sdtw_plan_info(int B, int N, int M, int *info);

/* Number of float32 elements of the score table for a (B,N,M) problem. */
size_t sdtw_score_elems(int B, int N, int M);

/* Number of float32 elements of the cost table kept between
 * sdtw_forward_sqeuclid_f32 and sdtw_backward_sqeuclid_f32. */
size_t sdtw_cost_elems(int B, int N, int M);

/* Workspace bytes of sdtw_forward_f32 / sdtw_backward_f32 (D input). */
size_t sdtw_workspace_bytes(int B, int N, int M);

/* Workspace bytes of the x, y entry points (sdtw_forward_xy_f32,
 * sdtw_backward_xy_f32, sdtw_forward_sqeuclid_f32, sdtw_backward_sqeuclid_f32). */
size_t sdtw_workspace_bytes_xy(int B, int N, int M, int dim);

/* Cost matrix D (B,N,M) from x (B,N,dim), y (B,M,dim).
 *   direct == 0: ||x_i||^2 + ||y_j||^2 - 2 x_i.y_j clamped at 0
 *                -- replaces softdtw_cuda/distances.py:6-28 (sqeuclidean)
 *   direct != 0: sum_k (x_ik - y_jk)^2
 *                -- the fused cost of softdtw_cuda/cuda/kernels.py:27-31 */
int sdtw_cost_sqeuclid_f32(const float *x, const float *y, float *D, int B, int N, int M, int dim,
                           int direct, void *stream);

/* Forward DP over a cost matrix: score (sdtw_score_elems) and out (B,) = R[N,M].
 * bandwidth <= 0 disables the Sakoe-Chiba band.
 * -- replaces softdtw_cuda/cuda/launcher.py:167-223 (softdtw_forward_cuda) */
int sdtw_forward_f32(const float *D, float *score, float *out, int B, int N, int M, float gamma,
                     float bandwidth, void *workspace, size_t workspace_bytes, void *stream);

/* Reverse DP: E (B,N,M) = grad_out[b] * d out[b] / d D[b,i,j] (grad_out NULL = ones).
 * -- replaces softdtw_cuda/cuda/launcher.py:226-300 (softdtw_backward_cuda_log)
 *    together with the scaling of softdtw_cuda/autograd.py:46-47 */
int sdtw_backward_f32(const float *score, const float *grad_out, float *E, int B, int N, int M,
                      float gamma, float bandwidth, void *workspace, size_t workspace_bytes,
                      void *stream);

/* Fused forward on x (B,N,dim), y (B,M,dim) with the direct squared-Euclidean
 * cost.  -- replaces softdtw_cuda/cuda/launcher.py:33-87
 *          (softdtw_forward_cuda_fused_sqeuclid) */
int sdtw_forward_xy_f32(const float *x, const float *y, float *score, float *out, int B, int N, int M,
                        int dim, float gamma, float bandwidth, void *workspace, size_t workspace_bytes,
                        void *stream);

/* Fused backward: grad_x (B,N,dim), grad_y (B,M,dim) of sum_b grad_out[b]*out[b]
 * (either gradient pointer may be NULL).
 * -- replaces softdtw_cuda/cuda/launcher.py:90-162
 *    (softdtw_backward_cuda_fused_sqeuclid) and the chain rule of
 *    softdtw_cuda/autograd_xy.py:32-51 */
int sdtw_backward_xy_f32(const float *x, const float *y, const float *score, const float *grad_out,
                         float *grad_x, float *grad_y, int B, int N, int M, int dim, float gamma,
                         float bandwidth, void *workspace, size_t workspace_bytes, void *stream);

/* Unfused x/y path: the cost ||x||^2 + ||y||^2 - 2 x.y clamped at 0 (as
 * softdtw_cuda/distances.py:6-28) is computed into `cost` (sdtw_cost_elems
 * floats, kept by the caller for the backward), then the forward DP runs on it.
 * With one row per lane the `score` buffer also marks the clamped cells (for
 * the backward's chain rule), so it differs from sdtw_forward_xy_f32's.
 * -- replaces softdtw_cuda/module.py:116-118 (pairwise_distance followed by
 *    SoftDTWAutograd.apply) for CUDA tensors */
int sdtw_forward_sqeuclid_f32(const float *x, const float *y, float *score, float *cost, float *out, int B,
                              int N, int M, int dim, float gamma, float bandwidth, void *workspace,
                              size_t workspace_bytes, void *stream);

/* Backward of sdtw_forward_sqeuclid_f32: grad_x, grad_y through the reverse DP
 * and the cost's chain rule, zero where the clamp at 0 was active.
 * -- replaces softdtw_cuda/autograd.py:33-48 followed by torch autograd of
 *    softdtw_cuda/distances.py:20-28 */
int sdtw_backward_sqeuclid_f32(const float *x, const float *y, const float *score, const float *cost,
                               const float *grad_out, float *grad_x, float *grad_y, int B, int N, int M, int dim,
                               float gamma, float bandwidth, void *workspace, size_t workspace_bytes,
                               void *stream);

/* normalize=True: the 3B problems (x_b, y_b), (x_b, x_b), (y_b, y_b), b < B,
 * read x (B,N,dim) and y (B,N,dim) in place, without concatenated copies.
 * `out` gets 3B losses in that order; score and cost are sized for 3B
 * problems of N x N (sdtw_score_elems(3B, N, N), sdtw_cost_elems(3B, N, N)).
 * The backward takes the 3B upstream gradients (NULL = ones) and writes
 * grad_x and grad_y (both required) of sum_p grad_out[p] * out[p], the self
 * pairs' two sides included.  Workspace bytes: the fused forward
 * sdtw_workspace_bytes_xy(3B, N, N, dim), the unfused forward
 * sdtw_workspace_bytes(3B, N, N), the backwards sdtw_workspace_bytes_norm(B, N, dim).
 * -- replaces softdtw_cuda/module.py:99-111 (torch.cat([x, x, y]),
 *    torch.cat([y, x, y]) and one call on the 3B pairs), with
 *    sdtw_forward_xy_f32 / sdtw_backward_xy_f32 (fused) or
 *    sdtw_forward_sqeuclid_f32 / sdtw_backward_sqeuclid_f32 (unfused) on them */
size_t sdtw_workspace_bytes_norm(int B, int N, int dim);
int sdtw_forward_xy_norm_f32(const float *x, const float *y, float *score, float *out, int B, int N, int dim,
                             float gamma, float bandwidth, void *workspace, size_t workspace_bytes, void *stream);
int sdtw_backward_xy_norm_f32(const float *x, const float *y, const float *score, const float *grad_out,
                              float *grad_x, float *grad_y, int B, int N, int dim, float gamma, float bandwidth,
                              void *workspace, size_t workspace_bytes, void *stream);
int sdtw_forward_sqeuclid_norm_f32(const float *x, const float *y, float *score, float *cost, float *out, int B,
                                   int N, int dim, float gamma, float bandwidth, void *workspace,
                                   size_t workspace_bytes, void *stream);
int sdtw_backward_sqeuclid_norm_f32(const float *x, const float *y, const float *score, const float *cost,
                                    const float *grad_out, float *grad_x, float *grad_y, int B, int N, int dim,
                                    float gamma, float bandwidth, void *workspace, size_t workspace_bytes,
                                    void *stream);

/* Chain rule of the unfused cost: given G = dL/dD (B,N,M) and the clamped cost
 * D used as the clamp mask (NULL = no mask), writes grad_x, grad_y.
 * -- replaces torch autograd of softdtw_cuda/distances.py:20-28 */
int sdtw_grad_sqeuclid_f32(const float *G, const float *D_mask, const float *x, const float *y,
                           float *grad_x, float *grad_y, int B, int N, int M, int dim, void *stream);

/* One iteration of the Soft-DTW barycenter, split at the point where the
 * multi-GPU barycenter all-reduces [gradient | loss] across ranks.
 *
 * sdtw_barycenter_grad_f32: for the barycenter bary (N,dim), the sequences
 * X (B,M,dim) and the weights w (B,), writes grad_loss (N*dim + 1 floats):
 *   grad_loss[0 : N*dim] = sum_b w[b] * d SoftDTW_gamma(bary, X[b]) / d bary,
 *   grad_loss[N*dim]     = sum_b w[b] * SoftDTW_gamma(bary, X[b]),
 * both reduced in a fixed order (bit-reproducible).  The fused (direct-form)
 * squared-Euclidean cost, no band.  Workspace: sdtw_barycenter_workspace_bytes.
 * -- replaces softdtw_cuda/barycenters.py:122-131 (expand, SoftDTW loss,
 *    weighted sum, backward)
 *
 * sdtw_barycenter_adam_f32: clips grad_loss[0:n] to 2-norm max_norm (factor
 * min(1, max_norm / (norm + 1e-6))), then one Adam step on bary (n floats)
 * with the moments exp_avg, exp_avg_sq and the learning rate
 * lr_table[*step]; records loss_hist[*step] = grad_loss[n] and
 * bary_hist[*step * n : ...] = the new bary, and increments *step (a device
 * int).  Does nothing once *step >= max_iter.  Every operand is a device
 * pointer, so the pair can be captured in a CUDA graph and replayed.
 * -- replaces softdtw_cuda/barycenters.py:134-137 (clip_grad_norm_, Adam
 *    step, cosine-annealing scheduler step) */
size_t sdtw_barycenter_workspace_bytes(int B, int N, int M, int dim);
/* Multi-GPU form of the Adam step: sums [gradient | loss] over `world` ranks
 * through exchange buffers in peer memory, then steps as
 * sdtw_barycenter_adam_f32 (one kernel per rank; replaces an all-reduce and the
 * Adam launch).  peers: device array of the `world` ranks' exchange buffers
 * (sdtw_barycenter_sync_bytes each, zeroed before first use, every one mapped
 * into this process, e.g. CUDA IPC or symmetric memory); epoch: a device u64,
 * zero before first use, advanced by one per call and equal on all ranks.
 * grad_loss (n + 1 floats, this rank's) is replaced by the sum.  Every rank
 * must make the same sequence of calls; a rank that does not arrive makes the
 * others' wait run out (status SDTW_ERR_TIMEOUT at the next call).
 * -- replaces the all-reduce of softdtw_cuda/distributed.py's sharded
 *    barycenter (no reference counterpart) and barycenters.py:134-137 */
size_t sdtw_barycenter_sync_bytes(size_t n, int world);
int sdtw_barycenter_sync_adam_f32(float *grad_loss, size_t n, const unsigned long long *peers, int world, int rank,
                                  unsigned long long *epoch, float *bary, float *exp_avg, float *exp_avg_sq,
                                  const float *lr_table, int max_iter, int *step, float *loss_hist, float *bary_hist,
                                  float beta1, float beta2, float eps, float max_norm, void *stream);
int sdtw_barycenter_grad_f32(const float *bary, const float *X, const float *w, float *grad_loss, int B, int N,
                             int M, int dim, float gamma, void *workspace, size_t workspace_bytes, void *stream);
int sdtw_barycenter_adam_f32(float *bary, float *exp_avg, float *exp_avg_sq, const float *grad_loss, size_t n,
                             const float *lr_table, int max_iter, int *step, float *loss_hist, float *bary_hist,
                             float beta1, float beta2, float eps, float max_norm, void *stream);

/* Score table <-> reference R layout (B,N+2,M+2): R[:,0,0] = 0, other borders
 * +inf, interior R = -T*gamma*ln 2.
 * -- the R tensor of softdtw_cuda/cuda/launcher.py:55-56, 177-178 */
int sdtw_score_to_R_f32(const float *score, float *R, int B, int N, int M, float gamma, void *stream);
int sdtw_R_to_score_f32(const float *R, float *score, int B, int N, int M, float gamma, void *stream);

/* Host implementation for CPU tensors (double precision, OpenMP over the
 * batch).  R is the reference layout (B,N+2,M+2); E is (B,N,M) scaled by
 * grad_out (NULL = ones).
 * -- replaces softdtw_cuda/cuda/launcher.py:307-324 and :356-361
 *    (_softdtw_forward_cpu_np, softdtw_forward_cpu) */
int sdtw_cpu_forward_f64(const double *D, double *R, double *out, int B, int N, int M, double gamma,
                         double bandwidth);
/* -- replaces softdtw_cuda/cuda/launcher.py:327-353 and :364-368
 *    (_softdtw_backward_cpu_np, softdtw_backward_cpu) */
int sdtw_cpu_backward_f64(const double *R, const double *grad_out, double *E, int B, int N, int M,
                          double gamma, double bandwidth);

/* Float64 CUDA path: the reference's float64 pipeline in double on the device
 * (one CTA per problem, a barrier per anti-diagonal; a correctness path, e.g.
 * for gradcheck on the GPU).  D, R, E device pointers; R is the reference
 * layout (B,N+2,M+2); out (B,).  Runs on `stream`, no workspace.
 * -- replaces softdtw_cuda/cuda/launcher.py:167-223 (softdtw_forward_cuda) for
 *    float64 tensors, with the arithmetic of launcher.py:307-324 */
int sdtw_forward_f64(const double *D, double *R, double *out, int B, int N, int M, double gamma,
                     double bandwidth, void *stream);
/* E (B,N,M) = grad_out[b] * dR[N,M]/dD (grad_out NULL = ones).
 * -- replaces softdtw_cuda/cuda/launcher.py:226-300 (softdtw_backward_cuda_log)
 *    for float64 tensors, with the arithmetic of launcher.py:327-353 and the
 *    scaling of softdtw_cuda/autograd.py:46-47 */
int sdtw_backward_f64(const double *D, const double *R, const double *grad_out, double *E, int B, int N, int M,
                      double gamma, double bandwidth, void *stream);
/* D (B,N,M) = sum_k (x_ik - y_jk)^2 in double (the fused cost's direct form),
 * N <= 65535.
 * -- the cost of softdtw_cuda/cuda/kernels.py:27-31 for float64 x, y */
int sdtw_cost_sqeuclid_f64(const double *x, const double *y, double *D, int B, int N, int M, int dim,
                           void *stream);

/* Chain rule of the fused cost in double: given G = dL/dD (B,N,M), writes
 * grad_x = 2 (x rowsum(G) - G y) and grad_y = 2 (y colsum(G) - G^T x)
 * (either pointer may be NULL), B <= 65535.
 * -- replaces the two bmm of softdtw_cuda/autograd_xy.py:41-49 for float64 x, y */
int sdtw_grad_sqeuclid_f64(const double *G, const double *x, const double *y, double *grad_x, double *grad_y,
                           int B, int N, int M, int dim, void *stream);

/* Allocation-free variant of sdtw_forward_f32 (no counterpart in the
 * reference).  For callers that cannot allocate device memory at call time --
 * a host runtime whose allocator owns all of device memory, a plugin boundary
 * that passes only inputs and outputs, a loop where cudaMalloc's possible
 * device synchronisation is not allowed -- it takes no workspace: its scratch
 * (band-wrap ring and the anti-diagonal copy of D) is a fixed 8 MiB device
 * array inside the library, present on every GPU that loads the library until
 * the process exits.  Problems whose scratch would exceed it are rejected with
 * SDTW_ERR_INVALID_ARGUMENT (roughly B*N*M up to 2 million cells; see
 * sdtw_workspace_bytes for the exact need).  It calls no cudaMalloc, cudaFree
 * or other allocating routine.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current; make
 * that first call before any stream capture.  All calls on a device share that
 * device's array, which keeps the previous call's contents (each call resets
 * what must start fresh): calls on one device that overlap on the GPU -- issued
 * on different streams without ordering -- race on it, so the caller must
 * order them, e.g. by issuing them on one stream.  A device-side wait of this
 * entry point that gives up records the failure in a device word inside the
 * library (it cannot use the mapped host record the other entry points
 * create); sdtw_status() reads and clears it, so call sdtw_status() after
 * synchronising the stream to learn whether the results are valid. */
int sdtw_forward_noalloc_f32(const float *D, float *score, float *out, int B, int N, int M, float gamma,
                             float bandwidth, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SDTW_B200_H */
