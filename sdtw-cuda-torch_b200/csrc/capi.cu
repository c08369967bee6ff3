// capi.cu -- the extern "C" entry points of libsdtw_b200.so (include/sdtw_b200.h).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/sdtw_b200.h"
#include "sdtw_kernels.h"

// Device-side "some wait failed" flag, one per device that loads the library.
__device__ int g_abort_flag;

namespace {

using namespace sdtw;

thread_local std::string g_last_error;
std::atomic<uint32_t> g_seq{1};
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
std::atomic<int> g_debug_stall{-1};
std::atomic<int> g_wpc_override{0};
std::atomic<int> g_cs_override{0};
std::atomic<int> g_k_override{0};
std::mutex g_init_mu;
int* g_status_host = nullptr;    // mapped pinned words: [0] status, [8..15] WaitDiag
int* g_status_dev = nullptr;     // their device address
int g_num_sms[64] = {0};

// Optional per-kernel timing (sdtw_timing_enable): CUDA events recorded on the
// launching stream around each kernel.
std::atomic<int> g_timing{0};
std::mutex g_timing_mu;
struct PendingEv {
    const char* name;
    cudaEvent_t e0, e1;
};
std::vector<PendingEv> g_pending;
std::vector<cudaEvent_t> g_ev_pool;
std::map<std::string, std::pair<double, long>> g_totals;

cudaEvent_t pool_event() {
    if (!g_ev_pool.empty()) {
        cudaEvent_t e = g_ev_pool.back();
        g_ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Kernels launched by the library since load (every launch site counts its
// kernels here).
std::atomic<unsigned long long> g_launches{0};

struct KernelTimer {
    const char* name;
    cudaStream_t st;
    cudaEvent_t e0 = nullptr;
    KernelTimer(const char* n, cudaStream_t s, int kernels = 1) : name(n), st(s) {
        g_launches.fetch_add(static_cast<unsigned long long>(kernels));
        // No timing events inside a stream capture (a CUDA graph): they would
        // be recorded at every replay, not now.
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (g_timing.load() && cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone) {
            std::lock_guard<std::mutex> lk(g_timing_mu);
            e0 = pool_event();
            cudaEventRecord(e0, st);
        }
    }
    ~KernelTimer() {
        if (e0) {
            std::lock_guard<std::mutex> lk(g_timing_mu);
            cudaEvent_t e1 = pool_event();
            cudaEventRecord(e1, st);
            g_pending.push_back({name, e0, e1});
        }
    }
};

constexpr float kLog2e = 1.4426950408889634f;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(SDTW_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

int ensure_status() {
    if (g_status_dev) return SDTW_OK;
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_status_dev) return SDTW_OK;
    int* h = nullptr;
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&h), 16 * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(status)");
    std::memset(h, 0, 16 * sizeof(int));
    int* d = nullptr;
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostGetDevicePointer(status)");
    g_status_host = h;
    g_status_dev = d;
    return SDTW_OK;
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (g_num_sms[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev] = n;
    }
    return g_num_sms[dev];
}

int* abort_flag_dev() {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_abort_flag) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

// Clears the status word and the current device's abort flag.
void clear_status() {
    *reinterpret_cast<volatile int*>(g_status_host) = 0;
    const int zero = 0;
    cudaMemcpyToSymbol(g_abort_flag, &zero, sizeof(int));
}

// Diagnostics of a failed wait: d points at a WaitDiag record (8 ints).
std::string diag_text_of(const volatile int* d) {
    char buf[256];
    std::snprintf(buf, sizeof buf,
                  "%s pass, %s wait, problem %d, warp %d, band %d: expected %d, last seen %d",
                  d[0] == 1 ? "forward"
                            : (d[0] == 2 ? "backward"
                                         : (d[0] == 5 ? "tensor-core gradient"
                                                      : (d[0] == 6 ? "tensor-core cost"
                                                                   : (d[0] == 7 ? "barycenter exchange" : "?")))),
                  d[1] == 1 ? "shared-memory ring"
                            : (d[1] == 2 ? "global ring"
                                         : (d[1] == 3 ? "flow-control"
                                                      : (d[1] == 4 ? "MMA completion"
                                                                   : (d[1] == 5 ? "aborted (another wait failed)"
                                                                                : (d[1] == 6 ? "value range"
                                                                                             : (d[1] == 7 ? "peer flag" : "?")))))),
                  d[2], d[3], d[4], d[5], d[6]);
    return buf;
}
std::string diag_text() { return diag_text_of(g_status_host + 8); }

// Text of a nonzero device status (the wait diagnostics `why` for a timeout).
std::string status_text(int s, const std::string& why) {
    if (s == kStatusRange)
        return "the forward's scores left the representable range: |R| / gamma must stay below 3.7e8 and "
               "|cost| * log2(e) / gamma below 4.2e6 per cell, and no cost may be NaN (use float64 inputs "
               "for larger ranges)";
    return "a device-side wait timed out (" + why + ")";
}
int status_code(int s) { return s == kStatusRange ? SDTW_ERR_RANGE : SDTW_ERR_TIMEOUT; }

// A failure recorded by an earlier launch surfaces at the next call.
int pending_status() {
    if (g_status_host) {
        int s = *reinterpret_cast<volatile int*>(g_status_host);
        if (s != 0) {
            std::string why = diag_text();
            clear_status();
            return fail(status_code(s), "an earlier launch failed: " + status_text(s, why));
        }
    }
    return SDTW_OK;
}

int check_dims(int B, int N, int M) {
    if (B <= 0 || N <= 0 || M <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "B, N and M must be > 0");
    if ((long long)N + 64 >= (1ll << 30) || (long long)M + 64 >= (1ll << 30))
        return fail(SDTW_ERR_INVALID_ARGUMENT, "sequence length too large");
    return SDTW_OK;
}

int check_gamma(float gamma) {
    if (!(gamma > 0.f) || !std::isfinite(gamma)) return fail(SDTW_ERR_INVALID_ARGUMENT, "gamma must be finite and > 0");
    return SDTW_OK;
}

WaitCtx wait_ctx() {
    WaitCtx w{};
    w.status = g_status_dev;
    w.diag = g_status_dev ? reinterpret_cast<volatile WaitDiag*>(g_status_dev + 8) : nullptr;
    w.abort_flag = abort_flag_dev();
    w.timeout_ns = g_timeout_ns.load();
    return w;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// |i - j| > bw  <=>  |i - j| > floor(bw) for integer |i - j| (launcher.py:315, :345).
int int_band(float bw) {
    if (!(bw > 0.f)) return 1 << 29;
    const double f = std::floor(static_cast<double>(bw));
    return f >= static_cast<double>(1 << 29) ? (1 << 29) : static_cast<int>(f);
}

// Resident clusters per geometry, cached per device (the occupancy query is a
// host call; the plan is computed at every launch).
int cached_cluster_fit(const WavePlan& p, int pass) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    const auto key = std::make_tuple(dev * 128 + pass, p.K, p.wpc, p.csize);
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    const int n = max_active_clusters(p, pass);
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = n;
    return n;
}

// Estimated duration (cycles) of the wavefront launches of a geometry with
// one row per lane.  The resident clusters run in waves; within a wave the
// stripes enter the pipeline kLagSteps anti-diagonal steps apart and each warp
// runs its n_bands stripes back to back, so a wave takes
//   max(n_bands * (M + 31) + (G - 1) * lag, (n_stripes - 1) * lag + M + 31)
// steps.  A step costs about kStepLatency cycles while a warp has its SM
// sub-partition to itself and about kStepPerWarp cycles per warp beyond that
// (issue-bound), for the busiest SM of the wave.  Fitted on B200 to the forward
// and reverse passes at B x N x M = 32 x 512^2, 16 x 4096^2, 192 x 1024^2 and
// 4096 x 100^2 under every geometry the plan can take.
double plan_cost(const WavePlan& q, int B, int M, int fit, int sms) {
    constexpr double kLagSteps = 40, kStepLatency = 350, kStepPerWarp = 100;
    if (fit <= 0) return 1e300;
    const int waves = (B + fit - 1) / fit;
    const int clusters = B < fit ? B : fit;
    const long long ctas = static_cast<long long>(clusters) * q.csize;
    const double per_sm = static_cast<double>((ctas + sms - 1) / sms);
    const double w = per_sm * q.wpc / 4.0;  // warps per SM sub-partition
    const double step = std::max(kStepLatency, kStepPerWarp * w);
    const double row = M + 31.0;
    const double steps = std::max(q.n_bands * row + (q.G - 1) * kLagSteps, (q.n_stripes - 1) * kLagSteps + row);
    return waves * steps * step;
}

// Launch geometry of a pass (0 forward, 1 reverse; each pass has its own
// kernels and occupancy, and the table layout depends only on the rows per
// lane, which both passes share).  make_plan's choice unless its clusters do not all fit on
// the GPU at once (a second wave would double the time): then the candidate
// with fewer waves, then fewer bands.  With one row per lane, the geometry of
// plan_cost's minimum replaces that choice when it is estimated at least 15 %
// faster.
WavePlan plan(int B, int N, int M, int pass) {
    const int wo = g_wpc_override.load(), co = g_cs_override.load(), ko = g_k_override.load();
    const int sms = num_sms();
    const WavePlan p = make_plan(B, N, M, sms, wo, co, ko);
    if (wo > 0 || co > 0) return p;
    WavePlan base = p;
    const int fit = cached_cluster_fit(p, pass);
    if (fit > 0 && B > fit) {
        auto waves = [&](int f) { return f > 0 ? (B + f - 1) / f : 1 << 30; };
        int best_w = waves(fit);
        for (int cs = 8; cs >= 1; cs /= 2) {
            if (cs == p.csize) continue;
            const WavePlan q = make_plan(B, N, M, sms, 0, cs, ko);
            const int w = waves(cached_cluster_fit(q, pass));
            if (w < best_w || (w == best_w && q.n_bands < base.n_bands)) {
                base = q;
                best_w = w;
            }
        }
    }
    if (p.K != 1) return base;
    const double base_c = plan_cost(base, B, M, cached_cluster_fit(base, pass), sms);
    WavePlan best = base;
    double best_c = base_c;
    for (int cs = 1; cs <= 8; cs *= 2)
        for (int wpc = 2; wpc <= wpc_max(1); wpc *= 2) {
            const WavePlan q = make_plan(B, N, M, sms, wpc, cs, ko);
            if (q.wpc != wpc || q.csize != cs) continue;
            if ((wpc / 2) * cs >= q.n_stripes) continue;  // half the warps would still hold every stripe
            const double c = plan_cost(q, B, M, cached_cluster_fit(q, pass), sms);
            if (c < best_c) {
                best = q;
                best_c = c;
            }
        }
    return best_c <= 0.85 * base_c ? best : base;
}

// Workspace layouts (each region 256-byte aligned):
//   D-input forward/backward : [wrap ring][WL table]
//   x/y forward              : [wrap ring][WL cost]
//   x/y backward, sqeuclid bwd: [wrap ring][WL E][gradient operands]
//     grad_small (one row per lane, dim <= 16): per-split column sums;
//     grad_wl (one row per lane, N or M above 128): x, y in the chunked
//     transposed layout (B, ceil(N/32), dim, 36) and (B, ceil(M/32), dim, 36);
//     grad_rm (otherwise): G, G^T, x^T, y^T row-major, rows padded to a
//     multiple of 32 floats
// The band-wrap ring (needed when a pass's plan has more than one band; its
// size does not depend on the plan) of the D-input passes, and of the x/y
// passes (whose forward may compute its costs from x and y: plan 2 + dp).
// The ring is sized whenever the problem has more than one stripe: every pass
// and launch picks its own plan (forward, reverse pass, their variants), and
// any of them may split the stripes into bands.
size_t wave_ws(int B, int N, int M) {
    const int K = rows_per_lane(N, g_k_override.load());
    const int stripes = (N + 32 * K - 1) / (32 * K);
    return stripes > 1 ? align_up(static_cast<size_t>(B) * M * 16u, 256) : 0;
}
size_t wave_ws_xy(int B, int N, int M, int dim) {
    (void)dim;
    return wave_ws(B, N, M);
}
size_t wl_bytes(int B, int N, int M) { return align_up(wl_cells(B, N, M, g_k_override.load()) * sizeof(float), 256); }
size_t pad32(int n) { return (static_cast<size_t>(n) + 31) & ~static_cast<size_t>(31); }
// The gradient from the wavefront layout (grad_wl, one row per lane) or from
// row-major operands (grad_rm): the latter for more rows per lane, and for
// problems of at most one 128-row tile each way, where each grad_wl CTA runs
// a single tile and its warp-specialised pipeline never fills.
bool grad_rm_path(int N, int M) {
    return rows_per_lane(N, g_k_override.load()) != 1 || (N <= 128 && M <= 128);
}
struct GradOperands {
    size_t g, gt, xt, yt, total;  // byte offsets from the start of the region
};
GradOperands grad_operands(int B, int N, int M, int dim) {
    GradOperands o;
    const size_t b = static_cast<size_t>(B);
    const WavePlan p = plan(B, N, M, 0);
    if (grad_small_supported(p, dim)) {  // per-split column sums of grad_small
        o.g = o.gt = o.xt = o.yt = 0;
        o.total = align_up(grad_small_part_bytes(p, dim), 256);
        return o;
    }
    if (!grad_rm_path(N, M)) {  // xTc, yTc: rows of 36 floats per 32 positions
        o.g = o.gt = 0;
        o.xt = 0;
        o.yt = align_up(b * (pad32(N) / 32) * dim * 36 * sizeof(float), 256);
        o.total = o.yt + align_up(b * (pad32(M) / 32) * dim * 36 * sizeof(float), 256);
        return o;
    }
    o.g = 0;
    o.gt = o.g + align_up(b * N * pad32(M) * sizeof(float), 256);
    o.xt = o.gt + align_up(b * M * pad32(N) * sizeof(float), 256);
    o.yt = o.xt + align_up(b * dim * pad32(N) * sizeof(float), 256);
    o.total = o.yt + align_up(b * dim * pad32(M) * sizeof(float), 256);
    return o;
}

// weights: the table keeps each cell's predecessor weights (the state of the
// x/y pairs' backward, one row per lane) instead of its score.
bool weight_store(int B, int N, int M) { return plan(B, N, M, 0).K == 1; }

// A launch with more than one band hands rows between bands through a ring in
// the workspace, checked by tags that carry the launch's sequence number.  The
// ring is reset before every such launch, so that a launch replayed from a
// CUDA graph (same sequence number, same workspace) never meets a previous
// replay's entries.
cudaError_t reset_wrap(const WavePlan& P, uint64_t* wrap, cudaStream_t stream) {
    if (P.n_bands <= 1) return cudaSuccess;
    return cudaMemsetAsync(wrap, 0xff, wrap_bytes(P), stream);
}

// Dw: the cost table, or null with x, y, dim, dp (> 0) for the fused costs.
int run_forward(const float* Dw, float* score, float* out, int B, int N, int M, float gamma, float bw,
                uint64_t* wrap, cudaStream_t stream, bool weights = false, const WaitCtx* wait = nullptr,
                SeqIn x = one_seq<const float>(nullptr), SeqIn y = one_seq<const float>(nullptr), int dim = 0,
                int dp = 0, bool x_shared = false, bool clamp_mask = false) {
    FwdArgs a{};
    const int pass = dp ? 2 + dp : 0;
    a.P = plan(B, N, M, pass);
    // The 128-register forward when all of the launch's clusters fit at once
    // at its occupancy (K = 1 only).
    if (a.P.K == 1 && dp < 8) {
        const WavePlan pw = plan(B, N, M, 32 + pass);
        if (cached_cluster_fit(pw, 32 + pass) >= B) {
            a.P = pw;
            a.wide = 1;
        }
    }
    a.x = x;
    a.x_bstride = x_shared ? 0 : static_cast<size_t>(N) * dim;
    a.clamp_mask = (clamp_mask && weights) ? 1 : 0;
    a.y = y;
    a.dim = dim;
    a.dp = dp;
    a.weights = weights ? 1 : 0;
    a.Dw = Dw;
    a.score = reinterpret_cast<float2*>(score);
    a.out = out;
    a.wrap = wrap;
    a.kk = kLog2e / gamma;
    a.inv_k = static_cast<float>(1.0 / static_cast<double>(a.kk));
    a.inv_k_d = static_cast<double>(gamma) * 0.6931471805599453;
    a.bw = bw > 0.f ? bw : -1.f;
    a.ibw = int_band(bw);
    a.seq = g_seq.fetch_add(1);
    a.debug_stall = g_debug_stall.load();
    a.wait = wait ? *wait : wait_ctx();
    cudaError_t e = reset_wrap(a.P, wrap, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(band-wrap ring)");
    {
        KernelTimer kt("wavefront_fwd", stream);
        e = launch_forward(a, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "forward launch");
    return SDTW_OK;
}

int run_backward(const float* score, const float* grad_out, float* Ew, int B, int N, int M, float bw,
                 uint64_t* wrap, cudaStream_t stream, bool weights = false, bool clamp_mask = false) {
    BwdArgs a{};
    a.P = plan(B, N, M, 1);
    a.weights = weights ? 1 : 0;
    a.clamp_mask = (weights && clamp_mask) ? 1 : 0;
    a.score = reinterpret_cast<const float2*>(score);
    a.grad_out = grad_out;
    a.Ew = Ew;
    a.wrap = wrap;
    a.bw = bw > 0.f ? bw : -1.f;
    a.ibw = int_band(bw);
    a.seq = g_seq.fetch_add(1);
    a.debug_stall = g_debug_stall.load();
    a.wait = wait_ctx();
    cudaError_t e = reset_wrap(a.P, wrap, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(band-wrap ring)");
    {
        KernelTimer kt("wavefront_bwd", stream);
        e = launch_backward(a, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
    return SDTW_OK;
}

// The reverse pass that applies the squared-Euclidean chain rule for grad_x
// itself (no E table), see bwdw_kernel.
int run_backward_grad(const float* score, const float* grad_out, int B, int N, int M, uint64_t* wrap,
                      cudaStream_t stream, const float* x, size_t x_bstride, const float* y, int dim, int gd, float* gx,
                      bool pdl = false) {
    BwdArgs a{};
    a.P = plan(B, N, M, 64 + gd);
    a.weights = 1;
    a.score = reinterpret_cast<const float2*>(score);
    a.grad_out = grad_out;
    a.wrap = wrap;
    a.bw = -1.f;
    a.ibw = int_band(0.f);
    a.seq = g_seq.fetch_add(1);
    a.debug_stall = g_debug_stall.load();
    a.wait = wait_ctx();
    a.x = x;
    a.y = y;
    a.dim = dim;
    a.gd = gd;
    a.x_bstride = x_bstride;
    a.gx = gx;
    a.pdl = (pdl && a.P.n_bands <= 1) ? 1 : 0;  // a multi-band launch follows its ring reset
    cudaError_t e = reset_wrap(a.P, wrap, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(band-wrap ring)");
    {
        KernelTimer kt("wavefront_bwd", stream);
        e = launch_backward(a, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
    return SDTW_OK;
}

int check_common(int B, int N, int M, float gamma) {
    int rc;
    if ((rc = check_dims(B, N, M)) || (rc = check_gamma(gamma))) return rc;
    if ((rc = ensure_status()) || (rc = pending_status())) return rc;
    return SDTW_OK;
}

int check_ws(void* ws, size_t have, size_t need) {
    if (have < need) return fail(SDTW_ERR_INVALID_ARGUMENT, "workspace too small");
    if (need && !ws) return fail(SDTW_ERR_INVALID_ARGUMENT, "null workspace");
    if (reinterpret_cast<uintptr_t>(ws) % 256u) return fail(SDTW_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    return SDTW_OK;
}

int check_score(const float* score) {
    if (!score) return fail(SDTW_ERR_INVALID_ARGUMENT, "null score");
    // The forward writes it with bulk copies of whole anti-diagonal rows.
    if (reinterpret_cast<uintptr_t>(score) % 16u) return fail(SDTW_ERR_INVALID_ARGUMENT, "score must be 16-byte aligned");
    return SDTW_OK;
}

}  // namespace

// ----------------------------------------------------------------------------
// Allocation-free forward.
//
// Some callers cannot allocate device memory when they call us: a host runtime
// whose allocator owns all of device memory and lends out no scratch, a plugin
// boundary that hands over only input and output buffers, or a latency-critical
// loop in which cudaMalloc (which can synchronise the device) is not allowed.
// For them the D-input forward has a variant whose scratch (band-wrap ring and
// the anti-diagonal copy of D) lives in a fixed device array compiled into the
// library.  Every GPU that loads the library holds this array until the process
// exits.  The caller still passes D, score and out.
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Status word ([0]) and the failed wait's diagnostics ([8..15], a WaitDiag) of
// the launches of the allocation-free forward: device memory, since that entry
// point may not create the mapped host status record the others use.
static __device__ int g_noalloc_status[16];
static std::atomic<unsigned long long> g_noalloc_used{0};  // bit d: device d ran it

// Host code cannot use a __device__ array's name as a device address; look the
// addresses up with the device current.  Done at every call (it allocates
// nothing), so an address is never kept past a device reset.
static int noalloc_addrs(int* dev, void** scratch, int** status) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= 64) return fail(SDTW_ERR_INVALID_ARGUMENT, "device index out of range");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    void* q = nullptr;
    e = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (e != cudaSuccess || !q) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc status)");
    *scratch = p;
    *status = static_cast<int*>(q);
    return SDTW_OK;
}

// Status of the allocation-free forward on the current device: its device
// word, read and cleared; 0 if that entry point never ran here.
static int noalloc_take_status(std::string* why) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    if (!(g_noalloc_used.load() & (1ull << dev))) return 0;
    int rec[16] = {0};
    // A synchronous copy: sdtw_status is called after the caller synchronised.
    if (cudaMemcpyFromSymbol(rec, g_noalloc_status, sizeof rec) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (rec[0] == 0) return 0;
    *why = diag_text_of(rec + 8);
    const int zero[16] = {0};
    cudaMemcpyToSymbol(g_noalloc_status, zero, sizeof zero);
    const int z = 0;
    cudaMemcpyToSymbol(g_abort_flag, &z, sizeof(int));
    return rec[0];
}

extern "C" {

const char* sdtw_version(void) { return "sdtw-b200 0.1.0 (sm_100a)"; }

const char* sdtw_error_string(int code) {
    switch (code) {
        case SDTW_OK: return "ok";
        case SDTW_ERR_INVALID_ARGUMENT: return "invalid argument";
        case SDTW_ERR_CUDA: return "CUDA runtime error";
        case SDTW_ERR_TIMEOUT: return "device-side wait timed out";
        case SDTW_ERR_RANGE: return "value range exceeded";
        default: return "unknown error";
    }
}

const char* sdtw_last_error_message(void) { return g_last_error.c_str(); }

int sdtw_status(void) {
    int s = g_status_host ? *reinterpret_cast<volatile int*>(g_status_host) : 0;
    if (s != 0) {
        g_last_error = status_text(s, diag_text());
        clear_status();
    }
    // The allocation-free forward records its failures in a device word.
    std::string why;
    const int s2 = noalloc_take_status(&why);
    if (s2 != 0 && s == 0) {
        g_last_error = "allocation-free forward: " + status_text(s2, why);
        s = s2;
    }
    return s;
}

void sdtw_set_plan_override(int warps_per_cta, int cluster_size, int rows_per_lane) {
    g_wpc_override.store(warps_per_cta > 0 ? warps_per_cta : 0);
    g_cs_override.store(cluster_size > 0 ? cluster_size : 0);
    g_k_override.store(rows_per_lane == 1 || rows_per_lane == 2 || rows_per_lane == 4 ? rows_per_lane : 0);
}

void sdtw_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : 1ull); }

void sdtw_timing_enable(int on) {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    g_timing.store(on ? 1 : 0);
    g_totals.clear();
}

int sdtw_timing_read(char* names, size_t names_len, double* total_ms, long* counts, int max_entries) {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    for (const PendingEv& p : g_pending) {
        float ms = 0.f;
        if (cudaEventSynchronize(p.e1) == cudaSuccess && cudaEventElapsedTime(&ms, p.e0, p.e1) == cudaSuccess) {
            auto& t = g_totals[p.name];
            t.first += ms;
            t.second += 1;
        }
        cudaGetLastError();
        g_ev_pool.push_back(p.e0);
        g_ev_pool.push_back(p.e1);
    }
    g_pending.clear();
    int n = 0;
    std::string joined;
    for (const auto& kv : g_totals) {
        if (n >= max_entries) break;
        if (total_ms) total_ms[n] = kv.second.first;
        if (counts) counts[n] = kv.second.second;
        if (n) joined += ",";
        joined += kv.first;
        ++n;
    }
    if (names && names_len) {
        std::strncpy(names, joined.c_str(), names_len - 1);
        names[names_len - 1] = '\0';
    }
    return n;
}

void sdtw_debug_stall_stripe(int stripe) { g_debug_stall.store(stripe); }

unsigned long long sdtw_launch_count(void) { return g_launches.load(); }

int sdtw_plan_info(int B, int N, int M, int* info) {
    if (!info) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    const WavePlan p = plan(B, N, M, 0);
    info[0] = p.K;
    info[1] = p.wpc;
    info[2] = p.csize;
    info[3] = p.n_bands;
    info[4] = p.n_stripes;
    info[5] = cached_cluster_fit(p, 0);
    return SDTW_OK;
}

size_t sdtw_score_elems(int B, int N, int M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return score_elems(B, N, M, g_k_override.load());
}

size_t sdtw_cost_elems(int B, int N, int M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return wl_cells(B, N, M, g_k_override.load());
}

size_t sdtw_workspace_bytes(int B, int N, int M) {
    if (B <= 0 || N <= 0 || M <= 0) return 0;
    return wave_ws(B, N, M) + wl_bytes(B, N, M);
}

size_t sdtw_workspace_bytes_xy(int B, int N, int M, int dim) {
    if (B <= 0 || N <= 0 || M <= 0 || dim <= 0) return 0;
    return wave_ws_xy(B, N, M, dim) + wl_bytes(B, N, M) + grad_operands(B, N, M, dim).total;
}

static int check_f64(int B, int N, int M, double gamma) {
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    if (!(gamma > 0.0) || !std::isfinite(gamma)) return fail(SDTW_ERR_INVALID_ARGUMENT, "gamma must be finite and > 0");
    return SDTW_OK;
}

int sdtw_forward_f64(const double* D, double* R, double* out, int B, int N, int M, double gamma, double bandwidth,
                     void* stream) {
    int rc = check_f64(B, N, M, gamma);
    if (rc) return rc;
    if (!D || !R || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    {
        KernelTimer kt("wavefront_fwd_f64", static_cast<cudaStream_t>(stream));
        e = launch_forward_f64(D, R, out, B, N, M, gamma, bandwidth > 0.0 ? bandwidth : -1.0,
                               static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "forward launch");
    return SDTW_OK;
}

int sdtw_backward_f64(const double* D, const double* R, const double* grad_out, double* E, int B, int N, int M,
                      double gamma, double bandwidth, void* stream) {
    int rc = check_f64(B, N, M, gamma);
    if (rc) return rc;
    if (!D || !R || !E) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    {
        KernelTimer kt("wavefront_bwd_f64", static_cast<cudaStream_t>(stream));
        e = launch_backward_f64(D, R, grad_out, E, B, N, M, gamma, bandwidth > 0.0 ? bandwidth : -1.0,
                                static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
    return SDTW_OK;
}

int sdtw_grad_sqeuclid_f64(const double* G, const double* x, const double* y, double* grad_x, double* grad_y, int B,
                           int N, int M, int dim, void* stream) {
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!G || !x || !y) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    {
        KernelTimer kt("grad_f64", static_cast<cudaStream_t>(stream), (grad_x ? 1 : 0) + (grad_y ? 1 : 0));
        e = launch_grad_f64(G, x, y, grad_x, grad_y, B, N, M, dim, static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "grad launch");
    return SDTW_OK;
}

int sdtw_cost_sqeuclid_f64(const double* x, const double* y, double* D, int B, int N, int M, int dim, void* stream) {
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (N > 65535 || B > 65535) return fail(SDTW_ERR_INVALID_ARGUMENT, "float64 cost: N and B must be <= 65535");
    if (!x || !y || !D) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    {
        KernelTimer kt("cost_f64", static_cast<cudaStream_t>(stream));
        e = launch_cost_f64(x, y, D, B, N, M, dim, static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "cost launch");
    return SDTW_OK;
}

int sdtw_cost_sqeuclid_f32(const float* x, const float* y, float* D, int B, int N, int M, int dim, int direct,
                           void* stream) {
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y || !D) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    if (!direct && cost_tc_supported(one_seq(x), one_seq(y), dim)) {
        // The expanded cost with its dot products on the tensor cores.
        if ((rc = ensure_status()) || (rc = pending_status())) return rc;
        KernelTimer kt("cost_rowmajor", static_cast<cudaStream_t>(stream));
        e = launch_cost_tc_rm(x, y, D, B, N, M, dim, wait_ctx(), static_cast<cudaStream_t>(stream));
    } else {
        KernelTimer kt("cost_rowmajor", static_cast<cudaStream_t>(stream));
        e = launch_cost(x, y, D, B, N, M, dim, direct != 0, static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "cost launch");
    return SDTW_OK;
}

int sdtw_forward_f32(const float* D, float* score, float* out, int B, int N, int M, float gamma, float bandwidth,
                     void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (!D || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t w0 = wave_ws(B, N, M);
    if ((rc = check_ws(workspace, workspace_bytes, w0 + wl_bytes(B, N, M)))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* Dw = reinterpret_cast<float*>(static_cast<char*>(workspace) + w0);
    const WavePlan p = plan(B, N, M, 0);
    cudaError_t e;
    {
        KernelTimer kt("rm_to_wl", st);
        e = launch_rm_to_wl(D, Dw, p, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "layout launch");
    return run_forward(Dw, score, out, B, N, M, gamma, bandwidth, static_cast<uint64_t*>(workspace), st);
}

int sdtw_backward_f32(const float* score, const float* grad_out, float* E, int B, int N, int M, float gamma,
                      float bandwidth, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (!E) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t w0 = wave_ws(B, N, M);
    if ((rc = check_ws(workspace, workspace_bytes, w0 + wl_bytes(B, N, M)))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* Ew = reinterpret_cast<float*>(static_cast<char*>(workspace) + w0);
    rc = run_backward(score, grad_out, Ew, B, N, M, bandwidth, static_cast<uint64_t*>(workspace), st);
    if (rc) return rc;
    cudaError_t e;
    {
        KernelTimer kt("wl_to_rm", st);
        e = launch_wl_to_rm(Ew, nullptr, E, plan(B, N, M, 0), st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "layout launch");
    return SDTW_OK;
}

// The fused forward over B problems whose sequences x, y name (one batch, or
// the normalized triple); the caller has checked the arguments.
static int forward_xy_common(const SeqIn& x, const SeqIn& y, float* score, float* out, int B, int N, int M, int dim,
                      float gamma, float bandwidth, void* workspace, cudaStream_t st) {
    const size_t w0 = wave_ws_xy(B, N, M, dim);
    // Up to 16 features: the costs are computed inside the forward from x and
    // y (no cost table); more features: a cost table first (see fused_dp).
    const int dp = weight_store(B, N, M) ? fused_dp(dim, x, y) : 0;
    if (dp)
        return run_forward(nullptr, score, out, B, N, M, gamma, bandwidth, static_cast<uint64_t*>(workspace), st, true,
                           nullptr, x, y, dim, dp);
    float* Dw = reinterpret_cast<float*>(static_cast<char*>(workspace) + w0);
    cudaError_t e;
    {
        KernelTimer kt("cost_wl", st);
        e = launch_cost_wl(x, y, Dw, plan(B, N, M, 0), dim, true, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "cost launch");
    return run_forward(Dw, score, out, B, N, M, gamma, bandwidth, static_cast<uint64_t*>(workspace), st,
                       weight_store(B, N, M));
}

int sdtw_forward_xy_f32(const float* x, const float* y, float* score, float* out, int B, int N, int M, int dim,
                        float gamma, float bandwidth, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if ((rc = check_ws(workspace, workspace_bytes, wave_ws_xy(B, N, M, dim) + wl_bytes(B, N, M)))) return rc;
    return forward_xy_common(one_seq(x), one_seq(y), score, out, B, N, M, dim, gamma, bandwidth, workspace,
                             static_cast<cudaStream_t>(stream));
}

// Backward through the x/y chain rule; mask_w (WL cost) applies the clamp mask
// of the unfused cost, or is null for the fused cost.
// marked: the shares carry the unfused forward's clamp marks (share store).
static int backward_xy_common(const SeqIn& x, const SeqIn& y, const float* score, const float* mask_w, bool marked,
                              const float* grad_out, const SeqOut& gxs, const SeqOut& gys, int B, int N, int M, int dim,
                              float bandwidth, void* workspace, cudaStream_t st) {
    const size_t w0 = wave_ws_xy(B, N, M, dim);
    float* Ew = reinterpret_cast<float*>(static_cast<char*>(workspace) + w0);
    const bool grad_x = !gxs.null(), grad_y = !gys.null();
    // Only grad_x of one batch, fused cost, up to 16 features, no band: the
    // reverse pass applies the chain rule as it goes and E never reaches memory.
    const int gd = (!mask_w && grad_x && !grad_y && x.per >= B && weight_store(B, N, M) &&
                    int_band(bandwidth) >= N + M)
                       ? grad_fused_gd(dim, y.p[0])
                       : 0;
    if (gd)
        return run_backward_grad(score, grad_out, B, N, M, static_cast<uint64_t*>(workspace), st, x.p[0],
                                 static_cast<size_t>(N) * dim, y.p[0], dim, gd, gxs.p[0]);
    int rc = run_backward(score, grad_out, Ew, B, N, M, bandwidth, static_cast<uint64_t*>(workspace), st,
                          weight_store(B, N, M), marked);
    if (rc) return rc;
    if (!grad_x && !grad_y) return SDTW_OK;
    GradTcArgs g{};
    g.P = plan(B, N, M, 0);
    g.Ew = Ew;
    g.Mw = mask_w;
    g.x = x;
    g.y = y;
    g.gx = gxs;
    g.gy = gys;
    g.dim = dim;
    g.tiles_x = grad_x ? (N + 127) / 128 : 0;
    g.tiles_y = grad_y ? (M + 127) / 128 : 0;
    g.wait = wait_ctx();
    cudaError_t e;
    char* region = static_cast<char*>(workspace) + w0 + wl_bytes(B, N, M);
    const GradOperands o = grad_operands(B, N, M, dim);
    if (grad_small_supported(g.P, dim)) {
        // Few features: the contraction on the FP32 pipes, one read of E.
        KernelTimer kt("grad_xy", st, grad_y ? 2 : 1);
        e = launch_grad_small(Ew, mask_w, x, y, gxs, gys, reinterpret_cast<float*>(region), g.P, dim, st,
                              static_cast<size_t>(N) * dim);
        if (e != cudaSuccess) return cuda_fail(e, "grad launch");
        return SDTW_OK;
    }
    if (!grad_rm_path(N, M)) {
        if ((reinterpret_cast<uintptr_t>(mask_w) & 15u) != 0)
            return fail(SDTW_ERR_INVALID_ARGUMENT, "cost table must be 16-byte aligned");
        // G straight from the wavefront layout; x, y in the chunked transposed layout.
        float* xTc = reinterpret_cast<float*>(region + o.xt);
        float* yTc = reinterpret_cast<float*>(region + o.yt);
        {
            KernelTimer kt("grad_operands", st);
            const SeqIn none = one_seq<const float>(nullptr);
            e = launch_transpose_chunked(grad_y ? x : none, xTc, N, grad_x ? y : none, yTc, M, B, dim, st);
        }
        if (e != cudaSuccess) return cuda_fail(e, "layout launch");
        g.xTc = xTc;
        g.yTc = yTc;
        grad_wl_geometry(dim, mask_w != nullptr, &g);
        {
            KernelTimer kt("grad_xy", st);
            e = launch_grad_wl(g, st);
        }
        if (e != cudaSuccess) return cuda_fail(e, "grad launch");
        return SDTW_OK;
    }
    // More rows per lane: operands in row-major layouts (mask applied to G),
    // then the tensor-core contractions with 16-byte operand copies.
    float* G = reinterpret_cast<float*>(region + o.g);
    float* GT = reinterpret_cast<float*>(region + o.gt);
    float* xT = reinterpret_cast<float*>(region + o.xt);
    float* yT = reinterpret_cast<float*>(region + o.yt);
    const int Np = static_cast<int>(pad32(N)), Mp = static_cast<int>(pad32(M));
    {
        KernelTimer kt("grad_operands", st, 1 + (grad_x ? 1 : 0) + (grad_y ? 1 : 0));
        e = launch_wl_to_rm_cm(Ew, mask_w, grad_x ? G : nullptr, Mp, grad_y ? GT : nullptr, Np, g.P, st);
        if (e == cudaSuccess && grad_x) e = launch_transpose_brc(y, yT, B, M, dim, Mp, st);
        if (e == cudaSuccess && grad_y) e = launch_transpose_brc(x, xT, B, N, dim, Np, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "layout launch");
    g.G = G;
    g.GT = GT;
    g.xT = xT;
    g.yT = yT;
    grad_rm_geometry(dim, &g.fb, &g.nt, &g.n_fblk, &g.tmem_cols, &g.stages);
    {
        KernelTimer kt("grad_xy", st);
        e = launch_grad_rm(g, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "grad launch");
    return SDTW_OK;
}

int sdtw_backward_xy_f32(const float* x, const float* y, const float* score, const float* grad_out, float* grad_x,
                         float* grad_y, int B, int N, int M, int dim, float gamma, float bandwidth, void* workspace,
                         size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if ((rc = check_ws(workspace, workspace_bytes, sdtw_workspace_bytes_xy(B, N, M, dim)))) return rc;
    return backward_xy_common(one_seq(x), one_seq(y), score, nullptr, false, grad_out, one_seq(grad_x), one_seq(grad_y),
                              B, N, M, dim, bandwidth, workspace, static_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------------------------------
// Barycenter iteration (barycenters.py:122-137 of the reference): the weighted
// loss and its gradient with respect to the barycenter, and the clipped Adam
// step.  Workspace: the x/y workspace, then the shares table, the broadcast
// barycenter (used when the forward cannot read one x for every problem), the
// per-problem gradients, the per-problem losses and the reduction partials.
namespace {
struct BaryLayout {
    size_t score, xb, gx, out, part, total;
};
BaryLayout bary_layout(int B, int N, int M, int dim) {
    BaryLayout L;
    const size_t nd = static_cast<size_t>(N) * dim;
    size_t o = sdtw_workspace_bytes_xy(B, N, M, dim);
    L.score = o;
    o += align_up(score_elems(B, N, M, g_k_override.load()) * sizeof(float), 256);
    L.xb = o;
    o += align_up(static_cast<size_t>(B) * nd * sizeof(float), 256);
    L.gx = o;
    o += align_up(static_cast<size_t>(B) * nd * sizeof(float), 256);
    L.out = o;
    o += align_up(static_cast<size_t>(B) * sizeof(float), 256);
    L.part = o;
    o += align_up(bary_reduce_part_floats(B, nd) * sizeof(float), 256);
    L.total = o;
    return L;
}
}  // namespace

size_t sdtw_barycenter_workspace_bytes(int B, int N, int M, int dim) {
    if (B <= 0 || N <= 0 || M <= 0 || dim <= 0) return 0;
    return bary_layout(B, N, M, dim).total;
}

int sdtw_barycenter_grad_f32(const float* bary, const float* X, const float* w, float* grad_loss, int B, int N, int M,
                             int dim, float gamma, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!bary || !X || !w || !grad_loss) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const BaryLayout L = bary_layout(B, N, M, dim);
    if ((rc = check_ws(workspace, workspace_bytes, L.total))) return rc;
    char* ws = static_cast<char*>(workspace);
    float* score = reinterpret_cast<float*>(ws + L.score);
    float* gx = reinterpret_cast<float*>(ws + L.gx);
    float* out = reinterpret_cast<float*>(ws + L.out);
    float* part = reinterpret_cast<float*>(ws + L.part);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t nd = static_cast<size_t>(N) * dim;
    const int dp = weight_store(B, N, M) ? fused_dp(dim, one_seq(bary), one_seq(X)) : 0;
    cudaError_t e;
    if (dp && grad_fused_gd(dim, X) == dp) {
        // The forward and the gradient read the one barycenter for every
        // problem (x batch stride 0); the costs are computed in the forward.
        uint64_t* wrap = static_cast<uint64_t*>(workspace);
        if ((rc = run_forward(nullptr, score, out, B, N, M, gamma, 0.f, wrap, st, true, nullptr, one_seq(bary),
                              one_seq(X), dim, dp, true)))
            return rc;
        // grad_x of every problem straight from the reverse pass.
        if ((rc = run_backward_grad(score, w, B, N, M, wrap, st, bary, 0, X, dim, dp, gx, true))) return rc;
    } else {
        // General path: the barycenter broadcast to every problem, then the
        // x/y pair.
        float* xb = reinterpret_cast<float*>(ws + L.xb);
        {
            KernelTimer kt("bary_broadcast", st);
            e = launch_bary_broadcast(bary, xb, B, nd, st);
        }
        if (e != cudaSuccess) return cuda_fail(e, "broadcast launch");
        if ((rc = sdtw_forward_xy_f32(xb, X, score, out, B, N, M, dim, gamma, 0.f, workspace, workspace_bytes, stream)))
            return rc;
        if ((rc = backward_xy_common(one_seq<const float>(xb), one_seq(X), score, nullptr, false, w, one_seq(gx),
                                     one_seq<float>(nullptr), B, N, M, dim, 0.f, workspace, st)))
            return rc;
    }
    {
        KernelTimer kt("bary_reduce", st, 2);
        e = launch_bary_reduce(gx, w, out, part, grad_loss, B, nd, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "reduce launch");
    return SDTW_OK;
}

int sdtw_barycenter_adam_f32(float* bary, float* exp_avg, float* exp_avg_sq, const float* grad_loss, size_t n,
                             const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                             float beta1, float beta2, float eps, float max_norm, void* stream) {
    int rc;
    if ((rc = ensure_status()) || (rc = pending_status())) return rc;
    if (!bary || !exp_avg || !exp_avg_sq || !grad_loss || !lr_table || !step || !loss_hist || !bary_hist)
        return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if (n == 0 || max_iter <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "n and max_iter must be > 0");
    if (!(beta1 >= 0.f && beta1 < 1.f) || !(beta2 >= 0.f && beta2 < 1.f) || !(eps >= 0.f) || !(max_norm > 0.f))
        return fail(SDTW_ERR_INVALID_ARGUMENT, "need 0 <= beta1, beta2 < 1, eps >= 0 and max_norm > 0");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        KernelTimer kt("bary_adam", st);
        e = launch_bary_adam(bary, exp_avg, exp_avg_sq, grad_loss, n, lr_table, max_iter, step, loss_hist, bary_hist,
                             beta1, beta2, eps, max_norm, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "adam launch");
    return SDTW_OK;
}

size_t sdtw_barycenter_sync_bytes(size_t n, int world) {
    if (n == 0 || world <= 0) return 0;
    return bary_sync_bytes(n, world);
}

int sdtw_barycenter_sync_adam_f32(float* grad_loss, size_t n, const unsigned long long* peers, int world, int rank,
                                  unsigned long long* epoch, float* bary, float* exp_avg, float* exp_avg_sq,
                                  const float* lr_table, int max_iter, int* step, float* loss_hist, float* bary_hist,
                                  float beta1, float beta2, float eps, float max_norm, void* stream) {
    int rc;
    if ((rc = ensure_status()) || (rc = pending_status())) return rc;
    if (!grad_loss || !peers || !epoch || !bary || !exp_avg || !exp_avg_sq || !lr_table || !step || !loss_hist ||
        !bary_hist)
        return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if (n == 0 || max_iter <= 0 || world <= 0 || rank < 0 || rank >= world || world > 512)
        return fail(SDTW_ERR_INVALID_ARGUMENT, "need n, max_iter > 0 and 0 <= rank < world <= 512");
    if (!(beta1 >= 0.f && beta1 < 1.f) || !(beta2 >= 0.f && beta2 < 1.f) || !(eps >= 0.f) || !(max_norm > 0.f))
        return fail(SDTW_ERR_INVALID_ARGUMENT, "need 0 <= beta1, beta2 < 1, eps >= 0 and max_norm > 0");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        KernelTimer kt("bary_sync_adam", st);
        e = launch_bary_sync_adam(grad_loss, n, peers, world, rank, epoch, bary, exp_avg, exp_avg_sq, lr_table, max_iter,
                                  step, loss_hist, bary_hist, beta1, beta2, eps, max_norm, wait_ctx(), st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "sync-adam launch");
    return SDTW_OK;
}

static int forward_sqeuclid_common(const SeqIn& x, const SeqIn& y, float* score, float* cost, float* out, int B, int N, int M,
                            int dim, float gamma, float bandwidth, void* workspace, cudaStream_t st);

int sdtw_forward_sqeuclid_f32(const float* x, const float* y, float* score, float* cost, float* out, int B, int N,
                              int M, int dim, float gamma, float bandwidth, void* workspace, size_t workspace_bytes,
                              void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y || !cost || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if (reinterpret_cast<uintptr_t>(cost) % 16u) return fail(SDTW_ERR_INVALID_ARGUMENT, "cost table must be 16-byte aligned");
    if ((rc = check_ws(workspace, workspace_bytes, wave_ws(B, N, M)))) return rc;
    return forward_sqeuclid_common(one_seq(x), one_seq(y), score, cost, out, B, N, M, dim, gamma, bandwidth, workspace,
                                   static_cast<cudaStream_t>(stream));
}

// The unfused forward over B problems whose sequences x, y name (one batch,
// or the normalized triple); the caller has checked the arguments.
static int forward_sqeuclid_common(const SeqIn& x, const SeqIn& y, float* score, float* cost, float* out, int B, int N, int M,
                            int dim, float gamma, float bandwidth, void* workspace, cudaStream_t st) {
    cudaError_t e;
    if (cost_tc_supported(x, y, dim)) {
        KernelTimer kt("cost_tc", st);
        e = launch_cost_tc(x, y, cost, plan(B, N, M, 0), dim, wait_ctx(), st);
    } else {
        KernelTimer kt("cost_wl", st);
        e = launch_cost_wl(x, y, cost, plan(B, N, M, 0), dim, false, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "cost launch");
    // With the share store the clamp mask of the gradient is marked in the
    // shares, so the reverse pass stores E already masked.
    return run_forward(cost, score, out, B, N, M, gamma, bandwidth, static_cast<uint64_t*>(workspace), st,
                       weight_store(B, N, M), nullptr, one_seq<const float>(nullptr), one_seq<const float>(nullptr), 0,
                       0, false, true);
}

int sdtw_backward_sqeuclid_f32(const float* x, const float* y, const float* score, const float* cost,
                               const float* grad_out, float* grad_x, float* grad_y, int B, int N, int M, int dim,
                               float gamma, float bandwidth, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_common(B, N, M, gamma)) || (rc = check_score(score))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y || !cost) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if ((rc = check_ws(workspace, workspace_bytes, sdtw_workspace_bytes_xy(B, N, M, dim)))) return rc;
    // Share store: E comes out of the reverse pass masked (the forward marked
    // the clamped costs); score store: the gradient kernels apply the mask.
    const bool ws = weight_store(B, N, M);
    return backward_xy_common(one_seq(x), one_seq(y), score, ws ? nullptr : cost, ws, grad_out, one_seq(grad_x),
                              one_seq(grad_y), B, N, M, dim, bandwidth, workspace, static_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------------------------------
// normalize=True (module.py:99-106 of the reference, which concatenates
// [x, x, y] and [y, x, y]): the 3B problems (x_b, y_b), (x_b, x_b), (y_b, y_b)
// read x and y in place.  The backward's gradients of the first B problems go
// straight to grad_x / grad_y; those of the self pairs go to four scratch
// blocks after the 3B-problem workspace and one kernel adds them in.
static size_t norm_block_bytes(int B, int N, int dim) {
    return align_up(static_cast<size_t>(B) * N * dim * sizeof(float), 256);
}
static size_t norm_scratch_off(int B, int N, int dim) {
    return align_up(sdtw_workspace_bytes_xy(3 * B, N, N, dim), 256);
}

size_t sdtw_workspace_bytes_norm(int B, int N, int dim) {
    if (B <= 0 || N <= 0 || dim <= 0 || B > (1 << 30) / 3) return 0;
    return norm_scratch_off(B, N, dim) + 4 * norm_block_bytes(B, N, dim);
}

// need: 0 = the fused forward's workspace, 1 = the unfused forward's, 2 = the backward's.
static int check_norm(const float* x, const float* y, const float* score, int B, int N, int dim, float gamma,
                      void* workspace, size_t workspace_bytes, int need) {
    int rc;
    if (B <= 0 || B > (1 << 30) / 3) return fail(SDTW_ERR_INVALID_ARGUMENT, "B must be > 0");
    if ((rc = check_common(3 * B, N, N, gamma)) || (rc = check_score(score))) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!x || !y) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t bytes = need == 0   ? wave_ws_xy(3 * B, N, N, dim) + wl_bytes(3 * B, N, N)
                         : need == 1 ? wave_ws(3 * B, N, N)
                                     : sdtw_workspace_bytes_norm(B, N, dim);
    return check_ws(workspace, workspace_bytes, bytes);
}

int sdtw_forward_xy_norm_f32(const float* x, const float* y, float* score, float* out, int B, int N, int dim,
                             float gamma, float bandwidth, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_norm(x, y, score, B, N, dim, gamma, workspace, workspace_bytes, 0))) return rc;
    if (!out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    return forward_xy_common(norm_x(x, y, B), norm_y(x, y, B), score, out, 3 * B, N, N, dim, gamma, bandwidth,
                             workspace, static_cast<cudaStream_t>(stream));
}

int sdtw_forward_sqeuclid_norm_f32(const float* x, const float* y, float* score, float* cost, float* out, int B, int N,
                                   int dim, float gamma, float bandwidth, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    int rc;
    if ((rc = check_norm(x, y, score, B, N, dim, gamma, workspace, workspace_bytes, 1))) return rc;
    if (!cost || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    if (reinterpret_cast<uintptr_t>(cost) % 16u) return fail(SDTW_ERR_INVALID_ARGUMENT, "cost table must be 16-byte aligned");
    return forward_sqeuclid_common(norm_x(x, y, B), norm_y(x, y, B), score, cost, out, 3 * B, N, N, dim, gamma,
                                   bandwidth, workspace, static_cast<cudaStream_t>(stream));
}

static int backward_norm(const float* x, const float* y, const float* score, const float* mask_w, bool marked,
                         const float* grad_out, float* grad_x, float* grad_y, int B, int N, int dim, float bandwidth,
                         void* workspace, cudaStream_t st) {
    if (!grad_x || !grad_y) return fail(SDTW_ERR_INVALID_ARGUMENT, "the normalized backward writes both gradients");
    char* scratch = static_cast<char*>(workspace) + norm_scratch_off(B, N, dim);
    const size_t blk = norm_block_bytes(B, N, dim);
    float* s0 = reinterpret_cast<float*>(scratch);            // (x, x): gradient of the first x
    float* s1 = reinterpret_cast<float*>(scratch + blk);      // (x, x): of the second
    float* s2 = reinterpret_cast<float*>(scratch + 2 * blk);  // (y, y): of the first y
    float* s3 = reinterpret_cast<float*>(scratch + 3 * blk);  // (y, y): of the second
    const SeqOut gx{{grad_x, s0, s2}, B};
    const SeqOut gy{{grad_y, s1, s3}, B};
    int rc = backward_xy_common(norm_x(x, y, B), norm_y(x, y, B), score, mask_w, marked, grad_out, gx, gy, 3 * B, N, N,
                                dim, bandwidth, workspace, st);
    if (rc) return rc;
    const size_t n = static_cast<size_t>(B) * N * dim;
    cudaError_t e;
    {
        KernelTimer kt("norm_fold", st, 2);
        e = launch_add2(grad_x, s0, s1, n, st);
        if (e == cudaSuccess) e = launch_add2(grad_y, s2, s3, n, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "fold launch");
    return SDTW_OK;
}

int sdtw_backward_xy_norm_f32(const float* x, const float* y, const float* score, const float* grad_out,
                              float* grad_x, float* grad_y, int B, int N, int dim, float gamma, float bandwidth,
                              void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_norm(x, y, score, B, N, dim, gamma, workspace, workspace_bytes, 2))) return rc;
    return backward_norm(x, y, score, nullptr, false, grad_out, grad_x, grad_y, B, N, dim, bandwidth, workspace,
                         static_cast<cudaStream_t>(stream));
}

int sdtw_backward_sqeuclid_norm_f32(const float* x, const float* y, const float* score, const float* cost,
                                    const float* grad_out, float* grad_x, float* grad_y, int B, int N, int dim,
                                    float gamma, float bandwidth, void* workspace, size_t workspace_bytes,
                                    void* stream) {
    int rc;
    if ((rc = check_norm(x, y, score, B, N, dim, gamma, workspace, workspace_bytes, 2))) return rc;
    if (!cost) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const bool ws = weight_store(3 * B, N, N);
    return backward_norm(x, y, score, ws ? nullptr : cost, ws, grad_out, grad_x, grad_y, B, N, dim, bandwidth,
                         workspace, static_cast<cudaStream_t>(stream));
}

int sdtw_grad_sqeuclid_f32(const float* G, const float* D_mask, const float* x, const float* y, float* grad_x,
                           float* grad_y, int B, int N, int M, int dim, void* stream) {
    int rc = check_dims(B, N, M);
    if (rc) return rc;
    if (dim <= 0) return fail(SDTW_ERR_INVALID_ARGUMENT, "dim must be > 0");
    if (!G || !x || !y) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e;
    {
        KernelTimer kt("grad_xy", static_cast<cudaStream_t>(stream), (grad_x ? 1 : 0) + (grad_y ? 1 : 0));
        e = launch_grad_xy(G, D_mask, x, y, grad_x, grad_y, B, N, M, dim, static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "grad launch");
    return SDTW_OK;
}

int sdtw_score_to_R_f32(const float* score, float* R, int B, int N, int M, float gamma, void* stream) {
    int rc;
    if ((rc = check_dims(B, N, M)) || (rc = check_gamma(gamma))) return rc;
    if (!score || !R) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    // The forward writes it with bulk copies of whole anti-diagonal rows.
    if (reinterpret_cast<uintptr_t>(score) % 16u) return fail(SDTW_ERR_INVALID_ARGUMENT, "score must be 16-byte aligned");
    WavePlan p = plan(B, N, M, 0);
    const float kk = kLog2e / gamma;
    cudaError_t e = launch_score_to_R(reinterpret_cast<const float2*>(score), R, p, static_cast<float>(1.0 / (double)kk),
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "score_to_R launch");
    return SDTW_OK;
}

int sdtw_R_to_score_f32(const float* R, float* score, int B, int N, int M, float gamma, void* stream) {
    int rc;
    if ((rc = check_dims(B, N, M)) || (rc = check_gamma(gamma))) return rc;
    if (!score || !R) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    WavePlan p = plan(B, N, M, 0);
    cudaError_t e = launch_R_to_score(R, reinterpret_cast<float2*>(score), p, kLog2e / gamma, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "R_to_score launch");
    return SDTW_OK;
}


int sdtw_forward_noalloc_f32(const float* D, float* score, float* out, int B, int N, int M, float gamma,
                             float bandwidth, void* stream) {
    int rc;
    if ((rc = check_dims(B, N, M)) || (rc = check_gamma(gamma)) || (rc = check_score(score))) return rc;
    if (!D || !out) return fail(SDTW_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t w0 = wave_ws(B, N, M);
    const size_t need = w0 + wl_bytes(B, N, M);
    if (need > kNoAllocScratchBytes)
        return fail(SDTW_ERR_INVALID_ARGUMENT,
                    "problem too large for the allocation-free forward: needs " + std::to_string(need) +
                        " bytes of scratch, the fixed array holds " + std::to_string(kNoAllocScratchBytes) +
                        " (use sdtw_forward_f32 with a workspace)");
    // A failure recorded by an earlier launch of another entry point still
    // surfaces here (its status record exists only if one of them ran).
    if ((rc = pending_status())) return rc;
    int dev = 0;
    void* base = nullptr;
    int* status = nullptr;
    if ((rc = noalloc_addrs(&dev, &base, &status))) return rc;
    g_noalloc_used.fetch_or(1ull << dev);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The array keeps the previous call's contents.  The anti-diagonal copy of D
    // is fully rewritten below; the band-wrap ring's slots are reset so that no
    // stale entry can carry a matching tag.
    if (w0) {
        cudaError_t e = cudaMemsetAsync(base, 0xff, w0, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(no-alloc ring)");
    }
    float* Dw = reinterpret_cast<float*>(static_cast<char*>(base) + w0);
    cudaError_t e;
    {
        KernelTimer kt("rm_to_wl", st);
        e = launch_rm_to_wl(D, Dw, plan(B, N, M, 0), st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "layout launch");
    WaitCtx w = wait_ctx();
    w.status = status;
    w.diag = reinterpret_cast<volatile WaitDiag*>(status + 8);
    return run_forward(Dw, score, out, B, N, M, gamma, bandwidth, static_cast<uint64_t*>(base), st, false, &w);
}

}  // extern "C"
