// sdtw_plan.h -- launch geometry and the score-store layout of the wavefront
// kernels (host and device).
//
// A problem (one (x_b, y_b) pair, N rows by M columns) is cut into horizontal
// stripes of 32*K rows.  One warp owns a stripe: lane l holds rows
// l*K .. l*K+K-1 of it and the warp sweeps the stripe's anti-diagonals, so at
// local step t lane l works on columns t - l*K - k.  Stripes form a chain:
// stripe s needs the bottom row of stripe s-1 (forward) or sends messages to it
// (backward).  G consecutive stripes ("a band") run concurrently on the G warps
// of one thread-block cluster (wpc warps per CTA, csize CTAs); longer problems
// loop over bands inside the same cluster, the last warp of band b handing its
// bottom row to the first warp of band b+1 through a global ring.
//
// Score store ("wavefront layout"): for problem b, stripe s, local
// anti-diagonal t in [0, n_diag) and in-stripe position p = k*32 + l,
//     score[((b*n_stripes + s)*n_diag + t)*(32*K) + p]      (a float2)
// holds T(row = s*32*K + l*K + k, col = t - l*K - k) = -R(row, col)*log2(e)/gamma
// as an unevaluated pair hi + lo.  One warp step writes 32 consecutive float2
// per k: a coalesced 256-byte store.
#pragma once

#include <cstddef>
#include <cstdint>

namespace sdtw {

struct WavePlan {
    int B, N, M;
    int K;          // rows per lane (template parameter of the kernels)
    int wpc;        // warps per CTA
    int csize;      // CTAs per problem (cluster size)
    int G;          // warps per band = wpc * csize
    int n_stripes;  // ceil(N / (32*K))
    int n_bands;    // ceil(n_stripes / G)
    int n_diag;     // anti-diagonal rows per stripe: wl_diag(M, 32K) (M + 32K - 1, padded)
};

// Anti-diagonal rows stored per stripe.  A stripe has M + 32K - 1 of them;
// the table is padded to a multiple of 16 plus 16 rows, so that the wavefront
// kernels may run whole step groups and prefetch up to 16 rows ahead without
// clamping addresses (the padding holds cells outside the table, which no
// real cell reads).
inline int wl_diag(int M, int sr) { return (M + sr - 1 + 15) / 16 * 16 + 16; }

// Rows per lane as a function of the problem only (the score layout depends on
// it, so forward and backward must agree).
inline int rows_per_lane(int N, int k_override = 0) {
    if (k_override == 1 || k_override == 2 || k_override == 4) return k_override;
    // One row per lane keeps the dependent chain of a step shortest.  Measured
    // on B200 with the occupancy-aware plan, one row per lane is also the
    // faster choice for long sequences (N = M = 4096: 2.5 ms forward at 1, 2.6
    // ms at 2); 2 and 4 stay available through the plan override.
    (void)N;
    return 1;
}

// Cells (with the layout's padding) of a (B,N,M) table in the wavefront layout.
inline size_t wl_cells(int B, int N, int M, int k_override = 0) {
    const int K = rows_per_lane(N, k_override);
    const size_t sr = 32u * (size_t)K;
    const size_t ns = ((size_t)N + sr - 1) / sr;
    return (size_t)B * ns * (size_t)wl_diag(M, (int)sr) * sr;
}

// float32 elements (2 per cell: hi, lo) of the score store.
inline size_t score_elems(int B, int N, int M, int k_override = 0) {
    return 2u * wl_cells(B, N, M, k_override);
}

// Stripes (chain warps) per CTA the wavefront kernels are compiled for: 8
// (with one DP row per lane the forward pairs each chain warp with a helper
// warp, 512 threads; with more rows per lane the registers need 255 per thread).
inline int wpc_max(int K) { (void)K; return 8; }

// wpc_override / cs_override / k_override (> 0) force the warps per CTA, the
// cluster size and the rows per lane (tests use them to exercise many bands
// and clusters on small problems).
inline WavePlan make_plan(int B, int N, int M, int num_sms, int wpc_override = 0, int cs_override = 0,
                          int k_override = 0) {
    WavePlan p{};
    p.B = B;
    p.N = N;
    p.M = M;
    p.K = rows_per_lane(N, k_override);
    const int sr = 32 * p.K;
    p.n_stripes = (N + sr - 1) / sr;
    p.n_diag = wl_diag(M, sr);
    // Spread a problem over up to 8 CTAs (portable cluster size) while the
    // batch alone would leave SMs idle, and further while a problem's stripes
    // would need more warps per CTA than the kernels allow (one band) and the
    // clusters still fit on the GPU at one CTA per SM.
    const int wmax = wpc_max(p.K);
    int cs = 1;
    while (cs < 8 && (long long)B * cs * 2 <= (long long)num_sms && cs * 2 <= p.n_stripes) cs *= 2;
    while (cs < 8 && (p.n_stripes + cs - 1) / cs > wmax && (long long)B * cs * 2 <= 2LL * num_sms) cs *= 2;
    if (cs_override > 0) cs = cs_override < 8 ? cs_override : 8;
    int wpc = (p.n_stripes + cs - 1) / cs;
    if (wpc > wmax) wpc = wmax;
    if (wpc < 1) wpc = 1;
    if (wpc_override > 0) wpc = wpc_override < wmax ? wpc_override : wmax;
    p.csize = cs;
    p.wpc = wpc;
    p.G = wpc * cs;
    p.n_bands = (p.n_stripes + p.G - 1) / p.G;
    return p;
}

// Global band-wrap ring: two tagged u64 per column per problem (hi and lo of
// the forward's bottom row; the reverse pass uses the first).
inline size_t wrap_bytes(const WavePlan& p) {
    return p.n_bands > 1 ? (size_t)p.B * (size_t)p.M * 16u : 0u;
}

}  // namespace sdtw
