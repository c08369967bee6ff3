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
//   * T is carried and stored as an unevaluated float32 pair (hi, lo),
//     T = hi + lo with |lo| <= ulp(hi)/2: the new cell is m_hi + delta with the
//     rounding error of that sum kept in lo (TwoSum), and D * log2(e)/gamma is
//     split exactly (TwoProduct).  |T| grows along the path while the backward
//     weights depend on differences of neighbouring T, so a plain float32 T
//     loses ~ulp(T)/gamma of accuracy per weight; the pair keeps the weights
//     at float32 relative accuracy.  (The lo of the max cancels out of
//     sum_k ex2(T_k - m), so no arg-max is needed.)
//   * the backward weight exp((R[c] - D[c] - R[p]) / gamma) equals the softmax
//     weight of predecessor p among c's three predecessors, so the reverse pass
//     recomputes it from the stored scores of c's predecessors, normalised to
//     sum to one.  It needs no cost values and no log-space E table.  (The x/y
//     entry points store the weights themselves instead of scores: the
//     kernels of wavefront_exp.cu.)
//   * one warp per stripe of 32*K rows, three live anti-diagonals in registers,
//     neighbour rows exchanged with one warp shuffle per step, stripe-to-stripe
//     rows handed over through tagged u64 ring slots in the consumer's shared
//     memory (DSMEM stores across the CTAs of a cluster), bounded waits only.
#include <type_traits>

#include "sdtw_device.cuh"
#include "sdtw_kernels.h"
#include "sdtw_plan.h"
#include "wavefront_ring.cuh"

namespace sdtw {

// Step bodies of the forward (compile-time phases, one store staging buffer
// each).  With the cost rows staged in shared memory one body measured as fast
// as two at C2 and 3.5 % faster at C3 (N = M = 4096: the smaller code); with
// the costs in a register queue, two had beaten one and three or four spilled.
constexpr int kFwdPhases = 1;
// The forward's cost rows are staged after its store buffers: [wpc][3][PF][32K]
// floats (three groups: the current one and two in flight).
__host__ __device__ constexpr int fwd_pf(int K) { return K >= 4 ? 4 : 8; }
__host__ __device__ constexpr size_t fwd_cost_offset(int wpc, int K) {
    return fwd_stage_offset(wpc) + static_cast<size_t>(wpc) * kFwdPhases * fwd_pf(K) * 32 * K * 8;
}
// End of the reverse pass's E staging ([wpc][nph][PF][32K] floats).
__host__ __device__ constexpr size_t bwd_stage_end(int wpc, int K, int nph) {
    return fwd_stage_offset(wpc) + static_cast<size_t>(wpc) * nph * fwd_pf(K) * 32 * K * 4;
}

// ============================================================== step groups
// Steps run in groups of PF.  Per group (warp-uniform code): the consumer lane
// reads and checks the PF ring slots it will need, the producer lane checks
// flow control once, and every 32 columns a relaxed store reports progress.
// Per step: shuffles, the cell math, one shared-memory read of the step's cost
// (forward) and one staged table store, one predicated ring store -- no
// branches.  A group's input rows are
// copied into shared memory two groups ahead, its output rows leave as one
// bulk copy (the score-store reverse pass loads its score rows one group ahead
// into registers).
template <int K>
struct StepCfg {
    static constexpr int PF = (K >= 4) ? 4 : 8;
};


// ============================================================== forward
// Ring slot pair layout (per consumer warp): kRing x {hi, lo} tagged u64;
// column c of band b's row above is tagged g = b * M + c and sits in slot
// g % kRing, so that the slots, like the flow-control counter, advance
// sequentially across band boundaries.
//
// Step code.  The anti-diagonal rows are padded (wl_diag), so every group runs
// PF whole steps; the cost rows of a group are copied into shared memory two
// groups ahead.  Cells outside the table (left of column 0, right of column M-1,
// rows past N) or the band are stored as -inf.  The rows of a group go out as
// one bulk copy from shared memory; the last cell's score is kept in registers
// by its lane as it passes.
template <int K, bool BANDED>
__global__ void __launch_bounds__(K == 1 ? 512 : 256) fwd_kernel(const FwdArgs a) {
    constexpr int PF = StepCfg<K>::PF;
    constexpr int NPH = kFwdPhases;  // step bodies (phases): store staging buffer per phase
    constexpr int SR = 32 * K;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    const int N = P.N, M = P.M;

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);                    // [wpc][kRing][2]
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * 2 * kRing);  // [wpc]
    // Table rows of a group are staged here ([NPH][PF][SR] float2 per warp, one
    // buffer per phase) and written by one bulk copy (the rows of a group are
    // contiguous): the warp never waits on global stores.
    float2* stage = reinterpret_cast<float2*>(smem_raw + fwd_stage_offset(wpc)) + warp * NPH * PF * SR;
    const uint32_t stage_s = smem_addr(stage);
    // Cost rows of group g are copied (16-byte cp.async) two groups ahead into
    // buffer (g - g_begin) % 3 of [3][PF][SR] floats.
    const float* cost = reinterpret_cast<const float*>(smem_raw + fwd_cost_offset(wpc, K)) + warp * 3 * PF * SR;
    const uint32_t cost_s = smem_addr(cost);
    for (int i = threadIdx.x; i < wpc * 2 * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    cluster_sync_all();

    const uint32_t my_consumed = smem_addr(consumed + warp);
    const uint32_t my_ring_s = smem_addr(ring + warp * 2 * kRing);
    uint64_t next_ring_g = 0;
    uint32_t prev_consumed = 0;
    if (g + 1 < P.G) next_ring_g = mapa_generic(ring + ((g + 1) % wpc) * 2 * kRing, (g + 1) / wpc);
    if (g > 0) prev_consumed = mapa_shared(smem_addr(consumed + (g - 1) % wpc), (g - 1) / wpc);

    const float kk = a.kk;
    // Cells outside the table or the band.
    const float NEG = neg_inf();
    const int ibw = a.ibw;
    WaitCtx wc = a.wait;
    wc.kernel = 1;
    wc.problem = b;
    wc.warp = g;
    bool ok = true;          // false once a wait of this lane failed
    bool quit = false;       // warp-uniform
    uint32_t cons_seen = 0;  // consumer progress last observed

    for (int band = 0; band < P.n_bands && !quit; ++band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) break;
        wc.band = band;
        const int R0 = s * SR;
        const bool has_in = R0 > 0;
        const bool in_wrap = (g == 0);
        const bool has_out = (s + 1 < P.n_stripes) && (s != a.debug_stall);
        const bool out_wrap = (g == P.G - 1);
        const uint32_t band_base = static_cast<uint32_t>(band) * static_cast<uint32_t>(M);
        const size_t sb = stripe_base(P, b, s);
        float2* Tl = a.score + sb + lane;  // this lane's position of anti-diagonal row 0 (k = 0)
        const float* Dl = a.Dw + sb + lane;
        // Global band-wrap ring: slot c = column c (two u64: hi, lo).
        const uint64_t wrap_g = reinterpret_cast<uint64_t>(a.wrap + static_cast<size_t>(b) * 2 * M);
        const uint64_t out_g = out_wrap ? wrap_g : next_ring_g;
        const uint32_t in_tag_wrap = wrap_tag(a.seq, band - 1);
        const uint32_t out_tag_wrap = wrap_tag(a.seq, band);
        const bool pub31 = has_out && lane == 31;

        // Everything before this band counts as consumed (see the reverse pass).
        st_release_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed, band_base);

        const int n_steps = M + SR - 1;
        const int n_groups = (n_steps + PF - 1) / PF;
        // Band-limited launch: only the groups whose anti-diagonals hold an
        // in-band cell of this stripe run, t in [R0 - ibw - 1, SR - 1 + (R0 + SR - 1 + ibw)]
        // (one step early, so that the first in-band cell has its diagonal
        // predecessor from the stripe above); the rows outside are written as -inf.
        int g_begin = 0, g_end = n_groups;
        if constexpr (BANDED) {
            const int t_lo = max(0, R0 - ibw - 1);
            const int t_hi = min(n_steps - 1, (SR - 1) + min(M - 1, R0 + SR - 1 + ibw));
            g_begin = (t_lo / PF) / NPH * NPH;
            g_end = max(g_begin, min(n_groups, t_hi / PF + 1));
        }
        const int t_begin = g_begin * PF;
        // Last column of the row above that is in the band (and so published by
        // the stripe above); the columns past it read as -inf without the ring.
        const int c_pub_max = BANDED ? min(M - 1, R0 - 1 + ibw) : M - 1;
        // Group gg's cost rows (PF * SR contiguous floats), or an empty commit
        // past the last group, so that every group finds its rows two commits back.
        auto cost_copy = [&](int gg) {
            if (gg < g_end) {
                const float* src = Dl - lane + static_cast<size_t>(gg) * PF * SR;
                const uint32_t dst = cost_s + static_cast<uint32_t>((gg - g_begin) % 3) * PF * SR * 4u;
#pragma unroll
                for (int i = 0; i < PF * SR / 128; ++i) cp_async16(dst + (lane + 32 * i) * 16u, src + (lane + 32 * i) * 4);
            }
            cp_async_commit();
        };
        cost_copy(g_begin);
        cost_copy(g_begin + 1);
        // The columns before t_begin are never read: report them consumed, so
        // that the stripe above may run up to a full ring ahead of this start.
        if (t_begin > 0)
            st_relaxed_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed,
                                      band_base + static_cast<uint32_t>(min(t_begin, M)));

        // Three live anti-diagonals: c* = step t-1, o* = step t-2, as (hi, lo).
        float ch[K], cl[K], oh[K], ol[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            ch[k] = oh[k] = NEG;
            cl[k] = ol[k] = 0.f;
        }
        float uph_prev = (R0 == 0) ? 0.f : NEG;  // T(R0-1, -1)
        float upl_prev = 0.f;
        const int q0 = lane * K;  // row offset of k = 0 in the stripe
        const int rows_left = N - R0;
        // The lane of the last row keeps the last cell's score (step t_last)
        // as it passes (the table rows go out by bulk copies).
        const int t_last = (s == P.n_stripes - 1 && (N - 1 - R0) / K == lane) ? N - 1 - R0 + M - 1 : -1;
        const int k_last = (N - 1 - R0) % K;
        float last_h = 0.f, last_l = 0.f;
        // Band-wrap input (global memory, an L2 round trip per load): the slots
        // of the next group are loaded one group ahead.  The data is normally
        // long written by then (the band above ran M + SR - 1 steps earlier);
        // a slot read too early shows an older tag and is polled again.
        uint64_t wpf_h = 0, wpf_l = 0;
        if (has_in && in_wrap && t_begin < M && t_begin + (lane & (PF - 1)) <= c_pub_max)
            ld_pair(wrap_g + static_cast<uint32_t>(t_begin + (lane & (PF - 1))) * 16u, wpf_h, wpf_l);

        auto group = [&](auto phase_c, int t0) {
            constexpr int PH = decltype(phase_c)::value;
            // ---- prologue: the row above for columns t0 .. t0+PF-1 (lane 0).
            float rin_h[PF], rin_l[PF];
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                rin_h[u] = NEG;
                rin_l[u] = 0.f;
            }
            if (has_in && t0 < M && t0 <= c_pub_max) {  // warp-uniform
                // Lane u (mod PF) reads slot u: one load instruction for the whole
                // group (measured on B200: eight loads issued by one lane cost about
                // 850 cycles per group, one warp-wide load about 200 with the
                // vote and the shuffles).  The tag vote makes the re-poll loop
                // below a uniform branch, taken only when the producer is behind.
                const uint32_t tg0 = in_wrap ? in_tag_wrap : band_base + static_cast<uint32_t>(t0);
                bool all = true;
                float vh = NEG, vl = 0.f;
                auto probe = [&]() {  // load + tag vote; re-polls repeat only this
                    const int u = lane & (PF - 1);
                    const int col = t0 + u;
                    const uint32_t tg = in_wrap ? tg0 : tg0 + static_cast<uint32_t>(u);
                    bool mine = true;
                    if (col <= c_pub_max) {
                        uint64_t eh, el;
                        if (in_wrap) ld_pair(wrap_g + static_cast<uint32_t>(col) * 16u, eh, el);
                        else ld_pair_shared(my_ring_s + (tg % kRing) * 16u, eh, el);
                        mine = tag_of(eh) == tg && tag_of(el) == tg;
                        vh = val_of(eh);
                        vl = val_of(el);
                    }
                    all = __all_sync(SDTW_FULL_MASK, mine);
                };
                if (in_wrap) {  // warp-uniform: the prefetched slots, then the next group's
                    const int col = t0 + (lane & (PF - 1));
                    bool mine = true;
                    if (col <= c_pub_max) {
                        mine = tag_of(wpf_h) == tg0 && tag_of(wpf_l) == tg0;
                        vh = val_of(wpf_h);
                        vl = val_of(wpf_l);
                    }
                    all = __all_sync(SDTW_FULL_MASK, mine);
                    if (col + PF <= c_pub_max) ld_pair(wrap_g + static_cast<uint32_t>(col + PF) * 16u, wpf_h, wpf_l);
                } else {
                    probe();
                }
                if (!all && ok) {  // uniform (vote)
                    uint64_t w0 = 0;
                    for (uint32_t it = 1;; ++it) {
                        probe();
                        if (all) break;
                        const int r = backoff(it, w0, wc);
                        if (r) {
                            if (lane == 0) record_giveup(wc, r, 1, tg0, 0);
                            ok = false;
                            break;
                        }
                    }
                }
                // The whole group at once: per-step shuffles measured slower here
                // (every stripe would pay them, the first one included).
#pragma unroll
                for (int w = 0; w < PF; ++w) {
                    rin_h[w] = __shfl_sync(SDTW_FULL_MASK, vh, w);
                    rin_l[w] = __shfl_sync(SDTW_FULL_MASK, vl, w);
                }
                const int done = min(t0 + PF, M);
                st_relaxed_cluster_u32_if(!in_wrap && report_due(done, PF, M) && lane == 0, prev_consumed,
                                          band_base + static_cast<uint32_t>(done));
            }
            // ---- flow control for the columns this group publishes (lane 31).
            if (has_out && !out_wrap) {  // warp-uniform
                const int col_last = min(t0 + PF - 1 - (SR - 1), M - 1);
                if (col_last >= 0) {
                    const uint32_t gc = band_base + static_cast<uint32_t>(col_last);
                    // Every lane tracks cons_seen identically (uniform branch).
                    if (__any_sync(SDTW_FULL_MASK, ok && gc >= static_cast<uint32_t>(kRing) &&
                                                       static_cast<int32_t>(cons_seen - (gc - kRing + 1)) < 0)) {
                        cons_seen = wait_counter_ge(my_consumed, gc - kRing + 1, wc);
                        ok = ok && static_cast<int32_t>(cons_seen - (gc - kRing + 1)) >= 0;
                    }
                }
            }
            // ---- PF steps.
            // This phase's staging buffer was last read by the copy NPH groups
            // ago; this group's cost rows (two commits back) have landed.
            if (lane == 0) bulk_wait_read<NPH - 1>();
            cp_async_wait<1>();
            __syncwarp();
            const int gg = t0 / PF;
            const float* cb = cost + ((gg - g_begin) % 3) * PF * SR + lane;
            cost_copy(gg + 2);  // into the buffer the previous group read
            float2* Tg = stage + PH * PF * SR + lane;
            const int colb0 = t0 - (SR - 1);  // bottom-row column of step t0
            const uint32_t tgo0 = out_wrap ? out_tag_wrap : band_base + static_cast<uint32_t>(colb0);
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int t = t0 + u;
                float c[K];
#pragma unroll
                for (int k = 0; k < K; ++k) c[k] = cb[u * SR + k * 32];
                float uph = __shfl_up_sync(SDTW_FULL_MASK, ch[K - 1], 1);
                float upl = __shfl_up_sync(SDTW_FULL_MASK, cl[K - 1], 1);
                uph = (lane == 0) ? rin_h[u] : uph;
                upl = (lane == 0) ? rin_l[u] : upl;
                const float dgh = uph_prev, dgl = upl_prev;
                uph_prev = uph;
                upl_prev = upl;
                float nh[K], nl[K];
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const float lh = ch[k], ll = cl[k];
                    const float uh = (k == 0) ? uph : ch[k > 0 ? k - 1 : 0];
                    const float ul = (k == 0) ? upl : cl[k > 0 ? k - 1 : 0];
                    const float dh = (k == 0) ? dgh : oh[k > 0 ? k - 1 : 0];
                    const float dl = (k == 0) ? dgl : ol[k > 0 ? k - 1 : 0];
                    // TwoProduct: c*kk = p + e exactly.
                    const float p = c[k] * kk;
                    const float e = fmaf(c[k], kk, -p);
                    const float m = max3f(dh, uh, lh);
                    const float ed = ex2f((dh - m) + dl), eu = ex2f((uh - m) + ul), el = ex2f((lh - m) + ll);
                    const float sm = ed + eu + el;
                    const float delta = lg2f(sm) - p;
                    // TwoSum: m + delta = hi + lo exactly; the product's error e
                    // joins lo (off the dependent chain).
                    const float hi = m + delta;
                    const float bb = hi - m;
                    const float lo = ((m - (hi - bb)) + (delta - bb)) - e;
                    // Cells outside the table (or the band) read as -inf.
                    const int col = t - (q0 + k);
                    bool live = static_cast<unsigned>(col) < static_cast<unsigned>(M) && q0 + k < rows_left;
                    if constexpr (BANDED)
                        live = live && static_cast<unsigned>(R0 + q0 + k - col + ibw) <= static_cast<unsigned>(2 * ibw);
                    nh[k] = live ? hi : NEG;
                    nl[k] = live ? lo : 0.f;
                    Tg[u * SR + k * 32] = make_float2(nh[k], nl[k]);
                    if (K == 1 || k == k_last) {
                        last_h = (t == t_last) ? nh[k] : last_h;
                        last_l = (t == t_last) ? nl[k] : last_l;
                    }
                }
                // Bottom row of the stripe goes to the next stripe's warp.
                const int colb = colb0 + u;
                const bool pub = pub31 && static_cast<unsigned>(colb) < static_cast<unsigned>(M);
                const uint32_t tgo = out_wrap ? tgo0 : tgo0 + static_cast<uint32_t>(u);
                const uint32_t slot = out_wrap ? static_cast<uint32_t>(colb) : (tgo % kRing);
                st_pair_if(pub, out_g + slot * 16u, pack_tagged(nh[K - 1], tgo), pack_tagged(nl[K - 1], tgo));
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    oh[k] = ch[k];
                    ol[k] = cl[k];
                    ch[k] = nh[k];
                    cl[k] = nl[k];
                }
            }
            // Rows t0 .. t0 + PF - 1 of the table: one bulk copy.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_s2g(Tl - lane + static_cast<size_t>(t0) * SR, stage_s + PH * PF * SR * 8u, PF * SR * 8u);
                bulk_commit();
            }
        };
        using P0 = std::integral_constant<int, 0>;
        using P1 = std::integral_constant<int, 1>;
        for (int gi = g_begin; gi < g_end; gi += NPH) {
            const int t0 = gi * PF;
            group(P0{}, t0);
            if constexpr (NPH >= 2) {
                if (gi + 1 < g_end) group(P1{}, t0 + PF);
            }
            if constexpr (NPH >= 3) {
                if (gi + 2 < g_end) group(std::integral_constant<int, 2>{}, t0 + 2 * PF);
            }
            if constexpr (NPH >= 4) {
                if (gi + 3 < g_end) group(std::integral_constant<int, 3>{}, t0 + 3 * PF);
            }
            if ((gi & 15) == 16 - NPH && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
        // The band's copies are complete before the fill stores below and the
        // next band's first group (which reuses phase 0's buffer and the cost buffers).
        if (lane == 0) bulk_wait_all();
        cp_async_wait<0>();
        __syncwarp();
        // Rows outside the groups that ran (padding, or out of the band): -inf,
        // like every cell outside the table.
        const float2 fill = make_float2(NEG, 0.f);
        for (int t = 0; t < t_begin; ++t)
#pragma unroll
            for (int k = 0; k < K; ++k) Tl[static_cast<size_t>(t) * SR + k * 32] = fill;
        for (int t = g_end * PF; t < P.n_diag; ++t)
#pragma unroll
            for (int k = 0; k < K; ++k) Tl[static_cast<size_t>(t) * SR + k * 32] = fill;
        if (!quit && t_last >= 0)
            a.out[b] = last_h <= -1.0e29f ? pos_inf() : fmaf(-last_h, a.inv_k, -last_l * a.inv_k);
    }
    // No CTA may leave while a peer can still write into its shared memory.
    cluster_sync_all();
}

// ============================================================== backward
template <int K>
__device__ __forceinline__ float2 load_score(const float2* __restrict__ S, const WavePlan& P, int b, int row, int col) {
    constexpr int SR = 32 * K;
    if (row < 0) return make_float2((col < 0) ? 0.f : neg_inf(), 0.f);
    if (col < 0) return make_float2(neg_inf(), 0.f);
    const int s = row / SR;
    const int q = row - s * SR;
    const int l = q / K;
    const int k = q - l * K;
    const size_t idx = ((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + (q + col)) * SR + k * 32 + l;
    return __ldg(S + idx);
}

// Reverse wavefront.  At reverse step t the lane holding row q handles cell
// (q, j = t - q) and needs the scores of its predecessors (q-1, j-1), (q-1, j)
// and (q, j-1): the stripe's anti-diagonal rows t-2 and t-1 (coalesced float2
// loads, PF steps ahead), the row above from the neighbour lane by shuffle,
// and for lane 0 the last row of the previous stripe (one prefetched load).
// E is written in the wavefront layout.
template <int K, bool BANDED>
__global__ void __launch_bounds__(K == 1 ? 512 : 256) bwd_kernel(const BwdArgs a) {
    constexpr int PF = StepCfg<K>::PF;
    // Prefetch distance: one group (K = 1, whose 512-thread launches leave 128
    // registers per thread), two groups (K > 1).
    constexpr int NPH = K == 1 ? 1 : 2;
    constexpr int PD = NPH * PF;
    constexpr int SR = 32 * K;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    const int N = P.N, M = P.M;

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * kRing);
    // E rows of a group are staged here ([NPH][PF][SR] floats per warp, one
    // buffer per phase, after the space the forward's rings take) and written
    // by one bulk copy (the rows of a group are contiguous).
    float* bstage = reinterpret_cast<float*>(smem_raw + fwd_stage_offset(wpc)) + warp * NPH * PF * SR;
    const uint32_t bstage_s = smem_addr(bstage);
    for (int i = threadIdx.x; i < wpc * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    cluster_sync_all();

    // Messages flow upward: the producer of this warp's input is warp g+1 (the
    // stripe below); this warp's output goes to warp g-1.
    const uint32_t my_consumed = smem_addr(consumed + warp);
    const uint64_t my_ring_g = reinterpret_cast<uint64_t>(ring + warp * kRing);
    const uint32_t my_ring_s = smem_addr(ring + warp * kRing);
    uint64_t up_ring_g = 0;
    uint32_t below_consumed = 0;
    if (g > 0) up_ring_g = mapa_generic(ring + ((g - 1) % wpc) * kRing, (g - 1) / wpc);
    if (g + 1 < P.G) below_consumed = mapa_shared(smem_addr(consumed + (g + 1) % wpc), (g + 1) / wpc);

    const float gb = a.grad_out ? __ldg(a.grad_out + b) : 1.f;
    const float NEG = neg_inf();
    const int ibw = a.ibw;
    WaitCtx wc = a.wait;
    wc.kernel = 2;
    wc.problem = b;
    wc.warp = g;
    bool ok = true;
    bool quit = false;
    uint32_t cons_seen = 0;  // lane 0: progress of the consumer above

    for (int band = P.n_bands - 1; band >= 0 && !quit; --band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) continue;
        wc.band = band;
        const int R0 = s * SR;
        const bool has_up = (s > 0) && (s != a.debug_stall);
        const bool up_wrap = (g == 0);
        const bool has_below = (s + 1 < P.n_stripes);
        const bool below_wrap = (g == P.G - 1);
        const uint32_t band_base = static_cast<uint32_t>(P.n_bands - 1 - band) * static_cast<uint32_t>(M);
        const size_t sb = stripe_base(P, b, s);
        float* Es = a.Ew + sb;
        const float2* Ts = a.score + sb;
        // Last row of the previous stripe, by column: Tp[col * SR].
        const float2* Tp = (s > 0) ? a.score + stripe_base(P, b, s - 1) + static_cast<size_t>(SR - 1) * SR + (K - 1) * 32 + 31
                                   : a.score;
        const uint64_t wrap_g = reinterpret_cast<uint64_t>(a.wrap + static_cast<size_t>(b) * 2 * M);
        const uint64_t in_g = below_wrap ? wrap_g : my_ring_g;
        const uint64_t out_g = up_wrap ? wrap_g : up_ring_g;
        const uint32_t in_tag_wrap = wrap_tag(a.seq, band + 1);
        const uint32_t out_tag_wrap = wrap_tag(a.seq, band);

        // Everything before this band counts as consumed: a warp whose stripe had
        // no producer below it in the previous (later-numbered) band never
        // advanced the counter, and the producer's flow control starts at band_base.
        st_release_cluster_u32_if(has_below && !below_wrap && lane == 31, below_consumed, band_base);

        const int n_steps = M + SR - 1;
        const int n_groups = (n_steps + PF - 1) / PF;
        const int t_last = n_groups * PF - 1;  // steps past n_steps - 1 touch cells outside the table
        // Band-limited launch: only the groups whose anti-diagonals hold an
        // in-band cell of this stripe run (group gi covers t_last - gi*PF down
        // to t_last - gi*PF - PF + 1); the rows outside are written as 0.
        int gi_begin = 0, gi_end = n_groups;
        if constexpr (BANDED) {
            const int t_lo = max(0, R0 - ibw);
            const int t_hi = min(n_steps - 1, (SR - 1) + min(M - 1, R0 + SR - 1 + ibw));
            gi_begin = ((t_last - t_hi) / PF) / NPH * NPH;
            gi_end = max(gi_begin, min(n_groups, (t_last - t_lo) / PF + 1));
        }
        const int t_top = t_last - gi_begin * PF;  // first (highest) step that runs
        // Columns of the row below that are in the band (and so sent by the
        // stripe below); messages for lower columns are zero without the ring.
        const int c_min = BANDED ? max(0, R0 + SR - ibw) : 0;
        // The columns above t_top - (SR - 1) are never read: report them
        // consumed, so that the stripe below may run up to a full ring ahead.
        if (t_top < t_last)
            st_relaxed_cluster_u32_if(has_below && !below_wrap && lane == 31, below_consumed,
                                      band_base + static_cast<uint32_t>(max(0, M - 1 - max(t_top - (SR - 1), -1))));
        // Queued loads: the step due in register slot j reads A(t-2) and
        // PS(t-1), refilled PD steps ahead from clamped (always valid)
        // addresses and used raw: a select on a loaded value would stall on the
        // load at issue.  Rows or
        // columns past either end only reach cells that are not live, or are
        // masked where they are consumed (the column -1 border below, and the
        // row above stripe 0, which is -inf).
        const bool ps_live = R0 > 0;
        const float2* Tl = Ts + lane;
        auto loadA = [&](int tp, int k) -> float2 {
            const int tc = min(max(tp, 0), n_steps - 1);
            return __ldg(Tl + static_cast<size_t>(tc) * SR + k * 32);
        };
        auto loadPS = [&](int col) -> float2 {
            const int cc = min(max(col, 0), M - 1);
            return __ldg(Tp + static_cast<size_t>(cc) * SR);
        };

        float2 aq[PD][K];  // A(t-2) for the step due in slot j
        float2 pq[PD];     // PS(t-1) for the step due in slot j
        float2 A1[K];      // A(t-1)
        float2 S1;         // row above at anti-diagonal t-1
#pragma unroll
        for (int j = 0; j < PD; ++j) {
            const int t = t_top - j;
#pragma unroll
            for (int k = 0; k < K; ++k) aq[j][k] = loadA(t - 2, k);
            pq[j] = loadPS(t - 1);
        }
#pragma unroll
        for (int k = 0; k < K; ++k) A1[k] = loadA(t_top - 1, k);
        const float2 ps = loadPS(t_top);
        S1.x = __shfl_up_sync(SDTW_FULL_MASK, A1[K - 1].x, 1);
        S1.y = __shfl_up_sync(SDTW_FULL_MASK, A1[K - 1].y, 1);
        if (lane == 0) S1 = ps_live ? ps : make_float2(NEG, 0.f);

        float accl[K], msg[K], dprev[K];
#pragma unroll
        for (int k = 0; k < K; ++k) accl[k] = msg[k] = dprev[k] = 0.f;
        const int q0 = lane * K;
        const int rows_left = N - R0;
        float* El = Es + lane;
        // Band-wrap input (global memory): the slots of the next group are
        // loaded one group ahead, as in the forward.
        uint64_t wpf = 0;
        {
            const int col = t_top - (SR - 1) - (lane & (PF - 1));
            if (has_below && below_wrap && col >= c_min && col < M) wpf = ld_one(in_g + static_cast<uint32_t>(col) * 16u);
        }

        auto group = [&](auto phase_c, int t0) {
            constexpr int PH = decltype(phase_c)::value;
            // ---- group prologue: messages for this lane's last row (lane 31),
            // columns colb(t) = t - (SR-1) for t = t0 .. t0-PF+1.
            // Lane u (mod PF) holds the message for column colb0 - u; step u
            // hands it to lane 31 with a shuffle of its own (measured on B200:
            // 5-18 % faster than broadcasting the group at once).
            float v = 0.f;
            const int colb0 = t0 - (SR - 1);
            if (has_below && colb0 - (PF - 1) < M && colb0 >= c_min) {  // warp-uniform
                bool all = true;
                auto probe = [&]() {
                    // Lane u (mod PF) reads slot u (one load instruction per group,
                    // as in the forward); once the tag vote has passed, step u hands
                    // slot u's value to lane 31.
                    const int u = lane & (PF - 1);
                    const int col = colb0 - u;
                    const uint32_t tg = below_wrap ? in_tag_wrap : band_base + static_cast<uint32_t>(M - 1 - col);
                    const uint32_t slot = below_wrap ? static_cast<uint32_t>(col) * 2u : (tg % kRing);
                    bool mine = true;
                    if (col >= c_min && col < M) {
                        const uint64_t e = below_wrap ? ld_one(in_g + slot * 8u) : ld_one_shared(my_ring_s + slot * 8u);
                        mine = tag_of(e) == tg;
                        v = val_of(e);
                    }
                    all = __all_sync(SDTW_FULL_MASK, mine);
                };
                if (below_wrap) {  // warp-uniform: the prefetched slots, then the next group's
                    const int col = colb0 - (lane & (PF - 1));
                    bool mine = true;
                    if (col >= c_min && col < M) {
                        mine = tag_of(wpf) == in_tag_wrap;
                        v = val_of(wpf);
                    }
                    all = __all_sync(SDTW_FULL_MASK, mine);
                    if (col - PF >= c_min && col - PF < M) wpf = ld_one(in_g + static_cast<uint32_t>(col - PF) * 16u);
                } else {
                    probe();
                }
                if (!all && ok) {  // uniform: the tag vote is warp-wide
                    uint64_t w0 = 0;
                    for (uint32_t it = 1;; ++it) {
                        probe();
                        if (all) break;
                        const int r = backoff(it, w0, wc);
                        if (r) {
                            if (lane == 0) record_giveup(wc, r, 1, static_cast<uint32_t>(colb0), 0);
                            ok = false;
                            break;
                        }
                    }
                }
                // Consumption counter: columns > colb0 - PF are now out of the ring.
                const int done = M - max(colb0 - PF + 1, 0);  // reversed columns consumed
                st_relaxed_cluster_u32_if(!below_wrap && lane == 31 && report_due(done, PF, M), below_consumed,
                                          band_base + static_cast<uint32_t>(done));
            }
            // ---- flow control for the messages this group publishes upward (lane 0, columns t0 .. t0-PF+1).
            if (has_up && !up_wrap) {  // warp-uniform
                const int col_last = max(t0 - (PF - 1), 0);
                if (col_last < M) {
                    const uint32_t gc = band_base + static_cast<uint32_t>(M - 1 - col_last);
                    if (__any_sync(SDTW_FULL_MASK, ok && gc >= static_cast<uint32_t>(kRing) &&
                                                       static_cast<int32_t>(cons_seen - (gc - kRing + 1)) < 0)) {
                        cons_seen = wait_counter_ge(my_consumed, gc - kRing + 1, wc);
                        ok = ok && static_cast<int32_t>(cons_seen - (gc - kRing + 1)) >= 0;
                    }
                }
            }
            // ---- PF reverse steps (step u fills staged row PF - 1 - u, i.e. t0 - u).
            if (lane == 0) bulk_wait_read<NPH - 1>();
            __syncwarp();
            float* Eg = bstage + PH * PF * SR + (PF - 1) * SR + lane;
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int t = t0 - u;
                constexpr int J0 = PH * PF;
                (void)J0;
                float2 A2[K];
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    A2[k] = aq[J0 + u][k];
                    aq[J0 + u][k] = loadA(t - 2 - PD, k);
                }
                float2 S2;
                {
                    const float2 ps = pq[J0 + u];
                    pq[J0 + u] = loadPS(t - 1 - PD);
                    S2.x = __shfl_up_sync(SDTW_FULL_MASK, A2[K - 1].x, 1);
                    S2.y = __shfl_up_sync(SDTW_FULL_MASK, A2[K - 1].y, 1);
                    S2.x = (lane == 0) ? (ps_live ? ps.x : NEG) : S2.x;
                    S2.y = (lane == 0) ? (ps_live ? ps.y : 0.f) : S2.y;
                }
                float below = __shfl_down_sync(SDTW_FULL_MASK, msg[0], 1);
                const float rv = __shfl_sync(SDTW_FULL_MASK, v, u);
                below = (lane == 31) ? rv : below;
                float nmsg[K];
#pragma unroll
                for (int k = K - 1; k >= 0; --k) {
                    const int q = q0 + k;
                    const int col = t - q;
                    const float in_below = (k == K - 1) ? below : msg[k < K - 1 ? k + 1 : 0];
                    float e = accl[k] + in_below;
                    float2 tl = A1[k];
                    float2 tu = (k == 0) ? S1 : A1[k > 0 ? k - 1 : 0];
                    float2 td = (k == 0) ? S2 : A2[k > 0 ? k - 1 : 0];
                    bool live = q < rows_left && static_cast<unsigned>(col) < static_cast<unsigned>(M);
                    if constexpr (BANDED)
                        live = live && static_cast<unsigned>(R0 + q - col + ibw) <= static_cast<unsigned>(2 * ibw);
                    e = (q == rows_left - 1 && col == M - 1) ? gb : e;
                    e = live ? e : 0.f;
                    // Predecessor scores; column -1 is the border (+inf R),
                    // except the corner (-1, -1) of row 0 (R = 0).
                    const bool c0 = (col == 0);
                    tl.x = c0 ? NEG : tl.x;
                    tl.y = c0 ? 0.f : tl.y;
                    td.x = c0 ? ((R0 + q == 0) ? 0.f : NEG) : td.x;
                    td.y = c0 ? 0.f : td.y;
                    Eg[-static_cast<ptrdiff_t>(u) * SR + k * 32] = e;
                    // Softmax of the predecessors' scores; the lo of the max cancels.
                    const float m = max3f(td.x, tu.x, tl.x);
                    const float ed = ex2f((td.x - m) + td.y);
                    const float eu = ex2f((tu.x - m) + tu.y);
                    const float el = ex2f((tl.x - m) + tl.y);
                    const float inv = live ? rcpf(ed + eu + el) : 0.f;
                    const float ei = e * inv;
                    accl[k] = ei * el;
                    nmsg[k] = fmaf(ei, eu, dprev[k]);
                    dprev[k] = ei * ed;
                }
                // Message of row 0 to the stripe above, column t.
                const bool pub = has_up && lane == 0 && static_cast<unsigned>(t) < static_cast<unsigned>(M);
                const uint32_t tgo = up_wrap ? out_tag_wrap : band_base + static_cast<uint32_t>(M - 1 - t);
                const uint32_t slot = up_wrap ? static_cast<uint32_t>(t) * 2u : (tgo % kRing);
                st_one_if(pub, out_g + slot * 8u, pack_tagged(nmsg[0], tgo));
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    msg[k] = nmsg[k];
                    A1[k] = A2[k];
                }
                S1 = S2;
            }
            // Rows t0 - PF + 1 .. t0 of E: one bulk copy.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_s2g(El - lane + static_cast<size_t>(t0 - PF + 1) * SR, bstage_s + PH * PF * SR * 4u, PF * SR * 4u);
                bulk_commit();
            }
        };
        using P0 = std::integral_constant<int, 0>;
        using P1 = std::integral_constant<int, 1>;
        for (int gi = gi_begin; gi < gi_end; gi += NPH) {
            const int t0 = t_last - gi * PF;
            group(P0{}, t0);
            if constexpr (NPH >= 2) {
                if (gi + 1 < gi_end) group(P1{}, t0 - PF);
            }
            if constexpr (NPH >= 4) {
                if (gi + 2 < gi_end) group(std::integral_constant<int, 2>{}, t0 - 2 * PF);
                if (gi + 3 < gi_end) group(std::integral_constant<int, 3>{}, t0 - 3 * PF);
            }
            if ((gi & 15) == 16 - NPH && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        // The band's copies are complete before the zero fill below and the
        // next band's first group.
        if (lane == 0) bulk_wait_all();
        cp_async_wait<0>();
        __syncwarp();
        // Rows outside the groups that ran (padding, or out of the band): zero,
        // like every cell outside the table.
        for (int t = 0; t <= t_last - gi_end * PF; ++t)
#pragma unroll
            for (int k = 0; k < K; ++k) El[static_cast<size_t>(t) * SR + k * 32] = 0.f;
        for (int t = t_top + 1; t < P.n_diag; ++t)
#pragma unroll
            for (int k = 0; k < K; ++k) El[static_cast<size_t>(t) * SR + k * 32] = 0.f;
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
    }
    cluster_sync_all();
}

// ============================================================== score <-> padded R
// R (B, N+2, M+2) in the reference launcher layout (launcher.py:55-56, 177-178):
// R[:,0,0] = 0, other borders +inf, interior R = -T * gamma * ln 2.
template <int K>
__global__ void score_to_R_kernel(const float2* __restrict__ S, float* __restrict__ R, WavePlan P, float inv_k) {
    const size_t total = static_cast<size_t>(P.B) * (P.N + 2) * (P.M + 2);
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(idx % (P.M + 2));
        const int i = static_cast<int>((idx / (P.M + 2)) % (P.N + 2));
        const int b = static_cast<int>(idx / (static_cast<size_t>(P.M + 2) * (P.N + 2)));
        float v;
        if (i == 0 && j == 0) {
            v = 0.f;
        } else if (i == 0 || j == 0 || i == P.N + 1 || j == P.M + 1) {
            v = pos_inf();
        } else {
            const float2 t = load_score<K>(S, P, b, i - 1, j - 1);
            v = (t.x == neg_inf()) ? pos_inf() : fmaf(-t.x, inv_k, -t.y * inv_k);
        }
        R[idx] = v;
    }
}

template <int K>
__global__ void R_to_score_kernel(const float* __restrict__ R, float2* __restrict__ S, WavePlan P, float kk) {
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
        float hi = -r * kk;
        float lo = fmaf(-r, kk, -hi);
        if (!(hi > neg_inf())) {  // R = +inf (unreachable or outside the band)
            hi = neg_inf();
            lo = 0.f;
        }
        S[((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + (q + col)) * SR + k * 32 + l] = make_float2(hi, lo);
    }
}

// ============================================================== launchers
static size_t ring_smem_bytes(const WavePlan& P) {
    return static_cast<size_t>(P.wpc) * 2 * kRing * 8u + static_cast<size_t>(P.wpc) * 4u;
}
// The reverse pass stages E rows ([wpc][phases][PF][32K] floats) at the same
// offset.
static size_t bwd_smem_bytes(const WavePlan& P) { return bwd_stage_end(P.wpc, P.K, P.K == 1 ? 1 : 2); }
// The forward adds its store staging ([wpc][phases][PF][32K] float2) and cost
// staging ([wpc][3][PF][32K] floats) after the ring.
static size_t fwd_smem_bytes(const WavePlan& P) {
    return fwd_cost_offset(P.wpc, P.K) + static_cast<size_t>(P.wpc) * 3 * fwd_pf(P.K) * 32 * P.K * 4u;
}

// Clusters of this geometry that can be resident at once on the current
// device for a pass (0: the forward kernels, 1: the reverse passes; the
// smaller figure of the pass's variants), or -1 if the runtime cannot tell.
// Clusters are placed within one GPC, so on B200 the figure can be below
// (SMs / cluster size).
int max_active_clusters(const WavePlan& P, int pass) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.csize);
    cfg.blockDim = dim3(P.wpc * 32);
    cfg.dynamicSmemBytes = ring_smem_bytes(P);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = P.csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // (kernel, dynamic shared memory, threads) of every pass this geometry may launch.
    const void* fns[4] = {nullptr, nullptr, nullptr, nullptr};
    size_t smem[4] = {0, 0, 0, 0};
    int threads[4] = {P.wpc * 32, P.wpc * 32, P.wpc * 32, P.wpc * 32};
    switch (P.K) {
        case 1: {
            const bool wide = pass >= 32 && pass < 64;
            const int fp = wide ? pass - 32 : pass;
            if (fp == 0) {
                fns[0] = fwdx_fn(false, false, 0, wide);
                smem[0] = fwdx_smem(P, 0, wide);
                threads[0] = fwdx_threads(P);
                fns[2] = fwdx_fn(false, true, 0, wide);
                smem[2] = fwdx_smem(P, 0, wide);
                threads[2] = fwdx_threads(P);
            } else if (pass >= 64) {
                fns[0] = bwdw_fn(false, pass - 64);
                smem[0] = bwdw_smem(P, pass - 64);
            } else if (fp >= 2) {
                fns[0] = fwdx_fn(false, true, fp - 2, wide);
                smem[0] = fwdx_smem(P, fp - 2, wide);
                threads[0] = fwdx_threads(P);
            } else {
                fns[1] = (const void*)bwd_kernel<1, false>;
                smem[1] = bwd_smem_bytes(P);
                fns[3] = bwdw_fn(false);
                smem[3] = bwdw_smem(P);
            }
            break;
        }
        case 2:
            fns[pass == 1] = pass != 1 ? (const void*)fwd_kernel<2, false> : (const void*)bwd_kernel<2, false>;
            smem[pass == 1] = pass != 1 ? fwd_smem_bytes(P) : bwd_smem_bytes(P);
            break;
        case 4:
            fns[pass == 1] = pass != 1 ? (const void*)fwd_kernel<4, false> : (const void*)bwd_kernel<4, false>;
            smem[pass == 1] = pass != 1 ? fwd_smem_bytes(P) : bwd_smem_bytes(P);
            break;
        default: return -1;
    }
    int best = -1;
    for (int i = 0; i < 4; ++i) {
        const void* fn = fns[i];
        if (!fn) continue;
        cfg.dynamicSmemBytes = smem[i];
        cfg.blockDim = dim3(threads[i]);
        if (cfg.dynamicSmemBytes > 48 * 1024 &&
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(cfg.dynamicSmemBytes)) != cudaSuccess) {
            (void)cudaGetLastError();
            return -1;
        }
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            return -1;
        }
        best = (best < 0 || n < best) ? n : best;
    }
    return best;
}

cudaError_t launch_forward(const FwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (P.K == 1) return launch_forward_x(args, stream);
    if (args.weights) return cudaErrorInvalidValue;
    // The band check runs only when a band can exclude a cell of the table.
    const bool banded = args.ibw < P.N + P.M;
    dim3 grid(P.B * P.csize), block(P.wpc * 32);
    void* kargs[] = {const_cast<FwdArgs*>(&args)};
    const void* fn = nullptr;
    switch (P.K) {
        case 2: fn = banded ? (const void*)fwd_kernel<2, true> : (const void*)fwd_kernel<2, false>; break;
        case 4: fn = banded ? (const void*)fwd_kernel<4, true> : (const void*)fwd_kernel<4, false>; break;
        default: return cudaErrorInvalidValue;
    }
    return launch_cluster(fn, grid, block, fwd_smem_bytes(P), P.csize, stream, kargs);
}

cudaError_t launch_backward(const BwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (args.weights) return launch_backward_w(args, stream);
    const bool banded = args.ibw < P.N + P.M;
    dim3 grid(P.B * P.csize), block(P.wpc * 32);
    void* kargs[] = {const_cast<BwdArgs*>(&args)};
    const void* fn = nullptr;
    switch (P.K) {
        case 1: fn = banded ? (const void*)bwd_kernel<1, true> : (const void*)bwd_kernel<1, false>; break;
        case 2: fn = banded ? (const void*)bwd_kernel<2, true> : (const void*)bwd_kernel<2, false>; break;
        case 4: fn = banded ? (const void*)bwd_kernel<4, true> : (const void*)bwd_kernel<4, false>; break;
        default: return cudaErrorInvalidValue;
    }
    return launch_cluster(fn, grid, block, bwd_smem_bytes(P), P.csize, stream, kargs);
}

cudaError_t launch_score_to_R(const float2* S, float* R, const WavePlan& P, float inv_k, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(P.B) * (P.N + 2) * (P.M + 2);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<size_t>((total + threads - 1) / threads, 148u * 16u));
    switch (P.K) {
        case 1: score_to_R_kernel<1><<<blocks, threads, 0, stream>>>(S, R, P, inv_k); break;
        case 2: score_to_R_kernel<2><<<blocks, threads, 0, stream>>>(S, R, P, inv_k); break;
        case 4: score_to_R_kernel<4><<<blocks, threads, 0, stream>>>(S, R, P, inv_k); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_R_to_score(const float* R, float2* S, const WavePlan& P, float kk, cudaStream_t stream) {
    const size_t total = static_cast<size_t>(P.B) * P.N * P.M;
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<size_t>((total + threads - 1) / threads, 148u * 16u));
    switch (P.K) {
        case 1: R_to_score_kernel<1><<<blocks, threads, 0, stream>>>(R, S, P, kk); break;
        case 2: R_to_score_kernel<2><<<blocks, threads, 0, stream>>>(R, S, P, kk); break;
        case 4: R_to_score_kernel<4><<<blocks, threads, 0, stream>>>(R, S, P, kk); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sdtw
