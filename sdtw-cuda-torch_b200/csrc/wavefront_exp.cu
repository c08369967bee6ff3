// wavefront_exp.cu -- the one-row-per-lane Soft-DTW wavefronts of sm_100a:
// the forward in the exponential domain (fwdx_kernel) and the reverse pass
// over the forward's predecessor weights (bwdw_kernel).
//
// Semantics follow the reference recurrences
//   forward   softdtw_cuda/cuda/kernels.py:126-187, launcher.py:307-324
//             R[i,j] = D[i-1,j-1] + softmin_gamma(R[i-1,j-1], R[i-1,j], R[i,j-1])
//   backward  softdtw_cuda/cuda/kernels.py:216-307, launcher.py:327-353
//             E[i,j] = sum over successors c of E[c] * exp((R[c] - D[c] - R[i,j]) / gamma)
// with R[0,0] = 0, the other borders +inf and band-pruned cells +inf.
//
// Exponential domain.  With P = exp(-R / gamma) the forward recurrence is
// linear:  P[i,j] = K[i,j] * (P[i-1,j-1] + P[i-1,j] + P[i,j-1]),
// K = exp(-D / gamma) = 2^(-D * log2(e) / gamma).  P spans far more than the
// float32 exponent range (R / gamma reaches 1e5 at B=32, N=M=512, D=64), so a
// cell holds a software float: a float32 mantissa m >= 1 and an int32
// exponent e, P = m * 2^e.  One cell is then
//   emax = max of the three predecessors' exponents,
//   each term m_k * K_mantissa scaled by 2^(e_k - emax) through an integer add
//   to its exponent field (terms below 2^-96 of the largest are dropped),
//   two float adds, and e = emax + K_exponent:
// a shuffle, an integer max, an integer add-max, an integer add and two float
// adds on the dependent chain, where the log-domain softmin needs two MUFU
// operations (ex2, lg2) there.  K's split into mantissa and exponent
// (one ex2) depends only on the cost and runs off the chain.  Mantissas grow
// by at most 6x a step and every held value is renormalised once per group of
// 8 steps.  The scaled terms are exact, so the weights of the reverse pass (a
// predecessor's term over their sum) have float32 relative accuracy at any
// magnitude of R.
// Valid exponents stay within +-2^29 (|R| / gamma < 3.7e8) and |D| * log2(e)
// / gamma below 2^22 per cell; a launch that leaves that range, or meets a NaN
// cost, records status 4 (value range) instead of returning wrong values
// silently.
//
// Reverse pass.  The reference's weight exp((R[c] - D[c] - R[p]) / gamma)
// equals the share of predecessor p in c's sum, so the forward stores each
// cell's (diagonal, upper) shares (the left one is 1 minus both) and the
// reverse step is three multiply-adds and a shuffle.  The D-input entry
// points, which hand the score table T = -R log2(e) / gamma to the caller,
// store T (as an unevaluated float32 pair) instead; their reverse pass
// recomputes the shares from T (bwd_kernel in wavefront.cu).
//
// Parallel structure (shared with wavefront.cu).  One warp owns a stripe of 32
// rows, one row per lane, and sweeps its anti-diagonals; the row above comes
// from the neighbour lane by shuffle, and for lane 0 from the previous
// stripe's warp through a ring of tagged u64 slots in the consumer's shared
// memory (DSMEM stores inside a thread-block cluster; a global ring between
// bands).  Steps run in groups of 8: per group the consumer checks the 8 ring
// slots it needs with one warp-wide load and a vote, the producer checks flow
// control once and publishes the stripe's bottom row for the group's 8
// columns with one warp-wide store, the cost rows of the group after next are
// copied into shared memory (cp.async), and the group's table rows leave as
// one bulk copy (cp.async.bulk).  Groups whose cells all lie inside the table
// run without masks.
#include <type_traits>

#include "sdtw_device.cuh"
#include "sdtw_kernels.h"
#include "sdtw_plan.h"
#include "wavefront_ring.cuh"

namespace sdtw {

namespace {
constexpr int kPF = 8;                   // steps per group
constexpr int kEneg = -(1 << 30);        // exponent of P = 0 (outside the table or the band)
constexpr int kShiftMin = -96;           // terms below 2^-96 of the largest are dropped
constexpr int kErange = 1 << 29;         // valid exponents lie in (-2^29, 2^29)
constexpr float kPmax = 4194304.f;       // |D| * log2(e) / gamma per cell must stay below 2^22
constexpr float kMagic = 12582912.f;     // 1.5 * 2^23: adding it rounds to an integer in the low bits
constexpr int kFwdStages = 2;            // forward: table-row staging buffers
constexpr int kBwdPhases = 2;            // reverse pass: E staging buffers (step bodies)
}  // namespace

// m * 2^s for s <= 0 by an add to the exponent field.  m is a normal float
// >= 1 below 2^26 and s >= kShiftMin, so the result is a normal float.
__device__ __forceinline__ float scale_pow2(float m, int s) {
    return __int_as_float(__float_as_int(m) + s * (1 << 23));
}

// NaN-propagating maximum (a NaN cost must not disappear from the range check).
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// The score T = e + log2(m) as an unevaluated float32 pair (hi, lo).  The
// exponent goes in as two exactly representable parts.
__device__ __forceinline__ float2 to_score(float m, int e) {
    const float l = lg2f(m);
    const float eh = static_cast<float>(e & ~0xfff);
    const float el = static_cast<float>(e & 0xfff);
    const float s1 = el + l;
    const float b1 = s1 - el;
    const float r1 = (el - (s1 - b1)) + (l - b1);
    const float hi = eh + s1;
    const float b2 = hi - eh;
    const float r2 = (eh - (hi - b2)) + (s1 - b2);
    return make_float2(hi, r1 + r2);
}

// ------------------------------------------------------------------ forward
// Shared memory: rings [wpc][kRing][2] u64 and counters [wpc] u32 (as in
// wavefront.cu), then per warp: the staged table rows of two groups
// [2][PF][32] float2 (a group's rows are written while the previous group's
// bulk copy still reads its buffer), the cost rows of three groups [3][PF][32]
// float, and the ring input and bottom-row output of one group [2][PF] uint2.
__host__ __device__ constexpr size_t fx_cost_off(int wpc) {
    return fwd_stage_offset(wpc) + static_cast<size_t>(wpc) * kFwdStages * kPF * 32 * 8;
}
__host__ __device__ constexpr size_t fx_stash_off(int wpc) {
    return fx_cost_off(wpc) + static_cast<size_t>(wpc) * 3 * kPF * 32 * 4;
}
__host__ __device__ constexpr size_t fx_smem_bytes(int wpc) {
    return fx_stash_off(wpc) + static_cast<size_t>(wpc) * 2 * kPF * 8;
}

__device__ __forceinline__ uint64_t pack_tagged_bits(uint32_t v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | static_cast<uint64_t>(v);
}

template <bool BANDED, bool W>
__global__ void __launch_bounds__(512) fwdx_kernel(const FwdArgs a) {
    constexpr int PF = kPF;
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
    float2* stage = reinterpret_cast<float2*>(smem_raw + fwd_stage_offset(wpc)) + warp * kFwdStages * PF * 32;
    const uint32_t stage_s = smem_addr(stage);
    const float* cost = reinterpret_cast<const float*>(smem_raw + fx_cost_off(wpc)) + warp * 3 * PF * 32;
    const uint32_t cost_s = smem_addr(cost);
    uint2* rin_s = reinterpret_cast<uint2*>(smem_raw + fx_stash_off(wpc)) + warp * 2 * PF;  // ring input (m, e)
    uint2* pub_s = rin_s + PF;                                                                  // bottom row (m, e)
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
    const int ibw = a.ibw;
    WaitCtx wc = a.wait;
    wc.kernel = 1;
    wc.problem = b;
    wc.warp = g;
    bool ok = true;          // false once a wait of this lane failed
    bool quit = false;       // warp-uniform
    bool bad = false;        // a valid exponent left its range
    float pmax = 0.f;        // largest |D| * log2(e) / gamma of a live cell (NaN if one was NaN)
    uint32_t cons_seen = 0;  // consumer progress last observed

    for (int band = 0; band < P.n_bands && !quit; ++band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) break;
        wc.band = band;
        const int R0 = s * 32;
        const bool has_in = R0 > 0;
        const bool in_wrap = (g == 0);
        const bool has_out = (s + 1 < P.n_stripes) && (s != a.debug_stall);
        const bool out_wrap = (g == P.G - 1);
        const uint32_t band_base = static_cast<uint32_t>(band) * static_cast<uint32_t>(M);
        const size_t sb = stripe_base(P, b, s);
        float2* Tl = a.score + sb + lane;  // this lane's position of anti-diagonal row 0
        const float* Dl = a.Dw + sb;
        const uint64_t wrap_g = reinterpret_cast<uint64_t>(a.wrap + static_cast<size_t>(b) * 2 * M);
        const uint64_t out_g = out_wrap ? wrap_g : next_ring_g;
        const uint32_t in_tag_wrap = wrap_tag(a.seq, band - 1);
        const uint32_t out_tag_wrap = wrap_tag(a.seq, band);

        // Everything before this band counts as consumed.
        st_release_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed, band_base);

        const int n_steps = M + 31;
        const int n_groups = (n_steps + PF - 1) / PF;
        // Band-limited launch: only the groups whose anti-diagonals hold an
        // in-band cell of this stripe run (one step early, so that the first
        // in-band cell has its diagonal predecessor); the rows outside are
        // written as cells outside the table.
        int g_begin = 0, g_end = n_groups;
        if constexpr (BANDED) {
            const int t_lo = max(0, R0 - ibw - 1);
            const int t_hi = min(n_steps - 1, 31 + min(M - 1, R0 + 31 + ibw));
            g_begin = t_lo / PF;
            g_end = max(g_begin, min(n_groups, t_hi / PF + 1));
        }
        const int t_begin = g_begin * PF;
        // Last column of the row above that is in the band (and so published
        // by the stripe above); the columns past it read as P = 0.
        const int c_pub_max = BANDED ? min(M - 1, R0 - 1 + ibw) : M - 1;
        // Group gg's cost rows (PF * 32 contiguous floats), or an empty commit
        // past the last group, so that every group finds its rows two commits back.
        auto cost_copy = [&](int gg) {
            if (gg < g_end) {
                const float* src = Dl + static_cast<size_t>(gg) * PF * 32;
                const uint32_t dst = cost_s + static_cast<uint32_t>((gg - g_begin) % 3) * PF * 32 * 4u;
#pragma unroll
                for (int i = 0; i < PF * 32 / 128; ++i) cp_async16(dst + (lane + 32 * i) * 16u, src + (lane + 32 * i) * 4);
            }
            cp_async_commit();
        };
        cost_copy(g_begin);
        cost_copy(g_begin + 1);
        if (t_begin > 0)
            st_relaxed_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed,
                                      band_base + static_cast<uint32_t>(min(t_begin, M)));

        // Cell state: own previous cell (left neighbour of the next step) and
        // the upper neighbour of the previous step (diagonal of the next).
        float m_l = 1.f;
        int e_l = kEneg;
        float m_d = 1.f;
        int e_d = (R0 == 0 && lane == 0) ? 0 : kEneg;  // R[0,0] = 0 above-left of cell (0, 0)
        const int rows_left = N - R0;
        const bool full_rows = rows_left >= 32;
        const int l_last = N - 1 - R0;
        const int t_last = (s == P.n_stripes - 1 && lane == l_last) ? l_last + M - 1 : -1;
        float last_m = 1.f;
        int last_e = kEneg;
        // Band-wrap input (global memory, an L2 round trip per load): the slots
        // of the next group are loaded one group ahead.
        uint64_t wpf_h = 0, wpf_l = 0;
        if (has_in && in_wrap && t_begin < M && t_begin + (lane & (PF - 1)) <= c_pub_max)
            ld_pair(wrap_g + static_cast<uint32_t>(t_begin + (lane & (PF - 1))) * 16u, wpf_h, wpf_l);

        auto group = [&](auto masked_c, int t0) {
            constexpr bool MASKED = decltype(masked_c)::value;
            // ---- ring input: the row above for columns t0 .. t0+PF-1, slot u
            // read by lane u (mod PF), kept in shared memory for lane 0's steps.
            {
                uint32_t vm = __float_as_uint(1.f), ve = static_cast<uint32_t>(kEneg);
                if (has_in && t0 < M && t0 <= c_pub_max) {  // warp-uniform
                    const int u = lane & (PF - 1);
                    const int col = t0 + u;
                    const uint32_t tg0 = in_wrap ? in_tag_wrap : band_base + static_cast<uint32_t>(t0);
                    bool all = true;
                    auto probe = [&]() {
                        const uint32_t tg = in_wrap ? tg0 : tg0 + static_cast<uint32_t>(u);
                        bool mine = true;
                        if (col <= c_pub_max) {
                            uint64_t eh, el;
                            if (in_wrap) ld_pair(wrap_g + static_cast<uint32_t>(col) * 16u, eh, el);
                            else ld_pair_shared(my_ring_s + (tg % kRing) * 16u, eh, el);
                            mine = tag_of(eh) == tg && tag_of(el) == tg;
                            vm = static_cast<uint32_t>(eh);
                            ve = static_cast<uint32_t>(el);
                        }
                        all = __all_sync(SDTW_FULL_MASK, mine);
                    };
                    if (in_wrap) {  // the prefetched slots, then the next group's
                        bool mine = true;
                        if (col <= c_pub_max) {
                            mine = tag_of(wpf_h) == tg0 && tag_of(wpf_l) == tg0;
                            vm = static_cast<uint32_t>(wpf_h);
                            ve = static_cast<uint32_t>(wpf_l);
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
                    const int done = min(t0 + PF, M);
                    st_relaxed_cluster_u32_if(!in_wrap && report_due(done, PF, M) && lane == 0, prev_consumed,
                                              band_base + static_cast<uint32_t>(done));
                }
                if (lane < PF) rin_s[lane] = make_uint2(vm, ve);
            }
            // ---- flow control for the columns this group publishes.
            if (has_out && !out_wrap) {  // warp-uniform
                const int col_last = min(t0 + PF - 1 - 31, M - 1);
                if (col_last >= 0) {
                    const uint32_t gc = band_base + static_cast<uint32_t>(col_last);
                    if (__any_sync(SDTW_FULL_MASK, ok && gc >= static_cast<uint32_t>(kRing) &&
                                                       static_cast<int32_t>(cons_seen - (gc - kRing + 1)) < 0)) {
                        cons_seen = wait_counter_ge(my_consumed, gc - kRing + 1, wc);
                        ok = ok && static_cast<int32_t>(cons_seen - (gc - kRing + 1)) >= 0;
                    }
                }
            }
            // ---- PF steps.  This group's staging buffer was last read by the
            // bulk copy of two groups ago; its cost rows (two commits back) have landed.
            const int gg = t0 / PF;
            const int sbuf = gg & (kFwdStages - 1);
            if (lane == 0) bulk_wait_read<kFwdStages - 1>();
            cp_async_wait<1>();
            __syncwarp();
            const float* cb = cost + ((gg - g_begin) % 3) * PF * 32 + lane;
            cost_copy(gg + 2);  // into the buffer the previous group read
            float2* Tg = stage + sbuf * PF * 32 + lane;
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int t = t0 + u;
                // K = 2^(-c * kk) = km * 2^ke, off the dependent chain.
                const float c = cb[u * 32];
                const float p = c * kk;
                const float r = __fadd_rd(-p, kMagic);
                const float fl = r - kMagic;
                const int ke = __float_as_int(r) - __float_as_int(kMagic);
                const float km = ex2f(fmaf(-c, kk, -fl));
                const uint2 ri = rin_s[u];
                float mu = __shfl_up_sync(SDTW_FULL_MASK, m_l, 1);
                int eu = __shfl_up_sync(SDTW_FULL_MASK, e_l, 1);
                mu = (lane == 0) ? __uint_as_float(ri.x) : mu;
                eu = (lane == 0) ? static_cast<int>(ri.y) : eu;
                const int emax = max(eu, max(e_d, e_l));
                const float vl = scale_pow2(m_l * km, __viaddmax_s32(e_l, -emax, kShiftMin));
                const float vd = scale_pow2(m_d * km, __viaddmax_s32(e_d, -emax, kShiftMin));
                const float vu = scale_pow2(mu * km, __viaddmax_s32(eu, -emax, kShiftMin));
                const float sum = (vl + vd) + vu;
                float mn = sum;
                int en = emax + ke;
                float pa = fabsf(p);
                if constexpr (!W) {
                    // Caller-supplied costs may be +inf (a forbidden cell): P = 0.
                    const bool cinf = c == pos_inf();
                    mn = cinf ? 1.f : mn;
                    en = cinf ? kEneg : en;
                    pa = cinf ? 0.f : pa;
                }
                float2 rec;
                if constexpr (W) {
                    // The shares of the diagonal and upper predecessors: all the
                    // reverse pass needs of this cell.
                    const float inv = rcpf(sum);
                    rec = make_float2(vd * inv, vu * inv);
                } else {
                    rec = (en == kEneg) ? make_float2(neg_inf(), 0.f) : to_score(mn, en);
                }
                if constexpr (MASKED) {
                    // Cells outside the table or the band: P = 0, shares 0.
                    const int col = t - lane;
                    bool live = static_cast<unsigned>(col) < static_cast<unsigned>(M) && lane < rows_left;
                    if constexpr (BANDED)
                        live = live && static_cast<unsigned>(R0 + lane - col + ibw) <= static_cast<unsigned>(2 * ibw);
                    mn = live ? mn : 1.f;
                    en = live ? en : kEneg;
                    rec = live ? rec : (W ? make_float2(0.f, 0.f) : make_float2(neg_inf(), 0.f));
                    pmax = live ? max_nan(pmax, pa) : pmax;
                    last_m = (t == t_last) ? mn : last_m;
                    last_e = (t == t_last) ? en : last_e;
                } else {
                    pmax = max_nan(pmax, pa);
                }
                Tg[u * 32] = rec;
                if (lane == 31) pub_s[u] = make_uint2(__float_as_uint(mn), static_cast<uint32_t>(en));
                m_d = mu;
                e_d = eu;
                m_l = mn;
                e_l = en;
            }
            // ---- renormalise the mantissas the next group starts from: the own
            // cell and the upper neighbour that becomes its diagonal.  (A value
            // moving down the diagonal passes from lane to lane every two
            // steps; at every group boundary it sits in one of the two, so each
            // value is renormalised at least once per group and grows by at
            // most 6x a step in between.)
            {
                const int bl = __float_as_int(m_l);
                e_l += (bl >> 23) - 127;
                m_l = __int_as_float((bl & 0x007fffff) | 0x3f800000);
                const int bd = __float_as_int(m_d);
                e_d += (bd >> 23) - 127;
                m_d = __int_as_float((bd & 0x007fffff) | 0x3f800000);
            }
            bad = bad || (e_l != kEneg && static_cast<unsigned>(e_l + kErange) > static_cast<unsigned>(2 * kErange));
            fence_proxy_async_smem();
            __syncwarp();
            // ---- the stripe's bottom row for columns t0-31 .. t0-31+PF-1: lane u
            // stores column t0 - 31 + u (both halves tagged).
            if (has_out) {  // warp-uniform
                const int colb = t0 - 31 + lane;
                const bool pub = lane < PF && static_cast<unsigned>(colb) < static_cast<unsigned>(M);
                const uint2 pv = pub_s[lane & (PF - 1)];
                const uint32_t tgo = out_wrap ? out_tag_wrap : band_base + static_cast<uint32_t>(colb);
                const uint32_t slot = out_wrap ? static_cast<uint32_t>(colb) : (tgo % kRing);
                st_pair_if(pub, out_g + slot * 16u, pack_tagged_bits(pv.x, tgo), pack_tagged_bits(pv.y, tgo));
            }
            // Rows t0 .. t0 + PF - 1 of the table: one bulk copy.
            if (lane == 0) {
                bulk_s2g(Tl - lane + static_cast<size_t>(t0) * 32, stage_s + sbuf * PF * 32 * 8u, PF * 32 * 8u);
                bulk_commit();
            }
        };
        for (int gi = g_begin; gi < g_end; ++gi) {
            const int t0 = gi * PF;
            if constexpr (!BANDED) {
                const bool interior = full_rows && t0 >= 32 && t0 + PF <= M;
                if (interior) group(std::false_type{}, t0);
                else group(std::true_type{}, t0);
            } else {
                group(std::true_type{}, t0);
            }
            if ((gi & 15) == 15 && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
        // The band's copies are complete before the fill stores below and the
        // next band's first group (which reuses the staging and cost buffers).
        if (lane == 0) bulk_wait_all();
        cp_async_wait<0>();
        __syncwarp();
        // Rows outside the groups that ran (padding, or out of the band).
        const float2 fill = W ? make_float2(0.f, 0.f) : make_float2(neg_inf(), 0.f);
        for (int t = 0; t < t_begin; ++t) Tl[static_cast<size_t>(t) * 32] = fill;
        for (int t = g_end * PF; t < P.n_diag; ++t) Tl[static_cast<size_t>(t) * 32] = fill;
        if (!quit && t_last >= 0)
            a.out[b] = (last_e == kEneg) ? pos_inf()
                                         : static_cast<float>(-(static_cast<double>(last_e) +
                                                                static_cast<double>(lg2f(last_m))) * a.inv_k_d);
    }
    if (__any_sync(SDTW_FULL_MASK, bad || !(pmax < kPmax)) && lane == 0) record_range(wc);
    // No CTA may leave while a peer can still write into its shared memory.
    cluster_sync_all();
}

// ------------------------------------------------------------------ reverse pass (weights)
// Shared memory: rings [wpc][kRing] u64 and counters [wpc] u32, then (at the
// forward's staging offset) per warp the E rows of kBwdPhases groups [ph][PF][32]
// float, the weights of three groups [3][PF][32] float2 and the messages of
// one group [PF] float.
__host__ __device__ constexpr size_t bw_w_off(int wpc) {
    return fwd_stage_offset(wpc) + static_cast<size_t>(wpc) * kBwdPhases * kPF * 32 * 4;
}
__host__ __device__ constexpr size_t bw_stash_off(int wpc) {
    return bw_w_off(wpc) + static_cast<size_t>(wpc) * 3 * kPF * 32 * 8;
}
__host__ __device__ constexpr size_t bw_smem_bytes(int wpc) {
    return bw_stash_off(wpc) + static_cast<size_t>(wpc) * kPF * 4;
}

// Reverse wavefront over the forward's shares.  At reverse step t the lane of
// row q handles cell (q, t - q):
//   E = (E of the right neighbour) * its left share       (accl, same lane)
//     + message from the row below: E(q+1, j) * upper share of (q+1, j)
//                                  + E(q+1, j+1) * diagonal share of (q+1, j+1)
// E(N-1, M-1) = grad_out[b] (autograd.py:46-47 multiplies it in).
template <bool BANDED>
__global__ void __launch_bounds__(512) bwdw_kernel(const BwdArgs a) {
    constexpr int PF = kPF;
    constexpr int NPH = kBwdPhases;
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
    float* bstage = reinterpret_cast<float*>(smem_raw + fwd_stage_offset(wpc)) + warp * NPH * PF * 32;
    const uint32_t bstage_s = smem_addr(bstage);
    const float2* wbuf = reinterpret_cast<const float2*>(smem_raw + bw_w_off(wpc)) + warp * 3 * PF * 32;
    const uint32_t wbuf_s = smem_addr(wbuf);
    float* pub_s = reinterpret_cast<float*>(smem_raw + bw_stash_off(wpc)) + warp * PF;
    for (int i = threadIdx.x; i < wpc * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    cluster_sync_all();

    // Messages flow upward: this warp's input comes from warp g+1 (the stripe
    // below), its output goes to warp g-1.
    const uint32_t my_consumed = smem_addr(consumed + warp);
    const uint64_t my_ring_g = reinterpret_cast<uint64_t>(ring + warp * kRing);
    const uint32_t my_ring_s = smem_addr(ring + warp * kRing);
    uint64_t up_ring_g = 0;
    uint32_t below_consumed = 0;
    if (g > 0) up_ring_g = mapa_generic(ring + ((g - 1) % wpc) * kRing, (g - 1) / wpc);
    if (g + 1 < P.G) below_consumed = mapa_shared(smem_addr(consumed + (g + 1) % wpc), (g + 1) / wpc);

    const float gb = a.grad_out ? __ldg(a.grad_out + b) : 1.f;
    const int ibw = a.ibw;
    WaitCtx wc = a.wait;
    wc.kernel = 2;
    wc.problem = b;
    wc.warp = g;
    bool ok = true;
    bool quit = false;
    uint32_t cons_seen = 0;

    for (int band = P.n_bands - 1; band >= 0 && !quit; --band) {
        const int s = band * P.G + g;
        if (s >= P.n_stripes) continue;
        wc.band = band;
        const int R0 = s * 32;
        const bool has_up = (s > 0) && (s != a.debug_stall);
        const bool up_wrap = (g == 0);
        const bool has_below = (s + 1 < P.n_stripes);
        const bool below_wrap = (g == P.G - 1);
        const uint32_t band_base = static_cast<uint32_t>(P.n_bands - 1 - band) * static_cast<uint32_t>(M);
        const size_t sb = stripe_base(P, b, s);
        float* El = a.Ew + sb + lane;
        const float2* Ts = a.score + sb;
        const uint64_t wrap_g = reinterpret_cast<uint64_t>(a.wrap + static_cast<size_t>(b) * 2 * M);
        const uint64_t in_g = below_wrap ? wrap_g : my_ring_g;
        const uint64_t out_g = up_wrap ? wrap_g : up_ring_g;
        const uint32_t in_tag_wrap = wrap_tag(a.seq, band + 1);
        const uint32_t out_tag_wrap = wrap_tag(a.seq, band);

        // Everything before this band counts as consumed.
        st_release_cluster_u32_if(has_below && !below_wrap && lane == 31, below_consumed, band_base);

        const int n_steps = M + 31;
        const int n_groups = (n_steps + PF - 1) / PF;
        const int t_last = n_groups * PF - 1;  // steps past n_steps - 1 touch cells outside the table
        // Band-limited launch: group gi covers steps t_last - gi*PF down to
        // t_last - gi*PF - PF + 1; the rows outside the groups that run are zero.
        int gi_begin = 0, gi_end = n_groups;
        if constexpr (BANDED) {
            const int t_lo = max(0, R0 - ibw);
            const int t_hi = min(n_steps - 1, 31 + min(M - 1, R0 + 31 + ibw));
            gi_begin = ((t_last - t_hi) / PF) / NPH * NPH;
            gi_end = max(gi_begin, min(n_groups, (t_last - t_lo) / PF + 1));
        }
        const int t_top = t_last - gi_begin * PF;  // first (highest) step that runs
        // Columns of the row below that are in the band (sent by the stripe below).
        const int c_min = BANDED ? max(0, R0 + 32 - ibw) : 0;
        if (t_top < t_last)
            st_relaxed_cluster_u32_if(has_below && !below_wrap && lane == 31, below_consumed,
                                      band_base + static_cast<uint32_t>(max(0, M - 1 - max(t_top - 31, -1))));
        // Group gi's shares: rows t0 - PF + 1 .. t0 (t0 = t_last - gi * PF),
        // or an empty commit past the last group.
        auto wcopy = [&](int gi) {
            if (gi < gi_end) {
                const float2* src = Ts + static_cast<size_t>(t_last - gi * PF - PF + 1) * 32;
                const uint32_t dst = wbuf_s + static_cast<uint32_t>((gi - gi_begin) % 3) * PF * 32 * 8u;
#pragma unroll
                for (int i = 0; i < PF * 32 / 64; ++i) cp_async16(dst + (lane + 32 * i) * 16u, src + (lane + 32 * i) * 2);
            }
            cp_async_commit();
        };
        wcopy(gi_begin);
        wcopy(gi_begin + 1);

        float accl = 0.f, msg = 0.f, dprev = 0.f;
        const int rows_left = N - R0;
        const bool full_rows = rows_left >= 32;
        // Band-wrap input (global memory): the slots of the next group are
        // loaded one group ahead.
        uint64_t wpf = 0;
        {
            const int col = t_top - 31 - (lane & (PF - 1));
            if (has_below && below_wrap && col >= c_min && col < M) wpf = ld_one(in_g + static_cast<uint32_t>(col) * 16u);
        }

        auto group = [&](auto phase_c, auto masked_c, int t0) {
            constexpr int PH = decltype(phase_c)::value;
            constexpr bool MASKED = decltype(masked_c)::value;
            // ---- messages for lane 31 (columns colb0 .. colb0-PF+1); lane u
            // (mod PF) holds column colb0 - u, handed to lane 31 at step u.
            float v = 0.f;
            const int colb0 = t0 - 31;
            if (has_below && colb0 - (PF - 1) < M && colb0 >= c_min) {  // warp-uniform
                bool all = true;
                const int u = lane & (PF - 1);
                const int col = colb0 - u;
                auto probe = [&]() {
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
                if (below_wrap) {
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
                if (!all && ok) {
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
                const int done = M - max(colb0 - PF + 1, 0);  // reversed columns consumed
                st_relaxed_cluster_u32_if(!below_wrap && lane == 31 && report_due(done, PF, M), below_consumed,
                                          band_base + static_cast<uint32_t>(done));
            }
            // ---- flow control for the messages this group publishes upward
            // (columns t0 .. t0-PF+1).
            if (has_up && !up_wrap) {
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
            cp_async_wait<1>();  // this group's shares, committed two groups back
            __syncwarp();
            const int gi = (t_last - t0) / PF;
            const float2* wb = wbuf + ((gi - gi_begin) % 3) * PF * 32 + (PF - 1) * 32 + lane;
            wcopy(gi + 2);  // into the buffer the previous group read
            float* Eg = bstage + PH * PF * 32 + (PF - 1) * 32 + lane;
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int t = t0 - u;
                const float2 w = wb[-u * 32];  // (diagonal, upper) shares of cell (lane, t - lane)
                float below = __shfl_down_sync(SDTW_FULL_MASK, msg, 1);
                const float rv = __shfl_sync(SDTW_FULL_MASK, v, u);
                below = (lane == 31) ? rv : below;
                float e = accl + below;
                if constexpr (MASKED) {
                    const int col = t - lane;
                    bool live = lane < rows_left && static_cast<unsigned>(col) < static_cast<unsigned>(M);
                    if constexpr (BANDED)
                        live = live && static_cast<unsigned>(R0 + lane - col + ibw) <= static_cast<unsigned>(2 * ibw);
                    e = (lane == rows_left - 1 && col == M - 1) ? gb : e;
                    e = live ? e : 0.f;
                }
                Eg[-u * 32] = e;
                const float dn = e * w.x;            // to the diagonal predecessor (two steps on)
                msg = fmaf(e, w.y, dprev);           // to the row above: upper share + previous diagonal
                accl = fmaf(-e, w.y, e - dn);        // left share: e * (1 - wd - wu)
                dprev = dn;
                if (lane == 0) pub_s[u] = msg;
            }
            __syncwarp();
            // ---- messages of row 0 to the stripe above: lane u stores column t0 - u.
            if (has_up) {
                const int col = t0 - lane;
                const bool pub = lane < PF && static_cast<unsigned>(col) < static_cast<unsigned>(M);
                const float pv = pub_s[lane & (PF - 1)];
                const uint32_t tgo = up_wrap ? out_tag_wrap : band_base + static_cast<uint32_t>(M - 1 - col);
                const uint32_t slot = up_wrap ? static_cast<uint32_t>(col) * 2u : (tgo % kRing);
                st_one_if(pub, out_g + slot * 8u, pack_tagged(pv, tgo));
            }
            // Rows t0 - PF + 1 .. t0 of E: one bulk copy.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_s2g(El - lane + static_cast<size_t>(t0 - PF + 1) * 32, bstage_s + PH * PF * 32 * 4u, PF * 32 * 4u);
                bulk_commit();
            }
        };
        using P0 = std::integral_constant<int, 0>;
        using P1 = std::integral_constant<int, 1>;
        auto run = [&](auto phase_c, int gi) {
            const int t0 = t_last - gi * PF;
            if constexpr (!BANDED) {
                const bool interior = full_rows && t0 - (PF - 1) >= 32 && t0 <= M - 1;
                if (interior) group(phase_c, std::false_type{}, t0);
                else group(phase_c, std::true_type{}, t0);
            } else {
                group(phase_c, std::true_type{}, t0);
            }
        };
        for (int gi = gi_begin; gi < gi_end; gi += NPH) {
            run(P0{}, gi);
            if (gi + 1 < gi_end) run(P1{}, gi + 1);
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
        // Rows outside the groups that ran (padding, or out of the band): zero.
        for (int t = 0; t <= t_last - gi_end * PF; ++t) El[static_cast<size_t>(t) * 32] = 0.f;
        for (int t = t_top + 1; t < P.n_diag; ++t) El[static_cast<size_t>(t) * 32] = 0.f;
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
    }
    cluster_sync_all();
}

// ------------------------------------------------------------------ launchers
size_t fwdx_smem(const WavePlan& P) { return fx_smem_bytes(P.wpc); }
size_t bwdw_smem(const WavePlan& P) { return bw_smem_bytes(P.wpc); }

const void* fwdx_fn(bool banded, bool weights) {
    if (weights) return banded ? (const void*)fwdx_kernel<true, true> : (const void*)fwdx_kernel<false, true>;
    return banded ? (const void*)fwdx_kernel<true, false> : (const void*)fwdx_kernel<false, false>;
}
const void* bwdw_fn(bool banded) {
    return banded ? (const void*)bwdw_kernel<true> : (const void*)bwdw_kernel<false>;
}

cudaError_t launch_forward_x(const FwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (P.K != 1) return cudaErrorInvalidValue;
    const bool banded = args.ibw < P.N + P.M;
    void* kargs[] = {const_cast<FwdArgs*>(&args)};
    return launch_cluster(fwdx_fn(banded, args.weights != 0), dim3(P.B * P.csize), dim3(P.wpc * 32), fwdx_smem(P),
                          P.csize, stream, kargs);
}

cudaError_t launch_backward_w(const BwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (P.K != 1 || !args.weights) return cudaErrorInvalidValue;
    const bool banded = args.ibw < P.N + P.M;
    void* kargs[] = {const_cast<BwdArgs*>(&args)};
    return launch_cluster(bwdw_fn(banded), dim3(P.B * P.csize), dim3(P.wpc * 32), bwdw_smem(P), P.csize, stream,
                          kargs);
}

}  // namespace sdtw
