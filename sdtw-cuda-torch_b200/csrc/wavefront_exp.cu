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
// 16 steps (so mantissas stay below 2^46).  The scaled terms are exact, so the weights of the reverse pass (a
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
// bands).  Steps run in groups of 16: per group the consumer checks the 16
// ring slots it needs with one warp-wide load and a vote, the producer checks
// flow control once and publishes the stripe's bottom row for the group's 16
// columns with one warp-wide store, the inputs of the group after next are
// copied into shared memory (cp.async), and every step's table row leaves as
// one coalesced 128- or 256-byte store.  Groups whose cells all lie inside the
// table run without masks.
#include <type_traits>

#include "sdtw_device.cuh"
#include "sdtw_kernels.h"
#include "sdtw_plan.h"
#include "wavefront_ring.cuh"

namespace sdtw {

namespace {
// Steps per group: the unit of hand-over between the warps of a pair, of the
// ring publish and of the prefetch.  Measured on B200, 16 against 8: C2
// forward 0.104 -> 0.089 ms, reverse pass 0.101 -> 0.082 ms, C3 4.43 -> 3.69
// ms per step (half the per-group synchronisation per step).  The forward's
// 64-register variant keeps 8 (fx_pf).
constexpr int kPF = 16;
constexpr int kEneg = -(1 << 30);        // exponent of P = 0 (outside the table or the band)
constexpr int kShiftMin = -96;           // terms below 2^-96 of the largest are dropped
constexpr int kErange = 1 << 29;         // valid exponents lie in (-2^29, 2^29)
constexpr float kPmax = 4194304.f;       // |D| * log2(e) / gamma per cell must stay below 2^22
constexpr float kMagic = 12582912.f;     // 1.5 * 2^23: adding it rounds to an integer in the low bits
constexpr int kFusedMaxDim = 16;         // the forward computes its costs for up to this many features
}  // namespace

// m * 2^s for s <= 0 by an add to the exponent field.  m is a normal float
// >= 1 below 2^48 and s >= kShiftMin, so the result is a normal float.
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
// Warp roles.  Warps [0, wpc) of a CTA carry the dependent chains, one stripe
// each; warp wpc + h is the helper of chain warp h (warps are placed on SM
// sub-partitions by index mod 4, so with wpc a multiple of 4 a pair shares a
// sub-partition and the helper issues in the chain warp's idle cycles).  Per
// group of PF steps the helper
//   * obtains every cell's cost: from a cost table (rows copied two groups
//     ahead into shared memory by cp.async), or, in the fused x/y mode
//     (DP > 0), computes it as sum_k (x_k - y_k)^2 (the direct form of
//     kernels.py:27-31) from its row of x, held in registers, and a window of
//     y rows in shared memory that cp.async copies fill two groups ahead -- no
//     (B, N, M) cost tensor exists in that mode,
//   * turns every cost into K = km * 2^ke (one ex2 per cell),
//   * reads the ring slots of the row above (the tag vote, and any wait for
//     the stripe above, happen here) and reports their consumption,
// and hands both over in one of kNB buffers guarded by mbarriers (full:
// helper to chain, empty: chain to helper).  The chain warp runs the steps,
// stores each cell's shares (or score) with one coalesced row store per step,
// and publishes its stripe's bottom row.
//
// Shared memory: rings [wpc][kRing][2] u64 and counters [wpc] u32 (as in
// wavefront.cu), then per pair: the helper's input (cost rows [3][PF][32]
// float, or the y window of kYRows rows of y_pitch(DP) floats), the handed-over K [kNB][PF][32] (km, ke), the ring
// input [kNB][PF] (m, e), the chain's bottom-row output [PF] (m, e), and the
// mbarriers [2][kNB].
constexpr int kNB = 3;
constexpr int kYRows = 128;            // y window rows per pair (ring of segments of PF rows)
// Steps per group of the forward: kPF for the 128-register variants; 8 for the
// 64-register variant, which serves launches with more problems than fit at
// once (short problems): its smaller buffers keep more CTAs resident and its
// stripes enter the pipeline 8 steps sooner (C5 forward 0.324 ms at 16, 0.267
// ms at 8).
__host__ __device__ constexpr int fx_pf(int dp, bool wide) { return (wide || dp >= 8) ? kPF : 8; }
// Segments before a group's own that its cells read (the 32 lanes reach 31
// rows back), and the window's segments.
__host__ __device__ constexpr int seg_back(int pf) { return (31 + pf - 1) / pf; }
static_assert(seg_back(8) + 3 <= kYRows / 8 && seg_back(kPF) + 3 <= kYRows / kPF,
              "the y window holds the segments read and the two in flight");
// Row pitch of the y window: for DP a multiple of 4, the number of 16-byte
// units per row is odd, so the 8 lanes of one 128-bit load phase, which read 8
// consecutive rows, hit distinct banks; DP = 4 also serves D < 4 with dense
// rows of D floats (odd D or 2: conflict-free for 32- and 64-bit loads).
__host__ __device__ constexpr int y_pitch(int dp) { return (dp / 4) % 2 ? dp : dp + 4; }
__host__ __device__ constexpr size_t fx_in_bytes(int dp, int pf) {
    return dp == 0 ? static_cast<size_t>(3) * pf * 32 * 4 : static_cast<size_t>(kYRows) * y_pitch(dp) * 4;
}
__host__ __device__ constexpr size_t fx_in_off(int wpc) { return fwd_stage_offset(wpc); }
__host__ __device__ constexpr size_t fx_k_off(int wpc, int dp, int pf) {
    return fx_in_off(wpc) + static_cast<size_t>(wpc) * fx_in_bytes(dp, pf);
}
__host__ __device__ constexpr size_t fx_rin_off(int wpc, int dp, int pf) {
    return fx_k_off(wpc, dp, pf) + static_cast<size_t>(wpc) * kNB * pf * 32 * 8;
}
__host__ __device__ constexpr size_t fx_pub_off(int wpc, int dp, int pf) {
    return fx_rin_off(wpc, dp, pf) + static_cast<size_t>(wpc) * kNB * pf * 8;
}
__host__ __device__ constexpr size_t fx_mbar_off(int wpc, int dp, int pf) {
    return fx_pub_off(wpc, dp, pf) + static_cast<size_t>(wpc) * pf * 8;
}
__host__ __device__ constexpr size_t fx_smem_bytes(int wpc, int dp, int pf) {
    return fx_mbar_off(wpc, dp, pf) + static_cast<size_t>(wpc) * 2 * kNB * 8;
}

__device__ __forceinline__ uint64_t pack_tagged_bits(uint32_t v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | static_cast<uint64_t>(v);
}

// Bounded wait for an mbarrier phase (kind 4 in the diagnostics).
__device__ __noinline__ bool mbar_wait_bounded(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(mbar, parity)) return true;
        const int r = backoff(it, t0, w);
        if (r) {
            record_giveup(w, r, 4, parity, 0);
            return false;
        }
    }
}
__device__ __forceinline__ bool mbar_wait_fx(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
    return mbar_try_wait(mbar, parity) || mbar_wait_bounded(mbar, parity, w);
}

// 512 threads (8 pairs) per CTA; two CTAs per SM except in the fused mode with
// 8 or 16 features, whose row of x takes registers.
// WIDE: up to 128 registers a thread (one CTA of 512 threads per SM) instead
// of 64 (two), for launches whose clusters all fit at once at that occupancy:
// the compiler interleaves more of the steps' independent work (C2 forward
// 0.118 -> 0.104 ms); launches with more problems than fit keep the
// occupancy.  The fused forward with 8 or more features always takes 128.
template <bool BANDED, bool W, int DP, bool WIDE, bool CM = false, bool SEG = false>
__global__ void __launch_bounds__(512, (DP >= 8 || WIDE) ? 1 : 2) fwdx_kernel(const FwdArgs a) {
    static_assert(!CM || (W && DP == 0), "clamp marks: shares of a cost table only");
    static_assert(!SEG || DP > 0, "sequence maps: fused costs only");
    constexpr int PF = fx_pf(DP, WIDE);
    constexpr int YSEG = kYRows / PF;      // window segments
    constexpr int SEGBACK = seg_back(PF);
    constexpr int YP = DP > 0 ? y_pitch(DP) : 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int wid = threadIdx.x >> 5;
    const bool helper = wid >= wpc;
    const int warp = helper ? wid - wpc : wid;  // the chain warp of this pair
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    const int N = P.N, M = P.M;
    pdl_trigger();

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);                    // [wpc][kRing][2]
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * 2 * kRing);  // [wpc]
    unsigned char* in_raw = smem_raw + fx_in_off(wpc) + static_cast<size_t>(warp) * fx_in_bytes(DP, PF);
    const float* cost = reinterpret_cast<const float*>(in_raw);  // table mode
    const uint32_t cost_s = smem_addr(cost);
    float* ywin = reinterpret_cast<float*>(in_raw);  // fused mode: [kYRows][YP]
    uint2* kbuf = reinterpret_cast<uint2*>(smem_raw + fx_k_off(wpc, DP, PF)) + warp * kNB * PF * 32;
    uint2* rin = reinterpret_cast<uint2*>(smem_raw + fx_rin_off(wpc, DP, PF)) + warp * kNB * PF;
    uint2* pub_s = reinterpret_cast<uint2*>(smem_raw + fx_pub_off(wpc, DP, PF)) + warp * PF;
    const uint32_t mb_full = smem_addr(reinterpret_cast<uint64_t*>(smem_raw + fx_mbar_off(wpc, DP, PF)) + warp * 2 * kNB);
    const uint32_t mb_empty = mb_full + kNB * 8u;
    for (int i = threadIdx.x; i < wpc * 2 * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    if (threadIdx.x < wpc * 2 * kNB)
        mbar_init(smem_addr(reinterpret_cast<uint64_t*>(smem_raw + fx_mbar_off(wpc, DP, PF)) + threadIdx.x), 32);
    if constexpr (DP > 0) {
        // y windows start as zeros (the rows left of column 0 are read only by
        // cells outside the table, whose values must stay finite).
        for (int i = threadIdx.x; i < wpc * kYRows * YP; i += blockDim.x) {
            const int w = i / (kYRows * YP);
            reinterpret_cast<float*>(smem_raw + fx_in_off(wpc) + static_cast<size_t>(w) * fx_in_bytes(DP, PF))
                [i - w * kYRows * YP] = 0.f;
        }
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    cluster_sync_all();
    // Set-up above touched shared memory only.  (The forward is launched
    // plainly; the wait is a no-op then.  Its trigger above lets a reverse pass
    // launched with programmatic serialization be scheduled early.)
    pdl_wait();

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
    bool bad = false;        // chain: a valid exponent left its range
    float pmax = 0.f;        // helper: largest |D| * log2(e) / gamma of a live cell (NaN if one was NaN)
    uint32_t cons_seen = 0;  // chain: consumer progress last observed
    uint32_t seqg = 0;       // groups run so far (both roles count alike): buffer seqg % kNB

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
        const uint64_t wrap_g = reinterpret_cast<uint64_t>(a.wrap + static_cast<size_t>(b) * 2 * M);
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
        const int rows_left = N - R0;
        const bool full_rows = rows_left >= 32;
        auto interior_group = [&](int t0) { return !BANDED && full_rows && t0 >= 32 && t0 + PF <= M; };

        if (helper) {
            // ================================================ helper
            const float* Dl = a.Dw + sb;
            const uint32_t in_tag_wrap = wrap_tag(a.seq, band - 1);
            // Last column of the row above that is in the band (published by
            // the stripe above); the columns past it read as P = 0.
            const int c_pub_max = BANDED ? min(M - 1, R0 - 1 + ibw) : M - 1;
            // Everything before this band counts as consumed.
            st_release_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed, band_base);
            auto cost_copy = [&](int gg) {
                if (gg < g_end) {
                    const float* src = Dl + static_cast<size_t>(gg) * PF * 32;
                    const uint32_t dst = cost_s + static_cast<uint32_t>((gg - g_begin) % 3) * PF * 32 * 4u;
#pragma unroll
                    for (int i = 0; i < PF * 32 / 128; ++i)
                        cp_async16(dst + (lane + 32 * i) * 16u, src + (lane + 32 * i) * 4);
                }
                cp_async_commit();
            };
            // ---- fused mode: this lane's row of x in registers (zeros past
            // the last row and past the last feature), and the y window.
            const int D = a.dim;
            const bool dense = DP > 0 && D < 4;  // rows of D < 4 floats, copied per segment
            unsigned long long xq[DP > 0 ? DP / 2 : 1];
            if constexpr (DP > 0) {
                float xv[DP];
                const float* xr = (SEG ? a.x.at(b, a.x_bstride) : a.x.p[0] + static_cast<size_t>(b) * a.x_bstride) +
                                  static_cast<size_t>(R0 + lane) * D;
#pragma unroll
                for (int f = 0; f < DP; ++f) xv[f] = (lane < rows_left && f < D) ? __ldg(xr + f) : 0.f;
#pragma unroll
                for (int f = 0; f < DP / 2; ++f)
                    xq[f] = (static_cast<unsigned long long>(__float_as_uint(xv[2 * f + 1])) << 32) |
                            __float_as_uint(xv[2 * f]);
            }
            // (Resolved here in the single-batch variant in the same form as
            // before the sequence maps existed: a select-based form measured
            // 2 % slower on the C3 forward, the address being re-derived per copy.)
            const float* yb = SEG ? a.y.at(b, static_cast<size_t>(M) * D) : a.y.p[0] + static_cast<size_t>(b) * M * D;
            // Rows seg*PF .. seg*PF+PF-1 of y (those below M) into window slot
            // seg mod YSEG by cp.async, one commit group per segment: 16-byte
            // copies into the padded rows, or 4-byte copies of dense rows (D < 4).
            // (Bulk copies of single rows measured several microseconds from
            // issue to landing on B200, more than the two groups of prefetch.)
            auto y_issue = [&](int seg) {
                if constexpr (DP > 0) {
                    const int sl = seg & (YSEG - 1);
                    const int r0 = seg * PF;
                    const int nr = (seg < g_end) ? max(0, min(PF, M - r0)) : 0;
                    if (dense) {
                        for (int e = lane; e < nr * D; e += 32)
                            cp_async4(smem_addr(ywin + sl * PF * D + e), yb + static_cast<size_t>(r0) * D + e);
                    } else {
                        const int cpr = D / 4;  // 16-byte chunks per row
                        for (int e = lane; e < nr * cpr; e += 32) {
                            const int r = e / cpr, k = e - r * cpr;
                            cp_async16(smem_addr(ywin + (sl * PF + r) * YP + 4 * k),
                                       yb + static_cast<size_t>(r0 + r) * D + 4 * k);
                        }
                    }
                    cp_async_commit();
                }
            };
            // Segment seg has landed (issued two groups before it is needed;
            // only the newest commit group may still be in flight).
            auto y_wait = [&](int seg) {
                (void)seg;
                if constexpr (DP > 0) {
                    cp_async_wait<1>();
                    __syncwarp();
                }
            };
            if constexpr (DP == 0) {
                cost_copy(g_begin);
                cost_copy(g_begin + 1);
            } else {
                // The window rows of the first group (segments g_begin -
                // SEGBACK .. g_begin) and the next one in flight.
                const int s_lo = max(0, g_begin - SEGBACK);
                for (int sg = s_lo; sg < g_begin + 2; ++sg) y_issue(sg);
            }
            if (t_begin > 0)
                st_relaxed_cluster_u32_if(has_in && !in_wrap && lane == 0, prev_consumed,
                                          band_base + static_cast<uint32_t>(min(t_begin, M)));
            // Band-wrap input (global memory, an L2 round trip per load): the
            // slots of the next group are loaded one group ahead.
            uint64_t wpf_h = 0, wpf_l = 0;
            if (has_in && in_wrap && t_begin < M && t_begin + (lane & (PF - 1)) <= c_pub_max)
                ld_pair(wrap_g + static_cast<uint32_t>(t_begin + (lane & (PF - 1))) * 16u, wpf_h, wpf_l);

            for (int gi = g_begin; gi < g_end; ++gi, ++seqg) {
                const int t0 = gi * PF;
                const uint32_t slot = seqg % kNB, use = seqg / kNB;
                // The chain warp has finished with this buffer's previous use.
                if (use > 0 && ok) ok = mbar_wait_fx(mb_empty + slot * 8u, (use - 1) & 1u, wc);
                // ---- the group's costs: from its cost rows (two commits back),
                // or from x and the y window.  All loads come before the first
                // store: the compiler cannot tell the input from the K buffer
                // apart, and a load placed after a store would serialise the cells.
                uint2* kb = kbuf + slot * PF * 32 + lane;
                const bool masked = !interior_group(t0);
                float cv[PF];
                if constexpr (DP == 0) {
                    cp_async_wait<1>();
                    __syncwarp();
                    const float* cb = cost + ((gi - g_begin) % 3) * PF * 32 + lane;
#pragma unroll
                    for (int u = 0; u < PF; ++u) cv[u] = cb[u * 32];
                } else {
                    y_wait(gi);
                    if (dense) {
#pragma unroll
                        for (int u = 0; u < PF; ++u) {
                            const float* yr = ywin + ((t0 + u - lane) & (kYRows - 1)) * D;
                            float c = 0.f;
#pragma unroll
                            for (int f = 0; f < 3; ++f) {
                                const float xf = __uint_as_float(static_cast<uint32_t>(xq[f >> 1] >> (32 * (f & 1))));
                                const float d = xf - yr[f < D ? f : 0];
                                c = (f < D) ? fmaf(d, d, c) : c;
                            }
                            cv[u] = c;
                        }
                    } else {
                        // Feature chunks outer, the group's 8 cells inner: 8
                        // independent accumulator chains interleave.
                        const ulonglong2* yw = reinterpret_cast<const ulonglong2*>(ywin);
                        int ro[PF];  // window row offsets (in 16-byte units) of the 8 cells
#pragma unroll
                        for (int u = 0; u < PF; ++u) ro[u] = ((t0 + u - lane) & (kYRows - 1)) * (YP / 4);
                        unsigned long long acc[PF];  // (even-feature, odd-feature) partial sums
#pragma unroll
                        for (int u = 0; u < PF; ++u) acc[u] = 0ull;
#pragma unroll
                        for (int k = 0; k < DP / 4; ++k) {
#pragma unroll
                            for (int u = 0; u < PF; ++u) {
                                const ulonglong2 yv = yw[ro[u] + k];
                                const unsigned long long d01 = sub_f32x2(xq[2 * k], yv.x);
                                const unsigned long long d23 = sub_f32x2(xq[2 * k + 1], yv.y);
                                acc[u] = fma_f32x2(d01, d01, acc[u]);
                                acc[u] = fma_f32x2(d23, d23, acc[u]);
                            }
                        }
#pragma unroll
                        for (int u = 0; u < PF; ++u) cv[u] = lo_f32x2(acc[u]) + hi_f32x2(acc[u]);
                    }
                    y_issue(gi + 2);  // into the slot of segment gi + 2 - YSEG, no longer read
                }
#pragma unroll
                for (int u = 0; u < PF; ++u) {
                    const float c = cv[u];
                    const float p = c * kk;
                    const float r = __fadd_rd(-p, kMagic);
                    const float fl = r - kMagic;
                    const int ke = __float_as_int(r) - __float_as_int(kMagic);
                    float km = ex2f(fmaf(-c, kk, -fl));
                    int kx = ke;
                    float pa = fabsf(p);
                    if constexpr (!W) {
                        // Caller-supplied costs may be +inf (a forbidden cell,
                        // P = 0): handed over as exponent kEneg.
                        const bool cinf = c == pos_inf();
                        pa = cinf ? 0.f : pa;
                        km = cinf ? 1.f : km;
                        kx = cinf ? kEneg : kx;
                    }
                    // Only cells inside the table (and the band) count for the
                    // range check; computed for every cell (a branch here would
                    // keep the compiler from interleaving the group's cells).
                    const int col = t0 + u - lane;
                    bool live = static_cast<unsigned>(col) < static_cast<unsigned>(M) && lane < rows_left;
                    if constexpr (BANDED)
                        live = live && static_cast<unsigned>(R0 + lane - col + ibw) <= static_cast<unsigned>(2 * ibw);
                    pmax = max_nan(pmax, (live || !masked) ? pa : 0.f);
                    // The clamp mark travels in K's mantissa sign bit (K > 0).
                    const uint32_t mark = (CM && !(c > 0.f)) ? 0x80000000u : 0u;
                    kb[u * 32] = make_uint2(__float_as_uint(km) | mark, static_cast<uint32_t>(kx));
                }
                if constexpr (DP == 0) cost_copy(gi + 2);  // into the buffer just read
                // ---- ring input: the row above for columns t0 .. t0+PF-1, slot u
                // read by lane u (mod PF).
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
                if (lane < PF) rin[slot * PF + lane] = make_uint2(vm, ve);
                mbar_arrive(mb_full + slot * 8u);  // release: the K and ring rows above
                if ((gi & 15) == 15 && __any_sync(SDTW_FULL_MASK, !ok)) {
                    quit = true;
                    ++seqg;
                    break;
                }
            }
            cp_async_wait<0>();
            __syncwarp();
            if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
            continue;
        }

        // ==================================================== chain warp
        float2* Tl = a.score + sb + lane;  // this lane's position of anti-diagonal row 0
        const uint64_t out_g = out_wrap ? wrap_g : next_ring_g;
        const uint32_t out_tag_wrap = wrap_tag(a.seq, band);
        // Cell state: own previous cell (left neighbour of the next step) and
        // the upper neighbour of the previous step (diagonal of the next).
        float m_l = 1.f;
        int e_l = kEneg;
        float m_d = 1.f;
        int e_d = (R0 == 0 && lane == 0) ? 0 : kEneg;  // R[0,0] = 0 above-left of cell (0, 0)
        const int l_last = N - 1 - R0;
        const int t_last = (s == P.n_stripes - 1 && lane == l_last) ? l_last + M - 1 : -1;
        float last_m = 1.f;
        int last_e = kEneg;

        auto group = [&](auto masked_c, int t0, uint32_t slot) {
            constexpr bool MASKED = decltype(masked_c)::value;
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
            // The group's K and ring input in registers before the stores of the
            // steps that use them (a shared load placed after a store would
            // wait for it).
            const uint2* kb = kbuf + slot * PF * 32 + lane;
            const uint2* ri_s = rin + slot * PF;
            // Half a group at a time keeps the registers of two CTAs per SM.
            constexpr int PH = PF / 2;
            uint2 kq[PH], rq[PH];
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                if (u % PH == 0) {
#pragma unroll
                    for (int v = 0; v < PH; ++v) {
                        kq[v] = kb[(u + v) * 32];
                        rq[v] = ri_s[u + v];
                    }
                }
                const int t = t0 + u;
                const uint32_t kbits = kq[u % PH].x;
                const float km = __uint_as_float(CM ? kbits & 0x7fffffffu : kbits);
                const int ke = static_cast<int>(kq[u % PH].y);
                const uint2 ri = rq[u % PH];
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
                if constexpr (!W) {
                    // A cell of cost +inf (marked by the helper): P = 0.
                    const bool cinf = ke == kEneg;
                    mn = cinf ? 1.f : mn;
                    en = cinf ? kEneg : en;
                }
                float2 rec;
                if constexpr (W) {
                    // The shares of the diagonal and upper predecessors: all the
                    // reverse pass needs of this cell.
                    // (With the clamp mark in the diagonal share's sign bit.)
                    const float inv = rcpf(sum);
                    rec = make_float2(CM ? __uint_as_float(__float_as_uint(vd * inv) | (kbits & 0x80000000u)) : vd * inv,
                                      vu * inv);
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
                    last_m = (t == t_last) ? mn : last_m;
                    last_e = (t == t_last) ? en : last_e;
                }
                Tl[static_cast<size_t>(t) * 32] = rec;  // one coalesced row store per step
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
            __syncwarp();
            // ---- the stripe's bottom row for columns t0-31 .. t0-31+PF-1: lane u
            // stores column t0 - 31 + u (both halves tagged).
            if (has_out) {  // warp-uniform
                const int colb = t0 - 31 + lane;
                const bool pub = lane < PF && static_cast<unsigned>(colb) < static_cast<unsigned>(M);
                const uint2 pv = pub_s[lane & (PF - 1)];
                const uint32_t tgo = out_wrap ? out_tag_wrap : band_base + static_cast<uint32_t>(colb);
                const uint32_t sl = out_wrap ? static_cast<uint32_t>(colb) : (tgo % kRing);
                st_pair_if(pub, out_g + sl * 16u, pack_tagged_bits(pv.x, tgo), pack_tagged_bits(pv.y, tgo));
            }
        };
        for (int gi = g_begin; gi < g_end; ++gi, ++seqg) {
            const int t0 = gi * PF;
            const uint32_t slot = seqg % kNB, use = seqg / kNB;
            // The helper has filled this buffer (K and the row above).
            if (ok) ok = mbar_wait_fx(mb_full + slot * 8u, use & 1u, wc);
            if constexpr (!BANDED) {
                if (interior_group(t0)) group(std::false_type{}, t0, slot);
                else group(std::true_type{}, t0, slot);
            } else {
                group(std::true_type{}, t0, slot);
            }
            mbar_arrive(mb_empty + slot * 8u);
            if ((gi & 15) == 15 && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                ++seqg;
                break;
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
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
// forward's staging offset) per warp the weights of three groups [3][PF][32]
// float2 and the messages of one group [PF] float.  E leaves by one coalesced
// 128-byte row store per step (measured on B200 faster than staging a group's
// rows in shared memory for one bulk copy: C2 reverse pass 0.131 -> 0.117 ms).
__host__ __device__ constexpr size_t bw_w_off(int wpc) {
    return fwd_stage_offset(wpc);
}
__host__ __device__ constexpr size_t bw_stash_off(int wpc) {
    return bw_w_off(wpc) + static_cast<size_t>(wpc) * 3 * kPF * 32 * 8;
}
// With grad_x (gd > 0) per warp also a window of y rows [kYRows][y_pitch(gd)]
// (ring of segments of PF rows, cp.async two groups ahead, like the fused
// forward's).
__host__ __device__ constexpr size_t bw_ywin_off(int wpc) {
    return bw_stash_off(wpc) + static_cast<size_t>(wpc) * kPF * 4;
}
__host__ __device__ constexpr size_t bw_smem_bytes(int wpc, int gd = 0) {
    return bw_ywin_off(wpc) + (gd == 0 ? 0 : static_cast<size_t>(wpc) * kYRows * y_pitch(gd) * 4);
}

// Reverse wavefront over the forward's shares.  At reverse step t the lane of
// row q handles cell (q, t - q):
//   E = (E of the right neighbour) * its left share       (accl, same lane)
//     + message from the row below: E(q+1, j) * upper share of (q+1, j)
//                                  + E(q+1, j+1) * diagonal share of (q+1, j+1)
// E(N-1, M-1) = grad_out[b] (autograd.py:46-47 multiplies it in).
//
// GD > 0 (grad_x only): the squared-Euclidean chain rule (autograd_xy.py:41-49)
// is applied as E is produced, and E is not stored.  Lane q (row i = R0 + q)
// keeps sum_j E_ij and sum_j E_ij y_j (y_j from the warp's y window) and
// writes grad_x[i] = 2 (x_i sum_j E_ij - sum_j E_ij y_j) at the end of its
// stripe.  (grad_y the same way -- column partials passed down the lanes by
// shuffles, one per feature per step -- measured slower on B200 than the E
// table and grad_small: C3 reverse pass 1.42 -> 2.96 ms against a 0.79 ms
// gradient kernel; the extra shuffles delay the chain's own.)
template <bool BANDED, int GD, bool CM = false>
__global__ void __launch_bounds__(GD > 0 ? 256 : 512, GD > 0 ? 2 : 1) bwdw_kernel(const BwdArgs a) {
    static_assert(!CM || GD == 0, "clamp marks: unfused costs only");
    constexpr int PF = kPF;
    constexpr int YSEG = kYRows / PF;      // window segments
    constexpr int SEGBACK = seg_back(PF);
    constexpr int YP = y_pitch(GD > 0 ? GD : 4);
    static_assert(GD == 0 || !BANDED, "the gradient mode runs without a band");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const WavePlan P = a.P;
    const int wpc = P.wpc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int crank = static_cast<int>(cluster_ctarank());
    const int b = blockIdx.x / P.csize;
    const int g = crank * wpc + warp;
    const int N = P.N, M = P.M;
    pdl_trigger();

    uint64_t* ring = reinterpret_cast<uint64_t*>(smem_raw);
    uint32_t* consumed = reinterpret_cast<uint32_t*>(ring + wpc * kRing);
    const float2* wbuf = reinterpret_cast<const float2*>(smem_raw + bw_w_off(wpc)) + warp * 3 * PF * 32;
    const uint32_t wbuf_s = smem_addr(wbuf);
    float* pub_s = reinterpret_cast<float*>(smem_raw + bw_stash_off(wpc)) + warp * PF;
    float* ywin = reinterpret_cast<float*>(smem_raw + bw_ywin_off(wpc)) + warp * kYRows * YP;
    for (int i = threadIdx.x; i < wpc * kRing; i += blockDim.x) ring[i] = ~0ull;
    if (threadIdx.x < wpc) consumed[threadIdx.x] = 0u;
    if constexpr (GD > 0) {
        // Window rows that are never copied (outside y) stay finite: they meet
        // only cells with E = 0.
        float* yw_all = reinterpret_cast<float*>(smem_raw + bw_ywin_off(wpc));
        for (int i = threadIdx.x; i < wpc * kYRows * YP; i += blockDim.x) yw_all[i] = 0.f;
    }
    cluster_sync_all();
    pdl_wait();  // the shares and y of the previous kernels are read from here on

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
            gi_begin = (t_last - t_hi) / PF;
            gi_end = max(gi_begin, min(n_groups, (t_last - t_lo) / PF + 1));
        }
        const int t_top = t_last - gi_begin * PF;  // first (highest) step that runs
        // Columns of the row below that are in the band (sent by the stripe below).
        const int c_min = BANDED ? max(0, R0 + 32 - ibw) : 0;
        if (t_top < t_last)
            st_relaxed_cluster_u32_if(has_below && !below_wrap && lane == 31, below_consumed,
                                      band_base + static_cast<uint32_t>(max(0, M - 1 - max(t_top - 31, -1))));
        const int rows_left = N - R0;
        const bool full_rows = rows_left >= 32;
        // ---- gradient mode: the row accumulators.
        const int D = a.dim;
        float racc[GD > 0 ? GD : 1], rsum = 0.f;  // row: sum_j E y_j, sum_j E
#pragma unroll
        for (int f = 0; f < (GD > 0 ? GD : 1); ++f) racc[f] = 0.f;
        const float* yb = GD > 0 ? a.y + static_cast<size_t>(b) * M * D : nullptr;
        // y rows 8 seg .. 8 seg + 7 (those inside y) into window slot seg mod
        // YSEG: 16-byte copies, or 4-byte copies into padded rows for D < 4.
        auto y_issue = [&](int seg) {
            if constexpr (GD > 0) {
                const int r0 = seg * PF;
                const int nr = (seg >= 0) ? max(0, min(PF, M - r0)) : 0;
                float* dst = ywin + (seg & (YSEG - 1)) * PF * YP;
                if (D < 4) {
                    for (int e = lane; e < nr * D; e += 32) {
                        const int r = e / D, f = e - r * D;
                        cp_async4(smem_addr(dst + r * YP + f), yb + static_cast<size_t>(r0) * D + e);
                    }
                } else {
                    const int cpr = D / 4;
                    for (int e = lane; e < nr * cpr; e += 32) {
                        const int r = e / cpr, k = e - r * cpr;
                        cp_async16(smem_addr(dst + r * YP + 4 * k), yb + static_cast<size_t>(r0 + r) * D + 4 * k);
                    }
                }
            }
        };
        // Group gi's shares: rows t0 - PF + 1 .. t0 (t0 = t_last - gi * PF),
        // or an empty commit past the last group.  In the gradient mode the
        // same commit carries the lowest y segment group gi reads (its cells
        // read segments k - SEGBACK .. k, k = n_groups - 1 - gi; the first
        // commit carries all of them).
        auto wcopy = [&](int gi) {
            if (gi < gi_end) {
                const float2* src = Ts + static_cast<size_t>(t_last - gi * PF - PF + 1) * 32;
                const uint32_t dst = wbuf_s + static_cast<uint32_t>((gi - gi_begin) % 3) * PF * 32 * 8u;
#pragma unroll
                for (int i = 0; i < PF * 32 / 64; ++i) cp_async16(dst + (lane + 32 * i) * 16u, src + (lane + 32 * i) * 2);
                if constexpr (GD > 0) {
                    const int k = n_groups - 1 - gi;
                    if (gi == gi_begin)
                        for (int sg = k; sg >= k - SEGBACK; --sg) y_issue(sg);
                    else
                        y_issue(k - SEGBACK);
                }
            }
            cp_async_commit();
        };
        wcopy(gi_begin);
        wcopy(gi_begin + 1);

        float accl = 0.f, msg = 0.f, dprev = 0.f;
        // Band-wrap input (global memory): the slots of the next group are
        // loaded one group ahead.
        uint64_t wpf = 0;
        {
            const int col = t_top - 31 - (lane & (PF - 1));
            if (has_below && below_wrap && col >= c_min && col < M) wpf = ld_one(in_g + static_cast<uint32_t>(col) * 16u);
        }

        auto group = [&](auto masked_c, int t0) {
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
            cp_async_wait<1>();  // this group's shares, committed two groups back
            __syncwarp();
            const int gi = (t_last - t0) / PF;
            const float2* wb = wbuf + ((gi - gi_begin) % 3) * PF * 32 + (PF - 1) * 32 + lane;
            wcopy(gi + 2);  // into the buffer the previous group read
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
                const float dn = e * (CM ? fabsf(w.x) : w.x);  // to the diagonal predecessor (two steps on)
                msg = fmaf(e, w.y, dprev);           // to the row above: upper share + previous diagonal
                accl = fmaf(-e, w.y, e - dn);        // left share: e * (1 - wd - wu)
                dprev = dn;
                if (lane == 0) pub_s[u] = msg;
                // The stored (and chain-ruled) E is zero where the forward marked
                // a clamped cost; the recurrence itself carries e unmasked.
                const float eo = (CM && (__float_as_uint(w.x) >> 31)) ? 0.f : e;
                if constexpr (GD == 0) {
                    El[static_cast<size_t>(t) * 32] = eo;  // one coalesced row store per step
                } else {
                    // Row: E y_j with y_j = window row t - lane.
                    const float4* yr = reinterpret_cast<const float4*>(ywin + ((t - lane) & (kYRows - 1)) * YP);
                    rsum += eo;
#pragma unroll
                    for (int q = 0; q < GD / 4; ++q) {
                        const float4 yv = yr[q];
                        racc[4 * q + 0] = fmaf(eo, yv.x, racc[4 * q + 0]);
                        racc[4 * q + 1] = fmaf(eo, yv.y, racc[4 * q + 1]);
                        racc[4 * q + 2] = fmaf(eo, yv.z, racc[4 * q + 2]);
                        racc[4 * q + 3] = fmaf(eo, yv.w, racc[4 * q + 3]);
                    }
                }
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

        };
        // One step body per loop iteration (two, unrolled, measured slower on
        // B200: C2 reverse pass 0.115 -> 0.103 ms, C3 1.42 -> 1.19 ms with one).
        auto run = [&](int gi) {
            const int t0 = t_last - gi * PF;
            if constexpr (!BANDED) {
                const bool interior = full_rows && t0 - (PF - 1) >= 32 && t0 <= M - 1;
                if (interior) group(std::false_type{}, t0);
                else group(std::true_type{}, t0);
            } else {
                group(std::true_type{}, t0);
            }
        };
        for (int gi = gi_begin; gi < gi_end; ++gi) {
            run(gi);
            if ((gi & 15) == 15 && __any_sync(SDTW_FULL_MASK, !ok)) {
                quit = true;
                break;
            }
        }
        // The band's copies are complete before the next band's first group.
        cp_async_wait<0>();
        __syncwarp();
        if constexpr (GD == 0) {
            // Rows outside the groups that ran (padding, or out of the band): zero.
            for (int t = 0; t <= t_last - gi_end * PF; ++t) El[static_cast<size_t>(t) * 32] = 0.f;
            for (int t = t_top + 1; t < P.n_diag; ++t) El[static_cast<size_t>(t) * 32] = 0.f;
        } else {
            if (lane < rows_left) {
                const float* xr = a.x + static_cast<size_t>(b) * a.x_bstride + static_cast<size_t>(R0 + lane) * D;
                float* go = a.gx + (static_cast<size_t>(b) * N + R0 + lane) * D;
#pragma unroll
                for (int f = 0; f < GD; ++f)
                    if (f < D) go[f] = 2.f * (__ldg(xr + f) * rsum - racc[f]);
            }
        }
        if (__any_sync(SDTW_FULL_MASK, !ok)) quit = true;
    }
    cluster_sync_all();
}

// ------------------------------------------------------------------ launchers
size_t fwdx_smem(const WavePlan& P, int dp, bool wide) { return fx_smem_bytes(P.wpc, dp, fx_pf(dp, wide)); }
int fwdx_threads(const WavePlan& P) { return 2 * P.wpc * 32; }  // a chain warp and its helper per stripe
size_t bwdw_smem(const WavePlan& P, int gd) { return bw_smem_bytes(P.wpc, gd); }

// dp: 0 = costs from a table; 4, 8, 16, 32, 64 = fused x/y costs with the
// features padded to dp (the x/y entry points, which store the shares).
const void* fwdx_fn(bool banded, bool weights, int dp, bool wide, bool cm, bool seg) {
    if (seg && dp > 0) {  // problems in several segments (the normalized triple)
        switch (dp) {
            case 4:
                if (wide) return banded ? (const void*)fwdx_kernel<true, true, 4, true, false, true>
                                        : (const void*)fwdx_kernel<false, true, 4, true, false, true>;
                return banded ? (const void*)fwdx_kernel<true, true, 4, false, false, true>
                              : (const void*)fwdx_kernel<false, true, 4, false, false, true>;
            case 8:
                return banded ? (const void*)fwdx_kernel<true, true, 8, true, false, true>
                              : (const void*)fwdx_kernel<false, true, 8, true, false, true>;
            case 16:
                return banded ? (const void*)fwdx_kernel<true, true, 16, true, false, true>
                              : (const void*)fwdx_kernel<false, true, 16, true, false, true>;
            default: return nullptr;
        }
    }
#define SDTW_FWDX(BW, WW, DD) \
    (wide ? (const void*)fwdx_kernel<BW, WW, DD, true> : (const void*)fwdx_kernel<BW, WW, DD, false>)
#define SDTW_FWDX_CM(BW) \
    (wide ? (const void*)fwdx_kernel<BW, true, 0, true, true> : (const void*)fwdx_kernel<BW, true, 0, false, true>)
    switch (dp) {
        case 0:
            if (weights && cm) return banded ? SDTW_FWDX_CM(true) : SDTW_FWDX_CM(false);
            if (weights) return banded ? SDTW_FWDX(true, true, 0) : SDTW_FWDX(false, true, 0);
            return banded ? SDTW_FWDX(true, false, 0) : SDTW_FWDX(false, false, 0);
        case 4: return banded ? SDTW_FWDX(true, true, 4) : SDTW_FWDX(false, true, 4);
        // 8 and 16 features: 128 registers either way.
        case 8: return banded ? (const void*)fwdx_kernel<true, true, 8, true> : (const void*)fwdx_kernel<false, true, 8, true>;
        case 16:
            return banded ? (const void*)fwdx_kernel<true, true, 16, true> : (const void*)fwdx_kernel<false, true, 16, true>;
        default: return nullptr;
    }
#undef SDTW_FWDX
#undef SDTW_FWDX_CM
}
// Feature padding of the fused forward for dim features, or 0 when the fused
// costs come from a cost table in the workspace: more than kFusedMaxDim
// features, a feature count above 3 that is not a multiple of 4, or x / y not
// 16-byte aligned.  Measured on B200 at B = 32, N = M = 512 (forward, cost
// included): 12 and 16 features 0.145 ms either way, 32 features 0.173 ms
// fused against 0.155 ms with the table, 64 features 0.239 against 0.175.
// Inside the wavefront every cell reads all of its y row from shared memory;
// the separate cost kernel reuses each load across four cells.
int fused_dp(int dim, const SeqIn& x, const SeqIn& y) {
    if (dim < 4) return 4;
    if (dim > kFusedMaxDim || dim % 4 || !x.aligned16() || !y.aligned16()) return 0;
    int dp = 4;
    while (dp < dim) dp *= 2;
    return dp;
}
const void* bwdw_fn(bool banded, int gd, bool cm) {
    if (gd == 0) {
        if (cm) return banded ? (const void*)bwdw_kernel<true, 0, true> : (const void*)bwdw_kernel<false, 0, true>;
        return banded ? (const void*)bwdw_kernel<true, 0> : (const void*)bwdw_kernel<false, 0>;
    }
    if (banded) return nullptr;
    switch (gd) {
        case 4: return (const void*)bwdw_kernel<false, 4>;
        case 8: return (const void*)bwdw_kernel<false, 8>;
        case 16: return (const void*)bwdw_kernel<false, 16>;
        default: return nullptr;
    }
}
// Feature padding of the reverse pass with gradients: as the fused forward's
// (up to 16 features; more, or a count above 3 that is not a multiple of 4,
// or y not 16-byte aligned: 0, E is stored and a gradient kernel follows).
int grad_fused_gd(int dim, const float* y) { return fused_dp(dim, one_seq(y), one_seq(y)); }

cudaError_t launch_forward_x(const FwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (P.K != 1 || P.wpc > 8 || (args.dp && !args.weights)) return cudaErrorInvalidValue;
    const bool banded = args.ibw < P.N + P.M;
    const bool seg = args.x.per < P.B || args.y.per < P.B;
    const void* fn = fwdx_fn(banded, args.weights != 0, args.dp, args.wide != 0, args.clamp_mask != 0, seg);
    if (!fn) return cudaErrorInvalidValue;
    void* kargs[] = {const_cast<FwdArgs*>(&args)};
    return launch_cluster(fn, dim3(P.B * P.csize), dim3(fwdx_threads(P)), fwdx_smem(P, args.dp, args.wide != 0), P.csize, stream,
                          kargs);
}

cudaError_t launch_backward_w(const BwdArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (P.K != 1 || !args.weights) return cudaErrorInvalidValue;
    const bool banded = args.ibw < P.N + P.M;
    const void* fn = bwdw_fn(banded, args.gd, args.clamp_mask != 0);
    if (!fn || (args.gd && (!args.x || !args.y || !args.gx || args.dim > args.gd))) return cudaErrorInvalidValue;
    void* kargs[] = {const_cast<BwdArgs*>(&args)};
    return launch_cluster(fn, dim3(P.B * P.csize), dim3(P.wpc * 32), bwdw_smem(P, args.gd), P.csize, stream, kargs,
                          args.pdl != 0);
}

}  // namespace sdtw
