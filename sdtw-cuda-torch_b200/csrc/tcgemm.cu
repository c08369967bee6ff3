// tcgemm.cu -- the chain rule of the squared-Euclidean cost on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory), in 3xTF32 so that the
// result keeps float32 accuracy.
//
//   grad_x[b,q,:] = 2 (x_q * sum_j G(q,j) - sum_j G(q,j) y_j)
//   grad_y[b,j,:] = 2 (y_j * sum_q G(q,j) - sum_q G(q,j) x_q)
//
// G = E, the reverse pass's output (fused cost), or E * (D > 0), the clamp mask
// of the unfused cost; both are read straight from the wavefront layout.  This
// replaces the two bmm of softdtw_cuda/autograd_xy.py:41-49 (fused) and torch's
// autograd of softdtw_cuda/distances.py:20-28 (unfused).
//
// One CTA (8 warps) computes a 128-row output tile (rows q for grad_x, rows j
// for grad_y) for one block of features.  Per K chunk of 32 it stages the G tile
// and the x or y tile in shared memory, each split into a tf32-exact high part
// (low 13 mantissa bits cleared) and the float32 remainder; one thread issues
// hi*hi + hi*lo + lo*hi as tcgen05.mma kind::tf32 (M=128, N = features + 1,
// K = 8 per instruction) into one float32 accumulator in tensor memory.  The
// extra column of ones in the B operand makes the accumulator's last column the
// row (or column) sum of G.  Two or three stages fed by cp.async: the copies
// of the next chunks overlap the split and MMAs of the current one, and the
// MMAs signal completion through an mbarrier (tcgen05.commit).  The epilogue reads the accumulator with tcgen05.ld
// (warp w may read tensor-memory lanes 32(w%4)..32(w%4)+31, i.e. those tile
// rows; the two warp groups take alternate 16-column chunks).
#include "sdtw_device.cuh"
#include "sdtw_kernels.h"

namespace sdtw {
namespace tc {

constexpr int kThreads = 256;  // 8 warps: all load; warp w reads accumulator lanes 32*(w%4)
constexpr int kTileM = 128;  // MMA M: output rows per CTA
constexpr int kKT = 32;      // K elements per stage (4 MMA K-steps of 8)

// Shared-memory operands use the canonical K-major layout without swizzle:
// a core matrix is 8 rows x 16 bytes (8 rows x 4 tf32), and element (r, k) of
// an R x 32 operand sits at
//     (r / 8) * kSBO + (k / 4) * kLBO + (r % 8) * 16 + (k % 4) * 4   bytes,
// i.e. the 8 k-chunks of a row group are adjacent (leading byte offset 128)
// and row groups are 1040 bytes apart (stride byte offset): 1024 + 16, so
// that consecutive row groups start four banks apart and the skewed tile
// writes below (32 rows with 32 different columns) hit 32 different banks.
// One MMA K-step (8 elements = 2 chunks) advances the start address by 256.
constexpr uint32_t kLBO = 128;
constexpr uint32_t kSBO = 1040;

__device__ __forceinline__ uint32_t op_off(int r, int k) {
    return static_cast<uint32_t>((r >> 3) * kSBO + (k >> 2) * kLBO + (r & 7) * 16 + (k & 3) * 4);
}

// Shared-memory matrix descriptor (tcgen05): start address, leading and stride
// byte offsets in 16-byte units, descriptor version 1 at bits 46-47, base offset
// 0, no swizzle (layout type 0 in bits 61-63).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((kLBO >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((kSBO >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    return d;
}

// Instruction descriptor for kind::tf32: float32 accumulator (bits 4-5 = 1),
// A and B tf32 (bits 7-9, 10-12 = 2), both K-major (bits 15, 16 = 0), N >> 3 in
// bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t mbar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(mbar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_saddr, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_saddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive accumulator columns of this warp's 32 lanes (one row per
// thread).  The wait is tied to the registers so that no use moves above it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r0, r1, r2, r3, r4, r5, r6, r7, r8, r9, r10, r11, r12, r13, r14, r15;
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7), "=r"(r8), "=r"(r9),
          "=r"(r10), "=r"(r11), "=r"(r12), "=r"(r13), "=r"(r14), "=r"(r15)
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r0), "+r"(r1), "+r"(r2), "+r"(r3), "+r"(r4), "+r"(r5), "+r"(r6), "+r"(r7), "+r"(r8),
                   "+r"(r9), "+r"(r10), "+r"(r11), "+r"(r12), "+r"(r13), "+r"(r14), "+r"(r15)
                 :
                 : "memory");
    v[0] = __uint_as_float(r0);
    v[1] = __uint_as_float(r1);
    v[2] = __uint_as_float(r2);
    v[3] = __uint_as_float(r3);
    v[4] = __uint_as_float(r4);
    v[5] = __uint_as_float(r5);
    v[6] = __uint_as_float(r6);
    v[7] = __uint_as_float(r7);
    v[8] = __uint_as_float(r8);
    v[9] = __uint_as_float(r9);
    v[10] = __uint_as_float(r10);
    v[11] = __uint_as_float(r11);
    v[12] = __uint_as_float(r12);
    v[13] = __uint_as_float(r13);
    v[14] = __uint_as_float(r14);
    v[15] = __uint_as_float(r15);
}

// 4-byte asynchronous global -> shared copy; src_bytes = 0 writes zero and
// reads nothing (the address is still a valid one).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Splits the float32 at hi_base + off in place into its tf32-exact high part
// (low 13 mantissa bits cleared) and writes the float32 remainder to lo_base +
// off; with a mask value, elements whose mask is not > 0 become zero.
__device__ __forceinline__ void split_in_place(unsigned char* hi_base, unsigned char* lo_base, uint32_t off) {
    const float v = *reinterpret_cast<const float*>(hi_base + off);
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    *reinterpret_cast<float*>(hi_base + off) = h;
    *reinterpret_cast<float*>(lo_base + off) = v - h;
}
__device__ __forceinline__ void split_in_place_masked(unsigned char* hi_base, unsigned char* lo_base,
                                                      const unsigned char* mask_base, uint32_t off) {
    float v = *reinterpret_cast<const float*>(hi_base + off);
    if (!(*reinterpret_cast<const float*>(mask_base + off) > 0.f)) v = 0.f;
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    *reinterpret_cast<float*>(hi_base + off) = h;
    *reinterpret_cast<float*>(lo_base + off) = v - h;
}

// Stores v as a tf32-exact high part and the float32 remainder.
__device__ __forceinline__ void st_split(unsigned char* hi_base, unsigned char* lo_base, uint32_t off, float v) {
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    *reinterpret_cast<float*>(hi_base + off) = h;
    *reinterpret_cast<float*>(lo_base + off) = v - h;
}

// Bounded wait for an mbarrier phase; false (and an error record) on timeout.
__device__ __noinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(mbar, parity)) return true;
        const int r = backoff(it, t0, w);
        if (r) {
            if (r == 1) record_error(w, kStatusTimeout, 4, parity, 0);
            return false;
        }
    }
}

}  // namespace tc

using namespace tc;

// Grid: x = (tiles_x + tiles_y) * n_fblk, y = problem.  blockIdx.x below
// tiles_x * n_fblk computes a grad_x tile, the rest grad_y tiles.
//
// Loading the G tile.  A 128 x 32 tile of G is skewed in the wavefront layout
// (cell (q, j) of stripe s sits in anti-diagonal row t = q_local + j), so each
// warp walks one "diagonal" d of the tile per iteration: lane l takes the slot
// of its row whose column makes t = const (or const + 32 m), which puts the 32
// lanes on at most K+1 anti-diagonal rows at consecutive positions (coalesced)
// and makes every loaded element a slot of this tile (no waste).  With
//   grad_x: rows q (tile), K = j (chunk): lane l, sub-row k: qloc = l*K + k,
//           kk = (d - qloc) mod 32, t = k0 + qloc + kk
//   grad_y: rows j (tile), K = q (chunk): lane pi: qloc = qb + pi,
//           jr = (d - pi) mod 128, t = r0 + qloc + jr
// 128 warp-iterations cover the 4096 slots of the tile: 16 per thread.  A
// slot's wavefront-layout offset relative to a per-chunk base, its
// shared-memory offset and its validity do not change from chunk to chunk, so
// they are computed once; only the last chunk (partial in K) checks the
// column or row against the sequence length.  The B tile is the block of 32
// rows of x or y; its ones column and zero padding never change and are
// written once.
//
// Pipeline: every thread copies its slots with 4-byte cp.async straight into
// the high-part buffer of a stage (zero-filled where out of range), up to
// `stages - 1` chunks ahead; when a chunk has landed, each thread splits its
// own slots in place (high part, remainder into the low-part buffer, the
// clamp mask applied from a third buffer), then one thread issues the MMAs.
// A stage is refilled once the mbarrier of its previous MMAs has completed.
template <int K, int NB, bool is_x>
__device__ __forceinline__ void grad_tile(const GradTcArgs& a, unsigned char* smem_raw) {
    constexpr int SR = 32 * K;
    constexpr int APER = kTileM * kKT / kThreads;  // A slots per thread (16)
    const WavePlan& P = a.P;
    const int N = P.N, M = P.M, dim = a.dim;
    const int b = blockIdx.y;
    const int nt = a.nt;
    const int fb = a.fb;
    const int S = a.stages;
    const bool masked = a.Mw != nullptr;
    const int local = is_x ? blockIdx.x : blockIdx.x - a.tiles_x * a.n_fblk;
    const int tile = local / a.n_fblk;
    const int f0 = (local % a.n_fblk) * fb;  // first feature of this block
    const int r0 = tile * kTileM;            // first output row (q for grad_x, j for grad_y)
    const int k_total = is_x ? M : N;        // contraction length
    const int rows_other = is_x ? M : N;
    const int n_chunks = (k_total + kKT - 1) / kKT;
    const float* __restrict__ Ew = a.Ew;
    const float* __restrict__ Mw = a.Mw;
    const float* __restrict__ ob = (is_x ? a.y : a.x) + static_cast<size_t>(b) * rows_other * dim + f0;
    const size_t prob = static_cast<size_t>(b) * P.n_stripes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Shared memory per stage: A_hi, A_lo (128 x 32), [mask raw (128 x 32)],
    // B_hi, B_lo (nt x 32); then the mbarriers and the tensor-memory address.
    const uint32_t a_bytes = kTileM / 8 * kSBO;
    const uint32_t b_bytes = static_cast<uint32_t>(nt) / 8 * kSBO;
    const uint32_t m_bytes = masked ? a_bytes : 0u;
    const uint32_t stage_bytes = 2 * a_bytes + m_bytes + 2 * b_bytes;
    unsigned char* ctrl = smem_raw + S * stage_bytes;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ctrl);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 64);
    const uint32_t smem_base = smem_addr(smem_raw);
    auto sA_hi = [&](int st) { return smem_raw + st * stage_bytes; };
    auto sMk = [&](int st) { return smem_raw + st * stage_bytes + 2 * a_bytes; };
    auto sB_hi = [&](int st) { return smem_raw + st * stage_bytes + 2 * a_bytes + m_bytes; };

    WaitCtx wc = a.wait;
    wc.kernel = 5;
    wc.problem = b;
    wc.warp = blockIdx.x;
    wc.band = 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) mbar_init(smem_addr(mbar + s), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), static_cast<uint32_t>(a.tmem_cols));
        tmem_relinquish();
    }
    // Constant B columns of every stage: ones at fb (row/column sums), zeros
    // above it.
    for (int e = threadIdx.x; e < (nt - fb) * kKT; e += kThreads) {
        const int f = fb + e % (nt - fb);
        const int kk = e / (nt - fb);
        for (int s = 0; s < S; ++s) {
            unsigned char* bh = sB_hi(s);
            const float v = f == fb ? 1.f : 0.f;
            *reinterpret_cast<float*>(bh + op_off(f, kk)) = v;
            *reinterpret_cast<float*>(bh + b_bytes + op_off(f, kk)) = 0.f;
        }
    }

    // ---- per-thread slots (chunk-invariant).
    // A: wavefront-layout offset relative to the chunk base; meta = shared
    // offset | kk << 16 (grad_x: column in the chunk) | valid << 24.
    uint32_t a_goff[APER], a_meta[APER];
#pragma unroll
    for (int i = 0; i < APER; ++i) {
        const int it = warp + (kThreads / 32) * i;
        uint32_t goff, soff, kk = 0, valid;
        if constexpr (is_x) {
            const int d = it & 31;
            const int rest = it >> 5;  // (stripe of the tile, sub-row)
            const int k = rest % K;
            const int sl = rest / K;
            const int qloc = lane * K + k;
            const int c = (d - qloc) & 31;
            goff = static_cast<uint32_t>((sl * P.n_diag + qloc + c) * SR + k * 32 + lane);
            soff = op_off(sl * SR + qloc, c);
            kk = static_cast<uint32_t>(c);
            valid = (r0 + sl * SR + qloc) < N;
        } else {
            const int jr = (it - lane) & (kTileM - 1);
            goff = static_cast<uint32_t>((jr + lane) * SR + (lane % K) * 32 + lane / K);
            soff = op_off(jr, lane);
            valid = (r0 + jr) < M;
        }
        a_goff[i] = goff;
        a_meta[i] = soff | (kk << 16) | (valid << 24);
    }
    // B: the rows k0 .. k0+31 of x or y, features f0 .. f0+fb-1: element e of
    // the block (row e / fb, feature e % fb).  meta = shared offset | row << 16 |
    // slot exists << 24 | feature in range << 25.
    const int nb_elems = kKT * fb;
    uint32_t b_goff[NB], b_meta[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u) {
        const int e = threadIdx.x + kThreads * u;
        const int kk = e / fb, f = e - (e / fb) * fb;  // kk < 32 whenever e < nb_elems
        const bool exists = e < nb_elems;
        const bool fin = exists && f0 + f < dim;
        b_goff[u] = fin ? static_cast<uint32_t>(kk * dim + f) : 0u;
        b_meta[u] = exists ? (op_off(f, kk) | (static_cast<uint32_t>(kk) << 16) | (1u << 24) |
                              (static_cast<uint32_t>(fin) << 25))
                           : 0u;
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = idesc_tf32(kTileM, nt);

    auto issue_chunk = [&](int c) {
        const int st = c % S;
        const int k0 = c * kKT;
        const bool last = (c == n_chunks - 1);
        size_t base;
        if constexpr (is_x) {
            base = ((prob + r0 / SR) * P.n_diag + k0) * SR;
        } else {
            const int s = k0 / SR;
            const int qb = k0 - s * SR;
            base = ((prob + s) * P.n_diag + r0 + qb) * SR + qb / K;
        }
        const float* Eb = Ew + base;
        const float* Mb = masked ? Mw + base : nullptr;
        const bool q_ok = is_x || (k0 + lane < N);  // grad_y: this lane's column q
        const uint32_t dA = smem_addr(sA_hi(st));
        const uint32_t dM = smem_addr(sMk(st));
#pragma unroll
        for (int i = 0; i < APER; ++i) {
            bool ok = (a_meta[i] >> 24) & 1u;
            if constexpr (is_x) ok = ok && (!last || k0 + static_cast<int>((a_meta[i] >> 16) & 0xFFu) < M);
            else ok = ok && q_ok;
            const uint32_t off = a_meta[i] & 0xFFFFu;
            const uint32_t g = ok ? a_goff[i] : 0u;  // in range either way: nothing is read when !ok
            cp_async4(dA + off, Eb + g, ok ? 4u : 0u);
            if (masked) cp_async4(dM + off, Mb + g, ok ? 4u : 0u);
        }
        const float* Bb = ob + static_cast<size_t>(k0) * dim;
        const uint32_t dB = smem_addr(sB_hi(st));
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            if ((b_meta[u] >> 24) & 1u) {
                const bool ok = ((b_meta[u] >> 25) & 1u) &&
                                (!last || k0 + static_cast<int>((b_meta[u] >> 16) & 0xFFu) < rows_other);
                cp_async4(dB + (b_meta[u] & 0xFFFFu), ok ? Bb + b_goff[u] : ob, ok ? 4u : 0u);
            }
        }
    };
    auto split_chunk = [&](int st) {
        unsigned char* ah = sA_hi(st);
        unsigned char* bh = sB_hi(st);
        if (masked) {
            const unsigned char* mk = sMk(st);
#pragma unroll
            for (int i = 0; i < APER; ++i) split_in_place_masked(ah, ah + a_bytes, mk, a_meta[i] & 0xFFFFu);
        } else {
#pragma unroll
            for (int i = 0; i < APER; ++i) split_in_place(ah, ah + a_bytes, a_meta[i] & 0xFFFFu);
        }
#pragma unroll
        for (int u = 0; u < NB; ++u)
            if ((b_meta[u] >> 24) & 1u) split_in_place(bh, bh + b_bytes, b_meta[u] & 0xFFFFu);
    };

    bool ok = true;
    // Prologue: chunks 0 .. S-2 in flight (one commit group per chunk slot, empty or not).
    for (int c = 0; c < S - 1; ++c) {
        if (c < n_chunks) issue_chunk(c);
        cp_async_commit();
    }
    for (int c = 0; c < n_chunks; ++c) {
        const int st = c % S;
        // Groups committed so far: chunks 0 .. c+S-2; chunk c's is complete when
        // at most S-2 newer ones are pending.
        if (S == 3) cp_async_wait<1>();
        else cp_async_wait<0>();
        split_chunk(st);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (threadIdx.x == 0 && ok) {
            const uint32_t aH = smem_base + static_cast<uint32_t>(sA_hi(st) - smem_raw);
            const uint32_t aL = aH + a_bytes;
            const uint32_t bH = smem_base + static_cast<uint32_t>(sB_hi(st) - smem_raw);
            const uint32_t bL = bH + b_bytes;
#pragma unroll
            for (int ks = 0; ks < kKT / 8; ++ks) {
                const uint32_t o = static_cast<uint32_t>(ks) * 2 * kLBO;
                const uint32_t acc0 = (c > 0 || ks > 0) ? 1u : 0u;
                mma_tf32(tmem, smem_desc(aH + o), smem_desc(bH + o), idesc, acc0);
                mma_tf32(tmem, smem_desc(aH + o), smem_desc(bL + o), idesc, 1u);
                mma_tf32(tmem, smem_desc(aL + o), smem_desc(bH + o), idesc, 1u);
            }
            mma_commit(smem_addr(mbar + st));
        }
        // Refill the stage of chunk c-1 with chunk c+S-1 once its MMAs are done.
        const int nc = c + S - 1;
        if (nc < n_chunks) {
            if (c >= 1 && ok) {
                const int pc = c - 1;
                ok = mbar_wait(smem_addr(mbar + pc % S), static_cast<uint32_t>((pc / S) & 1), wc);
            }
            issue_chunk(nc);
        }
        cp_async_commit();
    }
    // All MMAs done: the last commit covers every earlier one.
    if (n_chunks > 0 && ok) {
        const int cl = n_chunks - 1;
        ok = mbar_wait(smem_addr(mbar + cl % S), static_cast<uint32_t>((cl / S) & 1), wc);
    }
    cp_async_wait<0>();
    tc_fence_after();
    const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;

    if (all_ok) {
        // ---- epilogue: warp w reads tensor-memory lanes 32*(w%4) (tile rows),
        // column chunks of 16 alternating between the two warp groups.
        const int quarter = warp & 3;
        const int half = warp >> 2;
        const int r = r0 + quarter * 32 + lane;
        const int rows_out = is_x ? N : M;
        const float* own = is_x ? a.x : a.y;
        float* g = is_x ? a.gx : a.gy;
        const uint32_t tw = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float v[16];
        tmem_ld16(tw + static_cast<uint32_t>((fb / 16) * 16), v);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (i == fb % 16) sum = v[i];
        const size_t row_off = (static_cast<size_t>(b) * rows_out + r) * dim + f0;
        const bool vec = ((dim & 3) == 0) && ((f0 & 3) == 0) &&
                         ((reinterpret_cast<uintptr_t>(own) | reinterpret_cast<uintptr_t>(g)) & 15u) == 0;
        for (int c16 = half; c16 * 16 < fb; c16 += 2) {  // warp-uniform
            tmem_ld16(tw + static_cast<uint32_t>(c16 * 16), v);
            if (r < rows_out) {
                const int fl = c16 * 16;  // first feature of the chunk, within the block
                if (vec && fl + 16 <= fb && f0 + fl + 16 <= dim) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 o = __ldg(reinterpret_cast<const float4*>(own + row_off + fl) + u);
                        float4 w;
                        w.x = 2.f * (o.x * sum - v[4 * u + 0]);
                        w.y = 2.f * (o.y * sum - v[4 * u + 1]);
                        w.z = 2.f * (o.z * sum - v[4 * u + 2]);
                        w.w = 2.f * (o.w * sum - v[4 * u + 3]);
                        reinterpret_cast<float4*>(g + row_off + fl)[u] = w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int f = fl + i;
                        if (f < fb && f0 + f < dim) g[row_off + f] = 2.f * (__ldg(own + row_off + f) * sum - v[i]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(a.tmem_cols));
}

template <int K, int NB>
__global__ void __launch_bounds__(kThreads, 1) grad_tc_kernel(const GradTcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    if (static_cast<int>(blockIdx.x) < a.tiles_x * a.n_fblk) grad_tile<K, NB, true>(a, smem_raw);
    else grad_tile<K, NB, false>(a, smem_raw);
}

// Feature blocking: N of the MMA = features of the block + the ones column,
// rounded up to 16 (M = 128 needs N % 16 == 0, N <= 256).  With the clamp
// mask a stage holds one more 128 x 32 buffer, so blocks are narrower.
void grad_tc_geometry(int dim, bool masked, int* fb, int* nt, int* n_fblk, int* tmem_cols, int* stages) {
    const int fmax = masked ? 176 : 240;
    const int f = dim <= fmax ? dim : fmax;
    *fb = f;
    *nt = ((f + 1) + 15) / 16 * 16;
    *n_fblk = (dim + f - 1) / f;
    int tc = 32;
    while (tc < *nt) tc *= 2;
    *tmem_cols = tc;
    const size_t stage = (masked ? 3u : 2u) * (kTileM / 8) * kSBO + 2u * static_cast<size_t>(*nt) / 8 * kSBO;
    *stages = (3 * stage + 128 <= 227u * 1024u) ? 3 : 2;
}

static size_t grad_tc_smem_bytes(const GradTcArgs& a) {
    const size_t stage = (a.Mw ? 3u : 2u) * (kTileM / 8) * kSBO + 2u * static_cast<size_t>(a.nt) / 8 * kSBO;
    return static_cast<size_t>(a.stages) * stage + 128u;
}

template <int K, int NB>
static cudaError_t grad_tc_go(const GradTcArgs& args, dim3 grid, size_t smem, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(grad_tc_kernel<K, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    grad_tc_kernel<K, NB><<<grid, kThreads, smem, stream>>>(args);
    return cudaGetLastError();
}

template <int K>
static cudaError_t grad_tc_by_nb(const GradTcArgs& args, dim3 grid, size_t smem, cudaStream_t stream) {
    // B elements per thread: 32 rows x fb features over 256 threads.
    const int nb = (kKT * args.fb + kThreads - 1) / kThreads;
    if (nb <= 4) return grad_tc_go<K, 4>(args, grid, smem, stream);
    if (nb <= 8) return grad_tc_go<K, 8>(args, grid, smem, stream);
    if (nb <= 16) return grad_tc_go<K, 16>(args, grid, smem, stream);
    return grad_tc_go<K, 30>(args, grid, smem, stream);
}

cudaError_t launch_grad_tc(const GradTcArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (args.stages < 2 || args.stages > 3) return cudaErrorInvalidValue;
    const size_t smem = grad_tc_smem_bytes(args);
    dim3 grid((args.tiles_x + args.tiles_y) * args.n_fblk, P.B);
    switch (P.K) {
        case 1: return grad_tc_by_nb<1>(args, grid, smem, stream);
        case 2: return grad_tc_by_nb<2>(args, grid, smem, stream);
        case 4: return grad_tc_by_nb<4>(args, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

// ============================================================== unfused cost
// D = clamp(||x_q||^2 + ||y_j||^2 - 2 x_q . y_j, 0) in the wavefront layout,
// the expanded squared-Euclidean cost of softdtw_cuda/distances.py:6-28 with
// the dot products on the tensor cores (3xTF32, float32 accumulators in
// tensor memory).  One CTA (8 warps) per 128 x 128 tile (rows q, columns j) of
// one problem; K = features in chunks of 32, two stages fed by 16-byte
// cp.async (rows are 16-byte aligned: dim % 4 == 0), split in place into high
// parts and remainders.  Consecutive threads take consecutive rows of the same
// 16-byte column (conflict-free shared stores); each thread also sums the
// squares of the elements it splits, and the two threads of a row add their
// sums in a fixed order.  The
// epilogue writes the tile's cells into shared memory by anti-diagonal and
// stores anti-diagonal rows of the layout (cells of neighbouring tiles in the
// same rows are left alone).
constexpr int kCostStages = 2;

template <int K>
__global__ void __launch_bounds__(kThreads, 1) cost_tc_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                              float* __restrict__ Dw, const WavePlan P, int dim,
                                                              const WaitCtx wait) {
    constexpr int SR = 32 * K;
    constexpr int NSL = kTileM / SR;       // stripes in the 128-row tile
    constexpr int TL = SR + kTileM - 1;    // anti-diagonal rows of one stripe slice
    constexpr int UPT = kTileM * kKT / 4 / kThreads;  // 16-byte units per thread per operand (4)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const int N = P.N, M = P.M;
    const int j0 = blockIdx.x * kTileM;
    const int q0 = blockIdx.y * kTileM;
    const int b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t op_bytes = kTileM / 8 * kSBO;     // one 128 x 32 operand buffer
    const uint32_t stage_bytes = 4 * op_bytes;       // A_hi, A_lo, B_hi, B_lo
    unsigned char* ctrl = smem_raw + kCostStages * stage_bytes;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ctrl);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 64);
    float* xn = reinterpret_cast<float*>(ctrl + 128);  // [2][128] partial, then [128]
    float* yn = xn + 2 * kTileM;                      // [2][128] partial, then [128]
    const uint32_t smem_base = smem_addr(smem_raw);
    const float* xb = x + static_cast<size_t>(b) * N * dim;
    const float* yb = y + static_cast<size_t>(b) * M * dim;
    const int n_chunks = (dim + kKT - 1) / kKT;

    WaitCtx wc = wait;
    wc.kernel = 6;
    wc.problem = b;
    wc.warp = blockIdx.x;
    wc.band = blockIdx.y;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kCostStages; ++s) mbar_init(smem_addr(mbar + s), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), 128u);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = idesc_tf32(kTileM, kTileM);

    // Unit u = threadIdx.x + 256 i: row u % 128, features 4 (u / 128) .. +3 of
    // the chunk; a thread keeps one row (threadIdx.x % 128).
    const int urow = threadIdx.x & (kTileM - 1);
    float xs2 = 0.f, ys2 = 0.f;  // partial squared norms of the thread's row
    auto issue = [&](int c) {
        const int st = c % kCostStages;
        const uint32_t dA = smem_base + st * stage_bytes;
        const uint32_t dB = dA + 2 * op_bytes;
        const int f0 = c * kKT;
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
            const int u = threadIdx.x + kThreads * i;
            const int row = u & (kTileM - 1), kc = u >> 7;
            const int f = f0 + 4 * kc;
            const bool fx = q0 + row < N && f < dim;
            const bool fy = j0 + row < M && f < dim;
            const uint32_t off = op_off(row, 4 * kc);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dA + off),
                         "l"(fx ? xb + static_cast<size_t>(q0 + row) * dim + f : xb), "r"(fx ? 16u : 0u)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dB + off),
                         "l"(fy ? yb + static_cast<size_t>(j0 + row) * dim + f : yb), "r"(fy ? 16u : 0u)
                         : "memory");
        }
    };
    auto split = [&](int c) {
        const int st = c % kCostStages;
        unsigned char* A = smem_raw + st * stage_bytes;
        unsigned char* Bm = A + 2 * op_bytes;
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
            const int u = threadIdx.x + kThreads * i;
            const uint32_t off = op_off(u & (kTileM - 1), 4 * (u >> 7));
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                unsigned char* hi = o == 0 ? A : Bm;
                float4 v = *reinterpret_cast<const float4*>(hi + off);
                float4 h, l;
                h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
                h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
                h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
                h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
                l.x = v.x - h.x;
                l.y = v.y - h.y;
                l.z = v.z - h.z;
                l.w = v.w - h.w;
                *reinterpret_cast<float4*>(hi + off) = h;
                *reinterpret_cast<float4*>(hi + op_bytes + off) = l;
                float& acc = o == 0 ? xs2 : ys2;
                acc = fmaf(v.x, v.x, acc);
                acc = fmaf(v.y, v.y, acc);
                acc = fmaf(v.z, v.z, acc);
                acc = fmaf(v.w, v.w, acc);
            }
        }
    };

    bool ok = true;
    issue(0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int c = 0; c < n_chunks; ++c) {
        const int st = c % kCostStages;
        // Refill the other stage with chunk c+1 once the MMAs of chunk c-1 are done.
        if (c + 1 < n_chunks) {
            if (c >= 1 && ok) ok = mbar_wait(smem_addr(mbar + (c - 1) % kCostStages), static_cast<uint32_t>(((c - 1) / kCostStages) & 1), wc);
            issue(c + 1);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        split(c);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (threadIdx.x == 0 && ok) {
            const uint32_t aH = smem_base + st * stage_bytes;
            const uint32_t aL = aH + op_bytes;
            const uint32_t bH = aL + op_bytes;
            const uint32_t bL = bH + op_bytes;
#pragma unroll
            for (int ks = 0; ks < kKT / 8; ++ks) {
                const uint32_t o = static_cast<uint32_t>(ks) * 2 * kLBO;
                const uint32_t acc0 = (c > 0 || ks > 0) ? 1u : 0u;
                mma_tf32(tmem, smem_desc(aH + o), smem_desc(bH + o), idesc, acc0);
                mma_tf32(tmem, smem_desc(aH + o), smem_desc(bL + o), idesc, 1u);
                mma_tf32(tmem, smem_desc(aL + o), smem_desc(bH + o), idesc, 1u);
            }
            mma_commit(smem_addr(mbar + st));
        }
    }
    // Squared norms: threads r and r + 128 hold the two halves of row r.
    xn[(threadIdx.x >> 7) * kTileM + urow] = xs2;
    yn[(threadIdx.x >> 7) * kTileM + urow] = ys2;
    if (n_chunks > 0 && ok) {
        const int cl = n_chunks - 1;
        ok = mbar_wait(smem_addr(mbar + cl % kCostStages), static_cast<uint32_t>((cl / kCostStages) & 1), wc);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    tc_fence_after();
    const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
    if (threadIdx.x < kTileM) {
        xn[threadIdx.x] = xn[threadIdx.x] + xn[kTileM + threadIdx.x];
        yn[threadIdx.x] = yn[threadIdx.x] + yn[kTileM + threadIdx.x];
    }
    __syncthreads();

    if (all_ok) {
        // ---- epilogue: warp w holds tile rows 32 (w % 4) + lane, columns of
        // half w / 4; cells go to shared memory by (stripe slice, anti-diagonal).
        float* stg = reinterpret_cast<float*>(smem_raw);  // [NSL][TL][SR]
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;
        const int sl = r / SR, ql = r % SR;
        const int p = (ql % K) * 32 + ql / K;
        const float xr = xn[r];
        const uint32_t tw = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float v[16];
        for (int c16 = half * 4; c16 < half * 4 + 4; ++c16) {
            tmem_ld16(tw + static_cast<uint32_t>(c16 * 16), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int c = c16 * 16 + i;
                const float d = fmaxf((xr + yn[c]) - 2.f * v[i], 0.f);
                stg[(sl * TL + ql + c) * SR + p] = d;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 128u);
    if (all_ok) {
        const float* stg = reinterpret_cast<const float*>(smem_raw);
        for (int e = threadIdx.x; e < NSL * TL * SR; e += kThreads) {
            const int pp = e % SR;
            const int tl = (e / SR) % TL;
            const int sl = e / (SR * TL);
            const int ql = (pp % 32) * K + pp / 32;
            const int jl = tl - ql;   // column within the tile
            const int q = q0 + sl * SR + ql;
            const int j = j0 + jl;
            if (jl >= 0 && jl < kTileM && j < M && q < N) {
                const int s = q / SR;
                const int t = ql + j;
                Dw[((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + t) * SR + pp] = stg[e];
            }
        }
    }
}

static size_t cost_tc_smem_bytes(int K) {
    const size_t ops = static_cast<size_t>(kCostStages) * 4 * (kTileM / 8) * kSBO;
    const size_t stage = static_cast<size_t>(kTileM / (32 * K)) * (32 * K + kTileM - 1) * (32 * K) * sizeof(float);
    return (ops > stage ? ops : stage) + 128 + 4 * kTileM * sizeof(float);
}

bool cost_tc_supported(const float* x, const float* y, int dim) {
    return dim >= 16 && dim % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) == 0;
}

cudaError_t launch_cost_tc(const float* x, const float* y, float* Dw, const WavePlan& P, int dim, const WaitCtx& wait,
                           cudaStream_t stream) {
    const dim3 grid((P.M + kTileM - 1) / kTileM, (P.N + kTileM - 1) / kTileM, P.B);
    const size_t smem = cost_tc_smem_bytes(P.K);
    cudaError_t e = cudaSuccess;
    switch (P.K) {
        case 1:
            e = cudaFuncSetAttribute(cost_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e == cudaSuccess) cost_tc_kernel<1><<<grid, kThreads, smem, stream>>>(x, y, Dw, P, dim, wait);
            break;
        case 2:
            e = cudaFuncSetAttribute(cost_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e == cudaSuccess) cost_tc_kernel<2><<<grid, kThreads, smem, stream>>>(x, y, Dw, P, dim, wait);
            break;
        case 4:
            e = cudaFuncSetAttribute(cost_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e == cudaSuccess) cost_tc_kernel<4><<<grid, kThreads, smem, stream>>>(x, y, Dw, P, dim, wait);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace sdtw
