// tcgemm.cu -- the chain rule of the squared-Euclidean cost on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory), in 3xTF32 so that the
// result keeps float32 accuracy.
//
//   grad_x[b,q,:] = 2 (x_q * sum_j G(q,j) - sum_j G(q,j) y_j)
//   grad_y[b,j,:] = 2 (y_j * sum_q G(q,j) - sum_q G(q,j) x_q)
//
// G = E, the reverse pass's output (fused cost), or E * (D > 0), the clamp mask
// of the unfused cost.  This replaces the two bmm of
// softdtw_cuda/autograd_xy.py:41-49 (fused) and torch's autograd of
// softdtw_cuda/distances.py:20-28 (unfused).
//
// One CTA (8 warps) computes a 128-row output tile (rows q for grad_x, rows j
// for grad_y) for one block of features.  Per K chunk of 32 it stages the G tile
// and the x or y tile in shared memory, each split into a tf32-exact high part
// (low 13 mantissa bits cleared) and the float32 remainder; one thread issues
// the tcgen05.mma kind::tf32 instructions (M = 128, K = 8 per instruction) into
// float32 accumulators in tensor memory, and the MMAs signal completion through
// an mbarrier (tcgen05.commit).  The epilogue reads the accumulator with
// tcgen05.ld (warp w may read tensor-memory lanes 32(w%4)..32(w%4)+31, i.e.
// those tile rows; the two warp groups take alternate 16-column chunks).
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include <cudaTypedefs.h>

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

// Bounded wait for an mbarrier phase; false (and an error record) on timeout.
__device__ __noinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
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

}  // namespace tc

using namespace tc;

// ============================================================== gradients from row-major G
// The same contractions from operands in plain row-major layouts, so that
// every operand load is a coalesced 16-byte load: grad_x's A = G (rows q,
// K = j) and B = y^T (rows = features, K = j); grad_y's A = G^T (rows j,
// K = q) and B = x^T (rows = features, K = q).  G and G^T (clamp mask applied)
// come from the wavefront layout through wl_to_rm_cm_kernel, x^T and y^T from
// transpose_kernel; each has its rows padded with zeros to a multiple of 32
// floats, so a K chunk never needs a bound check.
//
// Each thread loads its 16-byte units of a chunk into registers two chunks
// ahead, splits them there into the tf32 high part and the remainder, and
// stores both into one of two shared-memory buffers.  B is stored as
// B' = [B_lo ; B_hi ; ones(16)], so that 3xTF32 and the row sums take two MMAs
// per K step (A is read twice, not three times, from shared memory):
//     D[:, 0 .. 2nt+16)   += A_hi * B'          (N = 2nt + 16)
//     D[:, nt .. 2nt+16)  += A_lo * [B_hi ; 1]  (N = nt + 16)
// giving A*B = D[:, 0..nt) + D[:, nt..2nt) and sum_k A = D[:, 2nt].  nt <= 112
// keeps N <= 256 and (at nt <= 64) two CTAs per SM.
constexpr int kRmMaxNt = 112;

// Thread t's i-th 16-byte unit of a 32-wide K chunk (i < 4): row
// 8 * (c >> 1) + (lane & 7), column 4 * (4 * (c & 1) + (lane >> 3)) with
// c = warp + 8 i; 8 consecutive lanes cover 8 rows of one 16-byte column, 128
// contiguous bytes of the shared-memory layout (no bank conflicts), and each
// row is read as two full 32-byte sectors.
__device__ __forceinline__ int rm_row(int warp, int lane, int i) { return 8 * ((warp + 8 * i) >> 1) + (lane & 7); }
__device__ __forceinline__ int rm_col(int warp, int lane, int i) {
    return 4 * (4 * ((warp + 8 * i) & 1) + (lane >> 3));
}

__device__ __forceinline__ void st_split4(unsigned char* hi, unsigned char* lo, uint32_t off_hi, uint32_t off_lo,
                                          float4 v) {
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    l.x = v.x - h.x;
    l.y = v.y - h.y;
    l.z = v.z - h.z;
    l.w = v.w - h.w;
    *reinterpret_cast<float4*>(hi + off_hi) = h;
    *reinterpret_cast<float4*>(lo + off_lo) = l;
}

template <int S>
using Slot = std::integral_constant<int, S>;

template <bool GX>
__device__ __forceinline__ void grad_rm_tile(const GradTcArgs& a, unsigned char* smem_raw) {
    const WavePlan& P = a.P;
    const int N = P.N, M = P.M, dim = a.dim;
    const int b = blockIdx.y;
    const int nt = a.nt;  // B rows: the feature block rounded up to 16
    const int fb = a.fb;
    const int local = GX ? blockIdx.x : blockIdx.x - a.tiles_x * a.n_fblk;
    const int tile = local / a.n_fblk;
    const int f0 = (local % a.n_fblk) * fb;
    const int r0 = tile * kTileM;
    const int rows_out = GX ? N : M;  // rows of A (output rows)
    const int kt = GX ? M : N;        // contraction length
    const int ld = (kt + 31) & ~31;   // row pitch of A and of B
    const int n_chunks = ld / kKT;
    const float* __restrict__ Ag = (GX ? a.G : a.GT) + static_cast<size_t>(b) * rows_out * ld;
    const float* __restrict__ Bg = (GX ? a.yT : a.xT) + static_cast<size_t>(b) * dim * ld;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b_units = nt / 4;  // (row group, column half) pairs of B

    const uint32_t a_bytes = kTileM / 8 * kSBO;
    const uint32_t b_bytes = static_cast<uint32_t>(2 * nt + 16) / 8 * kSBO;
    const uint32_t buf_bytes = 2 * a_bytes + b_bytes;
    unsigned char* ctrl = smem_raw + 2 * buf_bytes;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ctrl);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 64);
    const uint32_t smem_base = smem_addr(smem_raw);

    WaitCtx wc = a.wait;
    wc.kernel = 5;
    wc.problem = b;
    wc.warp = blockIdx.x;
    wc.band = 1;

    if (threadIdx.x == 0) {
        mbar_init(smem_addr(mbar + 0), 1);
        mbar_init(smem_addr(mbar + 1), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), static_cast<uint32_t>(a.tmem_cols));
        tmem_relinquish();
    }
    for (int e = threadIdx.x; e < 2 * 16 * kKT; e += kThreads) {  // the ones rows of both buffers
        const int bi = e / (16 * kKT), r = (e / kKT) % 16, k = e % kKT;
        *reinterpret_cast<float*>(smem_raw + bi * buf_bytes + 2 * a_bytes + op_off(2 * nt + r, k)) = 1.f;
    }

    float4 ra[2][4], rb[2][4];
    auto load = [&](auto slot, int c) {
        constexpr int S = decltype(slot)::value;
        const int k0 = c * kKT;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = r0 + rm_row(warp, lane, i);
            ra[S][i] = row < rows_out
                           ? __ldg(reinterpret_cast<const float4*>(Ag + static_cast<size_t>(row) * ld + k0 +
                                                                   rm_col(warp, lane, i)))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int fr = rm_row(warp, lane, i);
            const bool ok = warp + 8 * i < b_units && fr < fb && f0 + fr < dim;
            rb[S][i] = ok ? __ldg(reinterpret_cast<const float4*>(Bg + static_cast<size_t>(f0 + fr) * ld + k0 +
                                                                  rm_col(warp, lane, i)))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](auto slot, int c) {
        constexpr int S = decltype(slot)::value;
        unsigned char* Ah = smem_raw + (c & 1) * buf_bytes;
        unsigned char* Al = Ah + a_bytes;
        unsigned char* Bp = Al + a_bytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t off = op_off(rm_row(warp, lane, i), rm_col(warp, lane, i));
            st_split4(Ah, Al, off, off, ra[S][i]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (warp + 8 * i < b_units) {
                const int fr = rm_row(warp, lane, i), k = rm_col(warp, lane, i);
                st_split4(Bp, Bp, op_off(nt + fr, k), op_off(fr, k), rb[S][i]);
            }
        }
    };

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc1 = idesc_tf32(kTileM, 2 * nt + 16);
    const uint32_t idesc2 = idesc_tf32(kTileM, nt + 16);

    bool ok = true;
    auto step = [&](auto slot, int c) {
        if (c >= 2 && ok) ok = mbar_wait(smem_addr(mbar + (c & 1)), static_cast<uint32_t>(((c - 2) >> 1) & 1), wc);
        store(slot, c);
        if (c + 2 < n_chunks) load(slot, c + 2);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (threadIdx.x == 0 && ok) {
            const uint32_t aH = smem_base + (c & 1) * buf_bytes;
            const uint32_t aL = aH + a_bytes;
            const uint32_t bP = aL + a_bytes;
            const uint32_t bH = bP + static_cast<uint32_t>(nt / 8) * kSBO;
#pragma unroll
            for (int ks = 0; ks < kKT / 8; ++ks) {
                const uint32_t o = static_cast<uint32_t>(ks) * 2 * kLBO;
                mma_tf32(tmem, smem_desc(aH + o), smem_desc(bP + o), idesc1, (c > 0 || ks > 0) ? 1u : 0u);
                mma_tf32(tmem + static_cast<uint32_t>(nt), smem_desc(aL + o), smem_desc(bH + o), idesc2, 1u);
            }
            mma_commit(smem_addr(mbar + (c & 1)));
        }
    };

    load(Slot<0>{}, 0);
    if (n_chunks > 1) load(Slot<1>{}, 1);
    for (int c = 0; c < n_chunks; c += 2) {
        step(Slot<0>{}, c);
        if (c + 1 < n_chunks) step(Slot<1>{}, c + 1);
    }
    if (ok) {
        const int cl = n_chunks - 1;
        ok = mbar_wait(smem_addr(mbar + (cl & 1)), static_cast<uint32_t>((cl >> 1) & 1), wc);
    }
    tc_fence_after();
    const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;

    if (all_ok) {
        const int quarter = warp & 3;
        const int half = warp >> 2;
        const int r = r0 + quarter * 32 + lane;
        const size_t rstride = static_cast<size_t>(rows_out) * dim;
        const float* own = GX ? a.x.at(b, rstride) : a.y.at(b, rstride);
        float* g = GX ? a.gx.at(b, rstride) : a.gy.at(b, rstride);
        const uint32_t tw = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float v[16], w[16];
        tmem_ld16(tw + static_cast<uint32_t>(2 * nt), v);
        const float sum = v[0];
        const size_t row_off = static_cast<size_t>(r) * dim + f0;
        const bool vec = ((dim & 3) == 0) && ((f0 & 3) == 0) &&
                         ((reinterpret_cast<uintptr_t>(own) | reinterpret_cast<uintptr_t>(g)) & 15u) == 0;
        for (int c16 = half; c16 * 16 < fb; c16 += 2) {  // warp-uniform
            tmem_ld16(tw + static_cast<uint32_t>(c16 * 16), v);
            tmem_ld16(tw + static_cast<uint32_t>(nt + c16 * 16), w);
            if (r < rows_out) {
                const int fl = c16 * 16;
                if (vec && fl + 16 <= fb && f0 + fl + 16 <= dim) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 o = __ldg(reinterpret_cast<const float4*>(own + row_off + fl) + u);
                        float4 y4;
                        y4.x = 2.f * (o.x * sum - (v[4 * u + 0] + w[4 * u + 0]));
                        y4.y = 2.f * (o.y * sum - (v[4 * u + 1] + w[4 * u + 1]));
                        y4.z = 2.f * (o.z * sum - (v[4 * u + 2] + w[4 * u + 2]));
                        y4.w = 2.f * (o.w * sum - (v[4 * u + 3] + w[4 * u + 3]));
                        reinterpret_cast<float4*>(g + row_off + fl)[u] = y4;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int f = fl + i;
                        if (f < fb && f0 + f < dim)
                            g[row_off + f] = 2.f * (__ldg(own + row_off + f) * sum - (v[i] + w[i]));
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(a.tmem_cols));
}

__global__ void __launch_bounds__(kThreads, 2) grad_rm_kernel(const GradTcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    if (static_cast<int>(blockIdx.x) < a.tiles_x * a.n_fblk) grad_rm_tile<true>(a, smem_raw);
    else grad_rm_tile<false>(a, smem_raw);
}

// Feature blocks of at most kRmMaxNt features, of equal size.
void grad_rm_geometry(int dim, int* fb, int* nt, int* n_fblk, int* tmem_cols, int* stages) {
    const int nb = (dim + kRmMaxNt - 1) / kRmMaxNt;
    *n_fblk = nb;
    *fb = (dim + nb - 1) / nb;
    *nt = (*fb + 15) / 16 * 16;
    int tc = 32;
    while (tc < 2 * *nt + 16) tc *= 2;
    *tmem_cols = tc;
    *stages = 2;
}

static size_t grad_rm_smem(int nt) {
    return 2u * (2u * (kTileM / 8) * kSBO + static_cast<size_t>(2 * nt + 16) / 8 * kSBO) + 128;
}

cudaError_t launch_grad_rm(const GradTcArgs& args, cudaStream_t stream) {
    const WavePlan& P = args.P;
    if (args.nt < 16 || args.nt > kRmMaxNt || args.nt % 16) return cudaErrorInvalidValue;
    const size_t smem = grad_rm_smem(args.nt);
    dim3 grid((args.tiles_x + args.tiles_y) * args.n_fblk, P.B);
    cudaError_t e = cudaFuncSetAttribute(grad_rm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    grad_rm_kernel<<<grid, kThreads, smem, stream>>>(args);
    return cudaGetLastError();
}

// ============================================================== gradients from the wavefront layout
// One row per lane (32-row stripes).  G is read straight from the wavefront
// layout by the bulk-copy engine into a ring of shared-memory slots (completion
// counted in bytes on an mbarrier) and de-skewed from there while it is split
// into the MMA operands.  B comes from x or y in a chunked transposed layout
// (xTc[b][c][f][kk] = x[b][32c + kk][f], rows of 36 floats), one copy of
// nf * 144 contiguous bytes per chunk.  Copies are few and large: the engine's
// cost is per copy, and 128-byte copies run far below bandwidth.
//
//   grad_x tile (rows q in [r0, r0 + 128) = 4 stripes, K = j): chunk c covers
//     j in [32c, 32c + 32), whose cells sit in anti-diagonal rows
//     t in [32c, 32c + 63) of each stripe.  Load unit k is the 32-row block
//     t in [32k, 32k + 32) of the 4 stripes (4 KB each, one copy per stripe)
//     and B chunk k - 1; chunk c reads units c and c + 1.  Lanes take 32
//     consecutive rows q (cell (q, t - q) at slot word t*32 + q: one bank per
//     lane) and each thread 4 consecutive j, stored as one 16-byte vector.
//   grad_y tile (rows j in [r0, r0 + 128), K = q): chunk c is stripe c, whose
//     cells sit in rows t in [r0, r0 + 159); load unit c is one 2-D tensor copy
//     of those rows with the 128-byte swizzle (16-byte column group g of row r
//     lands at group g ^ (r % 8)), plus B chunk c.  Lanes take 8 rows j x 4
//     consecutive q, which the swizzle puts on 32 different banks; the stores
//     are 4-byte, 128 contiguous bytes per warp.
//
// Per chunk: the warp 0 lanes issue the copies S - 1 units ahead; every thread
// waits for its chunk's units, loads and splits its A and B elements into
// registers, waits for the previous chunk's MMAs (one operand buffer), stores
// them, and thread 0 issues the MMAs.  Cells outside the table (q >= N,
// j >= M) and the clamp mask (unfused cost, D <= 0) become zeros in the split.
constexpr int kWlMaxNt = 128;
constexpr int kWlSplitWarps = 16;
constexpr uint32_t kBPitch = 144;  // bytes per row of the chunked transposed x, y
constexpr int kYRows = 159;        // anti-diagonal rows of one grad_y chunk

__device__ __forceinline__ void tensor2d_g2s(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
        : "memory");
}
// try_wait that lets the hardware suspend the thread (up to about 1 us) until
// the phase completes, so that waiting warps do not take issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t mbar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(mbar), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}
__device__ __noinline__ bool mbar_wait_sleep(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_sleep(mbar, parity)) return true;
        const int r = backoff(it << 8, t0, w);  // every poll checks the clock
        if (r) {
            record_giveup(w, r, 4, parity, 0);
            return false;
        }
    }
}
// Bounded wait with an inline fast path (the slow path is a call).
__device__ __forceinline__ bool mbar_wait_fast(uint32_t mbar, uint32_t parity, const WaitCtx& w) {
    if (mbar_try_wait(mbar, parity)) return true;
    return mbar_wait_sleep(mbar, parity, w);
}
// Warp-uniform bounded wait: lane 0 polls, the result is broadcast, and every
// lane then observes the completed phase itself (acquire).  ok = false skips.
__device__ __forceinline__ bool warp_wait(uint32_t mbar, uint32_t parity, const WaitCtx& w, bool ok) {
    int r = 0;
    if ((threadIdx.x & 31) == 0) r = ok && mbar_wait_fast(mbar, parity, w) ? 1 : 0;
    r = __shfl_sync(0xffffffffu, r, 0);
    if (r) (void)mbar_try_wait(mbar, parity);
    return r != 0;
}
__device__ __forceinline__ float split_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }
__device__ __forceinline__ float ld_shared_f32(uint32_t saddr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(saddr));
    return v;
}

// Offset (floats) of anti-diagonal row t of stripe s of problem b, one row per lane.
__device__ __forceinline__ size_t wl_row(const WavePlan& P, int b, int s, int t) {
    return ((static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag + t) * 32;
}

__host__ __device__ constexpr uint32_t round1k(uint32_t v) { return (v + 1023u) & ~1023u; }
__host__ __device__ constexpr uint32_t wl_ops_bytes(int nt) {
    return round1k(2u * (kTileM / 8) * kSBO + static_cast<uint32_t>(2 * nt + 16) / 8 * kSBO);
}
__host__ __device__ constexpr uint32_t wl_a_ring(bool gx) {
    return gx ? 4u * 32u * 128u : round1k(static_cast<uint32_t>(kYRows) * 128u);
}
__host__ __device__ constexpr uint32_t wl_slot_bytes(int nt, bool gx, bool masked) {
    return round1k((masked ? 2u : 1u) * wl_a_ring(gx) + static_cast<uint32_t>(nt) * kBPitch);
}

template <bool GX>
__device__ __forceinline__ void grad_wl_tile(const GradTcArgs& a, unsigned char* smem_dyn) {
    // The 128-byte swizzle of the tensor copies is a function of address bits
    // 4-9, so the slots start on 1024-byte boundaries (1 KB spare is allocated).
    unsigned char* smem_raw = smem_dyn + ((1024u - (smem_addr(smem_dyn) & 1023u)) & 1023u);
    const WavePlan& P = a.P;
    const int N = P.N, M = P.M, dim = a.dim;
    const int b = blockIdx.y;
    const int nt = a.nt, fb = a.fb;
    const int S = GX ? a.stages_x : a.stages_y;
    const int NO = GX ? a.ops_x : a.ops_y;  // operand buffers (1 or 2)
    const int local = GX ? blockIdx.x : blockIdx.x - a.tiles_x * a.n_fblk;
    const int tile = local / a.n_fblk;
    const int f0 = (local % a.n_fblk) * fb;
    const int nf = min(fb, dim - f0);  // feature rows of B actually present
    const int r0 = tile * kTileM;
    const int rows_out = GX ? N : M;
    const int kt = GX ? M : N;
    const int n_chunks = (kt + kKT - 1) / kKT;
    const int n_units = GX ? n_chunks + 1 : n_chunks;
    const bool masked = a.Mw != nullptr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* __restrict__ Bsrc = (GX ? a.yTc : a.xTc) + static_cast<size_t>(b) * n_chunks * dim * (kBPitch / 4);

    // Shared memory: [NO operand buffers: A_hi | A_lo | B' = B_lo ; B_hi ; ones]
    // [S ring slots: A | mask A | B] [barriers], 1024-byte aligned blocks.
    const uint32_t a_op = kTileM / 8 * kSBO;
    const uint32_t ops_bytes = wl_ops_bytes(nt);
    const uint32_t a_ring = wl_a_ring(GX);
    const uint32_t a_ring_all = masked ? 2 * a_ring : a_ring;
    const uint32_t slot_bytes = wl_slot_bytes(nt, GX, masked);
    unsigned char* ring = smem_raw + NO * ops_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + S * slot_bytes);
    uint64_t* full = bars;            // [S]  unit landed (bytes)
    uint64_t* empty = bars + 4;       // [S]  slot read by the split warps
    uint64_t* opfull = bars + 8;      // [2]  operand buffer written by the split warps
    uint64_t* opempty = bars + 10;    // [2]  operand buffer read by the MMAs (commit)
    uint64_t* accfull = bars + 12;    //      all MMAs done (commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
    const uint32_t smem_base = smem_addr(smem_raw);
    const uint32_t ring_base = smem_base + NO * ops_bytes;

    WaitCtx wc = a.wait;
    wc.kernel = 5;
    wc.problem = b;
    wc.warp = blockIdx.x;
    wc.band = GX ? 1 : 2;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(smem_addr(full + i), 1);
            mbar_init(smem_addr(empty + i), kWlSplitWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(opfull + i), kWlSplitWarps);
            mbar_init(smem_addr(opempty + i), 1);
        }
        mbar_init(smem_addr(accfull), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), static_cast<uint32_t>(a.tmem_cols));
        tmem_relinquish();
    }
    for (int e = threadIdx.x; e < NO * 16 * kKT; e += blockDim.x) {  // the ones rows of B'
        const int o = e / (16 * kKT), r = (e / kKT) % 16, k = e % kKT;
        *reinterpret_cast<float*>(smem_raw + o * ops_bytes + 2 * a_op + op_off(2 * nt + r, k)) = 1.f;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == kWlSplitWarps) {
        // ================= copies
        int issued = 0;
        for (int k = 0; k < n_units; ++k) {
            const int sl = k % S;
            if (k >= S) ok = warp_wait(smem_addr(empty + sl), static_cast<uint32_t>((k / S - 1) & 1), wc, ok);
            if (!ok) break;
            const uint32_t dst = ring_base + sl * slot_bytes;
            const uint32_t bar = smem_addr(full + sl);
            const int bchunk = GX ? k - 1 : k;
            const int t0 = 32 * k;
            const int rows = GX ? max(0, min(32, P.n_diag - t0)) : kYRows;
            const int ns = GX ? min(4, P.n_stripes - r0 / 32) : 1;
            uint32_t bytes = static_cast<uint32_t>(rows * ns) * 128u * (masked ? 2u : 1u);
            if (bchunk >= 0) bytes += static_cast<uint32_t>(nf) * kBPitch;
            if (lane == 0) mbar_expect_tx(bar, bytes);
            __syncwarp();
            if (GX) {
                // Lanes 0 .. ns-1 copy the G blocks of the tile's stripes,
                // lanes ns .. 2ns-1 the mask blocks.
                if (rows > 0 && lane < ns * (masked ? 2 : 1)) {
                    const bool is_mask = lane >= ns;
                    const int st = is_mask ? lane - ns : lane;
                    const float* src = (is_mask ? a.Mw : a.Ew) + wl_row(P, b, r0 / 32 + st, t0);
                    const uint32_t d = dst + (is_mask ? a_ring : 0u) + static_cast<uint32_t>(st) * 4096u;
                    bulk_g2s(d, src, static_cast<uint32_t>(rows) * 128u, bar);
                }
            } else {
                // Rows t in [r0, r0 + 159) of stripe k: row (b * n_stripes + k) * n_diag + t of the 2-D view.
                const int y = (b * P.n_stripes + k) * P.n_diag + r0;
                if (lane == 1) tensor2d_g2s(dst, &a.tm_e, 0, y, bar);
                if (lane == 2 && masked) tensor2d_g2s(dst + a_ring, &a.tm_m, 0, y, bar);
            }
            if (bchunk >= 0 && lane == 3)
                bulk_g2s(dst + a_ring_all, Bsrc + (static_cast<size_t>(bchunk) * dim + f0) * (kBPitch / 4),
                         static_cast<uint32_t>(nf) * kBPitch, bar);
            __syncwarp();
            issued = k + 1;
        }
        // In-flight copies land before the CTA can exit: the split warps wait
        // for every unit on the normal path; after a failure, wait here.
        if (!ok && lane == 0)
            for (int k = max(0, issued - S); k < issued; ++k)
                mbar_wait_fast(smem_addr(full + k % S), static_cast<uint32_t>((k / S) & 1), wc);
    } else if (warp == kWlSplitWarps + 1) {
        // ================= MMAs (one thread)
        const int n1 = 2 * nt + 16;
        const uint32_t idesc1a = idesc_tf32(kTileM, n1 > 256 ? 256 : n1);
        const uint32_t idesc1b = idesc_tf32(kTileM, n1 > 256 ? n1 - 256 : 16);
        const uint32_t idesc2 = idesc_tf32(kTileM, nt + 16);
        if (lane == 0) {
            for (int c = 0; c < n_chunks; ++c) {
                const int o = c % NO;
                if (ok) ok = mbar_wait_fast(smem_addr(opfull + o), static_cast<uint32_t>((c / NO) & 1), wc);
                if (!ok) break;
                tc_fence_after();
                const uint32_t aH = smem_base + o * ops_bytes;
                const uint32_t aL = aH + a_op;
                const uint32_t bP = aL + a_op;
                const uint32_t bH = bP + static_cast<uint32_t>(nt / 8) * kSBO;
#pragma unroll
                for (int ks = 0; ks < kKT / 8; ++ks) {
                    const uint32_t off = static_cast<uint32_t>(ks) * 2 * kLBO;
                    const uint32_t acc = (c > 0 || ks > 0) ? 1u : 0u;
                    mma_tf32(tmem, smem_desc(aH + off), smem_desc(bP + off), idesc1a, acc);
                    if (n1 > 256)
                        mma_tf32(tmem + 256u, smem_desc(aH + off), smem_desc(bP + 32u * kSBO + off), idesc1b, acc);
                    mma_tf32(tmem + static_cast<uint32_t>(nt), smem_desc(aL + off), smem_desc(bH + off), idesc2, 1u);
                }
                mma_commit(smem_addr(opempty + o));
            }
            if (ok) mma_commit(smem_addr(accfull));
        }
        __syncwarp();
    } else {
        // ================= split warps: de-skew, split, store the operands
        // (kWlSplitWarps = 16 warps, 512 threads; indices below assume it).
        float4 ahi[2], alo[2];  // grad_x: 2 vectors; grad_y: 8 scalars in the same registers
        float4 bhi[2], blo[2];  // B: 16-byte units threadIdx.x + 512 i (nt * 8 of them)
        // B unit u: row f = 8 * ((u >> 3) % (nt / 8)) + (u & 7), column unit
        // (u >> 3) / (nt / 8): 8 consecutive lanes, 8 rows of one column unit.
        uint32_t b_src[2], b_dlo[2], b_dhi[2];
        uint32_t b_live = 0, b_has = 0;  // bit i: unit i exists; bit i: its row is a feature row
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = threadIdx.x + 512 * i;
            const int grp = u >> 3;
            const int f = 8 * (grp % (nt / 8)) + (u & 7), ku = grp / (nt / 8);
            b_src[i] = static_cast<uint32_t>(f) * kBPitch + static_cast<uint32_t>(ku) * 16u;
            b_dlo[i] = 2 * a_op + op_off(f, 4 * ku);
            b_dhi[i] = 2 * a_op + op_off(nt + f, 4 * ku);
            if (u < nt * 8) b_live |= 1u << i;
            if (u < nt * 8 && f < nf) b_has |= 1u << i;
        }
        // grad_x: row q = r0 + 32 (warp % 4) + lane, column units ku_i = warp / 4 + 4 i;
        // element (i, d) sits at byte gx_off[i][d] of slot c (bit i*4+d of
        // gx_sel clear) or c + 1 (set).
        const int gx_rg = warp & 3;
        const bool gx_row_ok = GX && r0 + 32 * gx_rg + lane < N;
        const uint32_t gx_dst = op_off(32 * gx_rg + lane, 0);
        uint32_t gx_off[2][4];
        uint32_t gx_sel = 0;
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int rel = lane + 4 * ((warp >> 2) + 4 * i) + d;  // t - 32c, 0 .. 62
                gx_off[i][d] = static_cast<uint32_t>(gx_rg) * 4096u + static_cast<uint32_t>(rel & 31) * 128u +
                               static_cast<uint32_t>(lane) * 4u;
                if (rel >= 32) gx_sel |= 1u << (4 * i + d);
            }
        // grad_y: element e (0 .. 7): row jl = 8 warp + (lane & 7), column ql = 4 e + lane / 8,
        // at byte gy_off[e] of the slot (128-byte swizzle).
        const int gy_i8 = lane & 7, gy_d = lane >> 3;
        const bool gy_row_ok = !GX && r0 + 8 * warp + gy_i8 < M;
        uint32_t gy_off[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int r = 4 * e + gy_d + 8 * warp + gy_i8;  // slot row (t - r0)
            gy_off[e] = static_cast<uint32_t>(r) * 128u +
                        (static_cast<uint32_t>(e ^ ((4 * e + gy_d + gy_i8) & 7)) << 4) + static_cast<uint32_t>(gy_d) * 4u;
        }
        // Every cell of the tile is in the table except in the last chunk (or
        // a last, partial row tile): elsewhere no bound checks are needed.
        const bool rows_full = r0 + kTileM <= rows_out;
        const uint32_t ring_s = smem_addr(ring);

        int s_c = 0;       // ring slot of unit c (and of c + 1: s_c1)
        uint32_t p_c = 0;  // phase parity of unit c: (c / S) & 1
        int o = 0;         // operand buffer of chunk c: c % NO
        uint32_t po = 0;   // (c / NO) & 1
        for (int c = 0; c < n_chunks && ok; ++c) {
            const int s_c1 = s_c + 1 == S ? 0 : s_c + 1;
            const uint32_t p_c1 = s_c1 == 0 ? p_c ^ 1u : p_c;
            // Unit c (grad_y) or c + 1 (grad_x; unit c was waited for by chunk c - 1).
            if (GX && c == 0) ok = warp_wait(smem_addr(full + 0), 0u, wc, ok);
            ok = warp_wait(smem_addr(full + (GX ? s_c1 : s_c)), GX ? p_c1 : p_c, wc, ok);
            if (!ok) break;
            const bool exact = rows_full && 32 * (c + 1) <= kt && !masked;  // warp-uniform
            if (GX) {
                const uint32_t base0 = ring_s + static_cast<uint32_t>(s_c) * slot_bytes;
                const uint32_t base1 = ring_s + static_cast<uint32_t>(s_c1) * slot_bytes;
                const int j_lim = M - 32 * c;  // columns j - 32c below this are in the table
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int ku = (warp >> 2) + 4 * i;
                    float v[4];
#pragma unroll
                    for (int d = 0; d < 4; ++d) {
                        const uint32_t a = ((gx_sel >> (4 * i + d)) & 1u ? base1 : base0) + gx_off[i][d];
                        const float x = ld_shared_f32(a);
                        if (exact) {
                            v[d] = x;
                        } else {
                            bool okc = gx_row_ok && 4 * ku + d < j_lim;
                            if (masked) okc = okc && ld_shared_f32(a + a_ring) > 0.f;
                            v[d] = okc ? x : 0.f;
                        }
                    }
                    ahi[i] = make_float4(split_hi(v[0]), split_hi(v[1]), split_hi(v[2]), split_hi(v[3]));
                    alo[i] = make_float4(v[0] - ahi[i].x, v[1] - ahi[i].y, v[2] - ahi[i].z, v[3] - ahi[i].w);
                }
            } else {
                const uint32_t base = ring_s + static_cast<uint32_t>(s_c) * slot_bytes;
                const int q_lim = N - 32 * c;
                float* hs = reinterpret_cast<float*>(ahi);
                float* ls = reinterpret_cast<float*>(alo);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t a = base + gy_off[e];
                    float x = ld_shared_f32(a);
                    if (!exact) {
                        bool okc = gy_row_ok && 4 * e + gy_d < q_lim;
                        if (masked) okc = okc && ld_shared_f32(a + a_ring) > 0.f;
                        x = okc ? x : 0.f;
                    }
                    hs[e] = split_hi(x);
                    ls[e] = x - hs[e];
                }
            }
            {
                const unsigned char* bslot = ring + static_cast<uint32_t>(GX ? s_c1 : s_c) * slot_bytes + a_ring_all;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (b_has & (1u << i)) v = *reinterpret_cast<const float4*>(bslot + b_src[i]);
                    bhi[i] = make_float4(split_hi(v.x), split_hi(v.y), split_hi(v.z), split_hi(v.w));
                    blo[i] = make_float4(v.x - bhi[i].x, v.y - bhi[i].y, v.z - bhi[i].z, v.w - bhi[i].w);
                }
            }
            // Release the slot this chunk was the last reader of (grad_x: unit
            // c, and unit c + 1 after the last chunk; grad_y: unit c).
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_addr(empty + s_c));
                if (GX && c + 1 == n_chunks) mbar_arrive(smem_addr(empty + s_c1));
            }
            // Operand buffer o, free once the MMAs of chunk c - NO are done.
            if (c >= NO) ok = warp_wait(smem_addr(opempty + o), po ^ 1u, wc, ok);
            if (!ok) break;
            unsigned char* Ob = smem_raw + o * ops_bytes;
            if (GX) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t off = gx_dst + static_cast<uint32_t>((warp >> 2) + 4 * i) * kLBO;
                    *reinterpret_cast<float4*>(Ob + off) = ahi[i];
                    *reinterpret_cast<float4*>(Ob + a_op + off) = alo[i];
                }
            } else {
                const float* hs = reinterpret_cast<const float*>(ahi);
                const float* ls = reinterpret_cast<const float*>(alo);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t off = static_cast<uint32_t>(warp) * kSBO + static_cast<uint32_t>(e) * kLBO +
                                         static_cast<uint32_t>(gy_i8) * 16u + static_cast<uint32_t>(gy_d) * 4u;
                    *reinterpret_cast<float*>(Ob + off) = hs[e];
                    *reinterpret_cast<float*>(Ob + a_op + off) = ls[e];
                }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (b_live & (1u << i)) {
                    *reinterpret_cast<float4*>(Ob + b_dlo[i]) = blo[i];
                    *reinterpret_cast<float4*>(Ob + b_dhi[i]) = bhi[i];
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(opfull + o));
            s_c = s_c1;
            p_c = p_c1;
            if (++o == NO) {
                o = 0;
                po ^= 1u;
            }
        }
        ok = warp_wait(smem_addr(accfull), 0u, wc, ok);
        tc_fence_after();
    }
    const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;

    if (all_ok && warp < kWlSplitWarps) {
        const int quarter = warp & 3;
        const int half = warp >> 2;  // column group (0 .. 3)
        const int r = r0 + quarter * 32 + lane;
        const size_t rstride = static_cast<size_t>(rows_out) * dim;
        const float* own = GX ? a.x.at(b, rstride) : a.y.at(b, rstride);
        float* g = GX ? a.gx.at(b, rstride) : a.gy.at(b, rstride);
        const uint32_t tw = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float v[16], w[16];
        tmem_ld16(tw + static_cast<uint32_t>(2 * nt), v);
        const float sum = v[0];
        const size_t row_off = static_cast<size_t>(r) * dim + f0;
        const bool vec = ((dim & 3) == 0) && ((f0 & 3) == 0) &&
                         ((reinterpret_cast<uintptr_t>(own) | reinterpret_cast<uintptr_t>(g)) & 15u) == 0;
        for (int c16 = half; c16 * 16 < fb; c16 += kWlSplitWarps / 4) {  // warp-uniform
            tmem_ld16(tw + static_cast<uint32_t>(c16 * 16), v);
            tmem_ld16(tw + static_cast<uint32_t>(nt + c16 * 16), w);
            if (r < rows_out) {
                const int fl = c16 * 16;
                if (vec && fl + 16 <= fb && f0 + fl + 16 <= dim) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 o = __ldg(reinterpret_cast<const float4*>(own + row_off + fl) + u);
                        float4 y4;
                        y4.x = 2.f * (o.x * sum - (v[4 * u + 0] + w[4 * u + 0]));
                        y4.y = 2.f * (o.y * sum - (v[4 * u + 1] + w[4 * u + 1]));
                        y4.z = 2.f * (o.z * sum - (v[4 * u + 2] + w[4 * u + 2]));
                        y4.w = 2.f * (o.w * sum - (v[4 * u + 3] + w[4 * u + 3]));
                        reinterpret_cast<float4*>(g + row_off + fl)[u] = y4;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int f = fl + i;
                        if (f < fb && f0 + f < dim)
                            g[row_off + f] = 2.f * (__ldg(own + row_off + f) * sum - (v[i] + w[i]));
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(a.tmem_cols));
}

constexpr int kWlThreads = 32 * (kWlSplitWarps + 2);  // split warps, the copy warp, the MMA warp

__global__ void __launch_bounds__(kWlThreads, 1) grad_wl_kernel(const __grid_constant__ GradTcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    pdl_trigger();
    pdl_wait();  // E and the transposed operands of the previous kernels
    if (static_cast<int>(blockIdx.x) < a.tiles_x * a.n_fblk) grad_wl_tile<true>(a, smem_raw);
    else grad_wl_tile<false>(a, smem_raw);
}

static size_t grad_wl_smem(int nt, bool gx, bool masked, int stages, int ops) {
    return static_cast<size_t>(ops) * wl_ops_bytes(nt) + static_cast<size_t>(stages) * wl_slot_bytes(nt, gx, masked) +
           256 + 1024;
}

bool grad_wl_supported(const WavePlan& P) { return P.K == 1; }

// Feature blocks of at most 128 features, of equal size.  Pipeline depths: the
// deepest that fits, preferring two operand buffers, then ring slots (grad_x
// needs 3: two resident units and one in flight; grad_y 2).
void grad_wl_geometry(int dim, bool masked, GradTcArgs* g) {
    const int nb = (dim + kWlMaxNt - 1) / kWlMaxNt;
    g->n_fblk = nb;
    g->fb = (dim + nb - 1) / nb;
    g->nt = (g->fb + 15) / 16 * 16;
    int tc = 32;
    while (tc < 2 * g->nt + 16) tc *= 2;
    g->tmem_cols = tc;
    const size_t cap = 227u * 1024u;
    for (int gx = 0; gx < 2; ++gx) {
        const int smin = gx ? 3 : 2;
        int best_s = smin, best_o = 1;
        bool found = false;
        for (int o = 2; o >= 1 && !found; --o)
            for (int s = 4; s >= smin; --s)
                if (grad_wl_smem(g->nt, gx, masked, s, o) <= cap) {
                    best_s = s;
                    best_o = o;
                    found = true;
                    break;
                }
        if (gx) {
            g->stages_x = best_s;
            g->ops_x = best_o;
        } else {
            g->stages_y = best_s;
            g->ops_y = best_o;
        }
    }
}

// 2-D view of a wavefront-layout table for the tensor copies: rows of 32
// floats (128 bytes), boxes of 159 rows, 128-byte swizzle.
static cudaError_t encode_rows(CUtensorMap* map, const float* base, const WavePlan& P) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    if (!encode) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {32, static_cast<cuuint64_t>(P.B) * P.n_stripes * P.n_diag};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kYRows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_grad_wl(const GradTcArgs& args_in, cudaStream_t stream) {
    GradTcArgs args = args_in;
    const WavePlan& P = args.P;
    if (P.K != 1 || args.nt < 16 || args.nt > kWlMaxNt || args.nt % 16) return cudaErrorInvalidValue;
    const bool masked = args.Mw != nullptr;
    if (((reinterpret_cast<uintptr_t>(args.Ew) | reinterpret_cast<uintptr_t>(args.Mw) |
          reinterpret_cast<uintptr_t>(args.xTc) | reinterpret_cast<uintptr_t>(args.yTc)) & 15u) != 0)
        return cudaErrorMisalignedAddress;
    const size_t smem =
        std::max(args.tiles_x ? grad_wl_smem(args.nt, true, masked, args.stages_x, args.ops_x) : 0,
                 args.tiles_y ? grad_wl_smem(args.nt, false, masked, args.stages_y, args.ops_y) : 0);
    if (smem > 227u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    if (args.tiles_y) {
        e = encode_rows(&args.tm_e, args.Ew, P);
        if (e == cudaSuccess && masked) e = encode_rows(&args.tm_m, args.Mw, P);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((args.tiles_x + args.tiles_y) * args.n_fblk, P.B);
    e = cudaFuncSetAttribute(grad_wl_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_pdl(false, grad_wl_kernel, grid, dim3(kWlThreads), smem, stream, args);
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
// ST = 1 or 2 operand stages.  One stage serialises copy, split and MMAs of a
// chunk but halves the shared memory, so that two CTAs share an SM and one's
// epilogue stores overlap the other's chunks.
// RM: the cost row-major (B, N, M) instead (distances.sqeuclidean): the tile is
// staged in shared memory rows of 129 floats and stored by coalesced rows.
template <int K, int ST, bool RM = false>
__global__ void __launch_bounds__(kThreads, 1) cost_tc_kernel(const SeqIn x, const SeqIn y, float* __restrict__ Dw,
                                                              const WavePlan P, int dim,
                                                              const WaitCtx wait) {
    static_assert(!RM || K == 1, "row-major output: one tile layout");
    constexpr int kCostStages = ST;
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
    // Barriers and norms follow both the operand stages and the epilogue's
    // staging area, which reuses the stages' space.
    constexpr uint32_t kStageArea = static_cast<uint32_t>(NSL * TL * SR * sizeof(float));
    // ST = 1: the operand stage plus separate raw buffers for x and y (the
    // next chunk's copies land there while this chunk's MMAs run).
    const uint32_t ops_area = ST == 1 ? 6 * op_bytes : kCostStages * stage_bytes;
    unsigned char* ctrl = smem_raw + (ops_area > kStageArea ? ops_area : kStageArea);
    float* npart = reinterpret_cast<float*>(ctrl + 128 + 4 * kTileM * sizeof(float));  // ST = 1: [2][128][8]
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ctrl);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 64);
    float* xn = reinterpret_cast<float*>(ctrl + 128);  // [2][128] partial, then [128]
    float* yn = xn + 2 * kTileM;                      // [2][128] partial, then [128]
    const uint32_t smem_base = smem_addr(smem_raw);
    const float* xb = x.at(b, static_cast<size_t>(N) * dim);
    const float* yb = y.at(b, static_cast<size_t>(M) * dim);
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
    // ST = 1 unit mapping (rm_row / rm_col): 8 consecutive lanes copy 8 rows of
    // one 16-byte column (128 contiguous bytes of shared memory), and each row
    // is read as 64 contiguous bytes of global memory.  Row norms accumulate
    // per unit and are summed in a fixed order at the end.
    float nx1[UPT], ny1[UPT];
#pragma unroll
    for (int i = 0; i < UPT; ++i) nx1[i] = ny1[i] = 0.f;
    const uint32_t rawA = smem_base + 4 * op_bytes, rawB = rawA + op_bytes;
    auto issue1 = [&](int c) {
        const int f0 = c * kKT;
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
            const int row = rm_row(warp, lane, i), k = rm_col(warp, lane, i);
            const int f = f0 + k;
            const bool fx = q0 + row < N && f < dim;
            const bool fy = j0 + row < M && f < dim;
            const uint32_t off = op_off(row, k);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(rawA + off),
                         "l"(fx ? xb + static_cast<size_t>(q0 + row) * dim + f : xb), "r"(fx ? 16u : 0u)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(rawB + off),
                         "l"(fy ? yb + static_cast<size_t>(j0 + row) * dim + f : yb), "r"(fy ? 16u : 0u)
                         : "memory");
        }
    };
    auto split1 = [&]() {
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
            const uint32_t off = op_off(rm_row(warp, lane, i), rm_col(warp, lane, i));
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                const float4 v = *reinterpret_cast<const float4*>(smem_raw + (4 + o) * op_bytes + off);
                float4 h, l;
                h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
                h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
                h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
                h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
                l.x = v.x - h.x;
                l.y = v.y - h.y;
                l.z = v.z - h.z;
                l.w = v.w - h.w;
                unsigned char* hi = smem_raw + 2 * o * op_bytes;
                *reinterpret_cast<float4*>(hi + off) = h;
                *reinterpret_cast<float4*>(hi + op_bytes + off) = l;
                float& acc = o == 0 ? nx1[i] : ny1[i];
                acc = fmaf(v.x, v.x, acc);
                acc = fmaf(v.y, v.y, acc);
                acc = fmaf(v.z, v.z, acc);
                acc = fmaf(v.w, v.w, acc);
            }
        }
    };
    if (ST == 1) {
        issue1(0);
        asm volatile("cp.async.commit_group;" ::: "memory");
        for (int c = 0; c < n_chunks; ++c) {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            // The operand stage is free once the MMAs of chunk c-1 are done.
            if (c >= 1 && ok) ok = mbar_wait(smem_addr(mbar), static_cast<uint32_t>((c - 1) & 1), wc);
            split1();
            // Each thread refills only the raw units it has just read.
            if (c + 1 < n_chunks) {
                issue1(c + 1);
                asm volatile("cp.async.commit_group;" ::: "memory");
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (threadIdx.x == 0 && ok) {
                const uint32_t aH = smem_base, aL = aH + op_bytes, bH = aL + op_bytes, bL = bH + op_bytes;
#pragma unroll
                for (int ks = 0; ks < kKT / 8; ++ks) {
                    const uint32_t o = static_cast<uint32_t>(ks) * 2 * kLBO;
                    const uint32_t acc0 = (c > 0 || ks > 0) ? 1u : 0u;
                    mma_tf32(tmem, smem_desc(aH + o), smem_desc(bH + o), idesc, acc0);
                    mma_tf32(tmem, smem_desc(aH + o), smem_desc(bL + o), idesc, 1u);
                    mma_tf32(tmem, smem_desc(aL + o), smem_desc(bH + o), idesc, 1u);
                }
                mma_commit(smem_addr(mbar));
            }
        }
    }
    if (ST == 2) {
        issue(0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int c = 0; ST == 2 && c < n_chunks; ++c) {
        const int st = c % kCostStages;
        if (ST == 2) {
            // Refill the other stage with chunk c+1 once the MMAs of chunk c-1 are done.
            if (c + 1 < n_chunks) {
                if (c >= 1 && ok) ok = mbar_wait(smem_addr(mbar + (c - 1) % kCostStages), static_cast<uint32_t>(((c - 1) / kCostStages) & 1), wc);
                issue(c + 1);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            // The single stage is free once the MMAs of chunk c-1 are done.
            if (c >= 1 && ok) ok = mbar_wait(smem_addr(mbar), static_cast<uint32_t>((c - 1) & 1), wc);
            issue(c);
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
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
    if (ST == 1) {
        // Squared norms: the 8 column units of row r, in column order.
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
            const int row = rm_row(warp, lane, i), ug = rm_col(warp, lane, i) / 4;
            npart[row * 8 + ug] = nx1[i];
            npart[kTileM * 8 + row * 8 + ug] = ny1[i];
        }
    } else {
        // Squared norms: threads r and r + 128 hold the two halves of row r.
        xn[(threadIdx.x >> 7) * kTileM + urow] = xs2;
        yn[(threadIdx.x >> 7) * kTileM + urow] = ys2;
    }
    if (n_chunks > 0 && ok) {
        const int cl = n_chunks - 1;
        ok = mbar_wait(smem_addr(mbar + cl % kCostStages), static_cast<uint32_t>((cl / kCostStages) & 1), wc);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    tc_fence_after();
    const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
    if (threadIdx.x < kTileM) {
        if (ST == 1) {
            float ax = 0.f, ay = 0.f;
#pragma unroll
            for (int ug = 0; ug < 8; ++ug) {
                ax += npart[threadIdx.x * 8 + ug];
                ay += npart[kTileM * 8 + threadIdx.x * 8 + ug];
            }
            xn[threadIdx.x] = ax;
            yn[threadIdx.x] = ay;
        } else {
            xn[threadIdx.x] = xn[threadIdx.x] + xn[kTileM + threadIdx.x];
            yn[threadIdx.x] = yn[threadIdx.x] + yn[kTileM + threadIdx.x];
        }
    }
    __syncthreads();

    if constexpr (RM) {
        // ---- row-major epilogue: thread (row r, column half) stages its 64
        // cells at stg[r][c] (pitch 129: the lanes' rows fall in distinct
        // banks), then warp w stores tile rows w, w + 8, ... as 128-float rows.
        constexpr int kPitch = kTileM + 1;
        float* stg = reinterpret_cast<float*>(smem_raw);
        if (all_ok) {
            const int quarter = warp & 3, half = warp >> 2;
            const int r = quarter * 32 + lane;
            const float xr = xn[r];
            const uint32_t tw = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
            float v[16];
            for (int c16 = half * 4; c16 < half * 4 + 4; ++c16) {
                tmem_ld16(tw + static_cast<uint32_t>(c16 * 16), v);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = c16 * 16 + i;
                    stg[r * kPitch + c] = fmaxf((xr + yn[c]) - 2.f * v[i], 0.f);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 0) tmem_dealloc(tmem, 128u);
        if (all_ok) {
            for (int rr = warp; rr < kTileM; rr += kThreads / 32) {
                const int q = q0 + rr;
                if (q >= N) break;
                float* drow = Dw + (static_cast<size_t>(b) * N + q) * M + j0;
#pragma unroll
                for (int k = 0; k < kTileM / 32; ++k) {
                    const int c = k * 32 + lane;
                    if (j0 + c < M) drow[c] = stg[rr * kPitch + c];
                }
            }
        }
        return;
    }
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
        // Anti-diagonal rows of the staged slices: warp w stores rows tl = w / NSL
        // + (8 / NSL) i of slice w % NSL; lane p (and p + 32, ... for K > 1) is
        // position p of the row.  Per slice: the rows' first and last columns
        // are known in closed form, so the loop body is a load, two compares
        // and a store.
        const float* stg = reinterpret_cast<const float*>(smem_raw);
        const int sl = warp % NSL;
        const int q_base = q0 + sl * SR;  // first row of the slice
        if (q_base < N) {
            const int s = q_base / SR;
            const size_t row0 = (static_cast<size_t>(b) * P.n_stripes + s) * P.n_diag;
#pragma unroll 8
            for (int tl = warp / NSL; tl < TL; tl += kThreads / 32 / NSL) {
#pragma unroll
                for (int kk = 0; kk < K; ++kk) {
                    const int pp = kk * 32 + lane;
                    const int ql = (pp % 32) * K + pp / 32;
                    const int jl = tl - ql;  // column within the tile
                    const int j = j0 + jl;
                    if (jl >= 0 && jl < kTileM && j < M && q_base + ql < N)
                        Dw[(row0 + ql + j) * SR + pp] = stg[(sl * TL + tl) * SR + pp];
                }
            }
        }
    }
}

static size_t cost_tc_smem_bytes(int K, int stages) {
    const size_t op = (kTileM / 8) * kSBO;
    const size_t ops = stages == 1 ? 6 * op : static_cast<size_t>(stages) * 4 * op;
    const size_t stage = static_cast<size_t>(kTileM / (32 * K)) * (32 * K + kTileM - 1) * (32 * K) * sizeof(float);
    return (ops > stage ? ops : stage) + 128 + 4 * kTileM * sizeof(float) + 2 * kTileM * 8 * sizeof(float);
}

bool cost_tc_supported(const SeqIn& x, const SeqIn& y, int dim) {
    return dim >= 16 && dim % 4 == 0 && x.aligned16() && y.aligned16();
}

template <int K, int ST, bool RM = false>
static cudaError_t cost_tc_go(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim,
                              const WaitCtx& wait, cudaStream_t stream) {
    const dim3 grid((P.M + kTileM - 1) / kTileM, (P.N + kTileM - 1) / kTileM, P.B);
    size_t smem = cost_tc_smem_bytes(K, ST);
    if (RM) smem = std::max(smem, static_cast<size_t>(kTileM) * (kTileM + 1) * sizeof(float) + 128 +
                                      4 * kTileM * sizeof(float) + 2 * kTileM * 8 * sizeof(float));
    cudaError_t e = cudaFuncSetAttribute(cost_tc_kernel<K, ST, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cost_tc_kernel<K, ST, RM><<<grid, kThreads, smem, stream>>>(x, y, Dw, P, dim, wait);
    return cudaGetLastError();
}

cudaError_t launch_cost_tc_rm(const float* x, const float* y, float* D, int B, int N, int M, int dim,
                              const WaitCtx& wait, cudaStream_t stream) {
    WavePlan P{};
    P.B = B;
    P.N = N;
    P.M = M;
    P.K = 1;
    return cost_tc_go<1, 1, true>(one_seq(x), one_seq(y), D, P, dim, wait, stream);
}

cudaError_t launch_cost_tc(const SeqIn& x, const SeqIn& y, float* Dw, const WavePlan& P, int dim, const WaitCtx& wait,
                           cudaStream_t stream) {
    // One stage where that lets two CTAs share an SM (K <= 2: the shared memory
    // is then the epilogue's staging area, under 100 KB).  Measured on B200
    // (K = 1): C2 unfused cost 50 -> 38 us, 64 x 1024 x 1024 x 128 x 3 problems
    // 1.27 -> 0.95 ms.
    switch (P.K) {
        case 1: return cost_tc_go<1, 1>(x, y, Dw, P, dim, wait, stream);
        case 2: return cost_tc_go<2, 1>(x, y, Dw, P, dim, wait, stream);
        case 4: return cost_tc_go<4, 2>(x, y, Dw, P, dim, wait, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sdtw
