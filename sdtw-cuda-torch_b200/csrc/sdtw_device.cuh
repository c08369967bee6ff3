// sdtw_device.cuh -- device helpers shared by the Soft-DTW kernels (sm_100a).
//
// * MUFU wrappers (ex2/lg2/rcp .approx.ftz) written as inline PTX.
// * Cluster shared-memory (DSMEM) and global-memory accessors with explicit
//   memory-model qualifiers, used by the warp-chain ring handoff.
// * Bounded waits: every spin has a wall-clock limit (%globaltimer); when it
//   runs out the waiter records an error code in the status word and the kernel
//   unwinds instead of hanging.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define SDTW_FULL_MASK 0xffffffffu

namespace sdtw {

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ float pos_inf() { return __int_as_float(0x7f800000); }

// ---------------------------------------------------------------- MUFU ops
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2f(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcpf(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) { return fmaxf(fmaxf(a, b), c); }

// ---------------------------------------------------------------- cluster / smem
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster
// (valid in the shared::cluster window, including rank == own rank).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 64-bit stores/loads are single-copy atomic, so a (value, tag) pair packed in
// one u64 is seen whole or not at all: no separate flag or fence is needed.
__device__ __forceinline__ void st_cluster_u64(uint32_t cluster_addr, uint64_t v) {
    asm volatile("st.relaxed.cluster.shared::cluster.u64 [%0], %1;" ::"r"(cluster_addr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_cluster_u64(uint32_t own_saddr) {
    uint64_t v;
    asm volatile("ld.relaxed.cluster.shared::cta.u64 %0, [%1];" : "=l"(v) : "r"(own_saddr) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.release.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_cluster_u32(uint32_t own_saddr) {
    uint32_t v;
    asm volatile("ld.acquire.cluster.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(own_saddr) : "memory");
    return v;
}
__device__ __forceinline__ void st_gpu_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_gpu_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint64_t pack_tagged(float v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | static_cast<uint64_t>(__float_as_uint(v));
}
__device__ __forceinline__ uint32_t tag_of(uint64_t e) { return static_cast<uint32_t>(e >> 32); }
__device__ __forceinline__ float val_of(uint64_t e) { return __uint_as_float(static_cast<uint32_t>(e)); }

// ---------------------------------------------------------------- bounded waits
// Status word: 0 = ok; otherwise the first error code recorded by any kernel.
// It lives in mapped pinned host memory so the host can read it without a
// device synchronisation.
enum : int {
    kStatusOk = 0,
    kStatusTimeout = 3,
};

struct WaitCtx {
    volatile int* status;   // mapped pinned host word (may be null)
    uint64_t timeout_ns;    // wall-clock limit for one wait
};

__device__ __forceinline__ void record_error(const WaitCtx& w, int code) {
    if (w.status) *w.status = code;  // plain volatile store; racing writers store the same code
}
__device__ __forceinline__ bool aborted(const WaitCtx& w) { return w.status && *w.status != 0; }

// Wait until the u64 at own-CTA smem address `saddr` carries `tag`; return its
// value in `out`.  Returns false (after recording kStatusTimeout) when the
// limit runs out or another waiter has already recorded an error.
static __device__ __noinline__ bool wait_smem_tag_slow(uint32_t saddr, uint32_t tag, float& out, const WaitCtx& w) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        uint64_t e = ld_cluster_u64(saddr);
        if (tag_of(e) == tag) {
            out = val_of(e);
            return true;
        }
        if ((it & 31u) == 0u) {
            if (aborted(w)) return false;
            if (globaltimer_ns() - t0 > w.timeout_ns) {
                record_error(w, kStatusTimeout);
                return false;
            }
            __nanosleep(64);
        }
    }
}
__device__ __forceinline__ bool wait_smem_tag(uint32_t saddr, uint32_t tag, float& out, const WaitCtx& w) {
    uint64_t e = ld_cluster_u64(saddr);
    if (tag_of(e) == tag) {
        out = val_of(e);
        return true;
    }
    return wait_smem_tag_slow(saddr, tag, out, w);
}

static __device__ __noinline__ bool wait_gmem_tag_slow(const uint64_t* p, uint32_t tag, float& out, const WaitCtx& w) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        uint64_t e = ld_gpu_u64(p);
        if (tag_of(e) == tag) {
            out = val_of(e);
            return true;
        }
        if ((it & 31u) == 0u) {
            if (aborted(w)) return false;
            if (globaltimer_ns() - t0 > w.timeout_ns) {
                record_error(w, kStatusTimeout);
                return false;
            }
            __nanosleep(64);
        }
    }
}
__device__ __forceinline__ bool wait_gmem_tag(const uint64_t* p, uint32_t tag, float& out, const WaitCtx& w) {
    uint64_t e = ld_gpu_u64(p);
    if (tag_of(e) == tag) {
        out = val_of(e);
        return true;
    }
    return wait_gmem_tag_slow(p, tag, out, w);
}

// Wait until the u32 counter at own-CTA smem address `saddr` is >= `need`.
static __device__ __noinline__ bool wait_counter_ge(uint32_t saddr, uint32_t need, uint32_t& seen, const WaitCtx& w) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        seen = ld_acquire_cluster_u32(saddr);
        if (static_cast<int32_t>(seen - need) >= 0) return true;
        if ((it & 31u) == 0u) {
            if (aborted(w)) return false;
            if (globaltimer_ns() - t0 > w.timeout_ns) {
                record_error(w, kStatusTimeout);
                return false;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace sdtw
