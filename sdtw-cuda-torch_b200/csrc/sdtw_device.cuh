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
// Predicated forms (no branch around the store).
__device__ __forceinline__ void st_cluster_u64_if(bool p, uint32_t cluster_addr, uint64_t v) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.relaxed.cluster.shared::cluster.u64 [%1], %2;\n\t}" ::"r"(
            static_cast<int>(p)),
        "r"(cluster_addr), "l"(v)
        : "memory");
}
// Progress reports of the ring flow control.  A release store would wait for
// every earlier store of the thread (the score rows written to global memory)
// to be performed: measured on B200 that cost the consumer warps about 150
// cycles per step.  The report only needs to follow the reads of the ring
// slots it releases; those values were consumed (their tags voted on with
// __any_sync) before the report is issued, so the loads have completed.  A
// slot overwritten early could only show a newer tag, which the consumer
// rejects (it would time out, never read a wrong value).
__device__ __forceinline__ void st_relaxed_cluster_u32_if(bool p, uint32_t cluster_addr, uint32_t v) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.relaxed.cluster.shared::cluster.u32 [%1], %2;\n\t}" ::"r"(
            static_cast<int>(p)),
        "r"(cluster_addr), "r"(v)
        : "memory");
}
__device__ __forceinline__ void st_release_cluster_u32_if(bool p, uint32_t cluster_addr, uint32_t v) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.release.cluster.shared::cluster.u32 [%1], %2;\n\t}" ::"r"(
            static_cast<int>(p)),
        "r"(cluster_addr), "r"(v)
        : "memory");
}
__device__ __forceinline__ void st_gpu_u64_if(bool p, uint64_t* ptr, uint64_t v) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.relaxed.gpu.global.u64 [%1], %2;\n\t}" ::"r"(
                     static_cast<int>(p)),
                 "l"(ptr), "l"(v)
                 : "memory");
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
// Generic-address forms: one instruction serves a remote shared-memory slot
// (through mapa) and a global ring slot alike.
__device__ __forceinline__ uint64_t mapa_generic(const void* p, uint32_t rank) {
    uint64_t r;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
    return r;
}
// Two tagged u64 (each single-copy atomic; the pair need not be) in one store.
__device__ __forceinline__ void st_pair_if(bool p, uint64_t generic_addr, uint64_t a, uint64_t b) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.relaxed.cluster.v2.u64 [%1], {%2, %3};\n\t}" ::"r"(
            static_cast<int>(p)),
        "l"(generic_addr), "l"(a), "l"(b));
}
__device__ __forceinline__ void st_one_if(bool p, uint64_t generic_addr, uint64_t a) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q st.relaxed.cluster.u64 [%1], %2;\n\t}" ::"r"(
                     static_cast<int>(p)),
                 "l"(generic_addr), "l"(a));
}
__device__ __forceinline__ void ld_pair(uint64_t generic_addr, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.cluster.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(generic_addr));
}
__device__ __forceinline__ uint64_t ld_one(uint64_t generic_addr) {
    uint64_t a;
    asm volatile("ld.relaxed.cluster.u64 %0, [%1];" : "=l"(a) : "l"(generic_addr));
    return a;
}
// The same reads for a ring in this CTA's shared memory, by shared-window
// address.  Measured on B200, the generic-address forms above cost a consumer
// warp about 1000 cycles per group of 8 slots even when the data was ready;
// these cost about as much as ordinary shared loads.
__device__ __forceinline__ void ld_pair_shared(uint32_t saddr, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.cluster.shared::cta.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(saddr));
}
__device__ __forceinline__ uint64_t ld_one_shared(uint32_t saddr) {
    uint64_t a;
    asm volatile("ld.relaxed.cluster.shared::cta.u64 %0, [%1];" : "=l"(a) : "r"(saddr));
    return a;
}
// 16-byte global -> shared asynchronous copies (per-thread groups).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// 4-byte global -> shared asynchronous copy (any 4-byte alignment).
// Programmatic dependent launch.  A kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may be scheduled while the
// kernel before it in the stream is finishing; pdl_wait() blocks until that
// kernel has completed and its memory is visible, so it must come before the
// first access to global memory the previous kernel writes or reads.
// pdl_trigger() lets the next such kernel be launched once every CTA of this
// one has executed it (or exited).  Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch of a kernel that calls pdl_wait() before touching global memory,
// with programmatic stream serialization when `pdl`.  Used inside the
// barycenter iteration, a chain of short library kernels replayed from a CUDA
// graph (512 sequences: 0.122 -> 0.103 ms per iteration).  In the loss path
// measured on B200 it gained nothing on the device and made a step followed by
// a device-to-host copy ~20 us slower, so those launches keep the plain form.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared -> global bulk copies (async proxy), for staged table rows.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_s2g(void* gdst, uint32_t ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N bulk groups still reading their shared-memory sources.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every bulk group of this thread complete (its global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// mbarriers in this CTA's shared memory (shared-window addresses).
__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(mbar) : "memory");
}
// True once the phase of the given parity has completed.
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

// Arrival that also expects `bytes` of asynchronous copies on the barrier.
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
}
// Global -> shared bulk copy (async proxy), completion counted in bytes on an
// mbarrier.  Source and destination 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}

// Packed float32 pairs (sm_100 f32x2 arithmetic): a 64-bit register holds two
// floats, low half first.
__device__ __forceinline__ unsigned long long sub_f32x2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ float lo_f32x2(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f32x2(unsigned long long v) {
    return __uint_as_float(static_cast<uint32_t>(v >> 32));
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
// device synchronisation; kernels only write it (once, on failure).  Waiters
// learn about another waiter's failure from `abort_flag` in device memory,
// which they read at most every few thousand polls.
enum : int {
    kStatusOk = 0,
    kStatusTimeout = 3,
    kStatusRange = 4,  // a value left the range of the exponential-domain forward
};

// Where a wait gave up (written next to the status word, for diagnostics).
struct WaitDiag {
    int kernel;   // 1 forward, 2 backward
    int kind;     // 1 smem tag, 2 global tag, 3 flow-control counter
    int problem;  // batch index
    int warp;     // warp index within the band chain
    int band;
    int expect;   // expected tag / counter value
    int seen;     // last tag / counter value seen
    int pad;
};

struct WaitCtx {
    volatile int* status;      // mapped pinned host word (may be null)
    volatile WaitDiag* diag;   // mapped pinned host record (may be null)
    volatile int* abort_flag;  // device word, nonzero once any wait failed (may be null)
    uint64_t timeout_ns;       // wall-clock limit for one wait
    int kernel, problem, warp, band;
};

__device__ __forceinline__ void record_error(const WaitCtx& w, int code, int kind, uint32_t expect, uint32_t seen) {
    if (w.abort_flag) *w.abort_flag = 1;
    if (w.diag) {
        w.diag->kernel = w.kernel;
        w.diag->kind = kind;
        w.diag->problem = w.problem;
        w.diag->warp = w.warp;
        w.diag->band = w.band;
        w.diag->expect = static_cast<int>(expect);
        w.diag->seen = static_cast<int>(seen);
    }
    __threadfence_system();
    if (w.status) *w.status = code;
}

// A wait that gave up because another wait had failed (the abort flag) also
// marks its launch as failed, so that no launch can finish with a wrong
// result and an ok status, whichever status word the first failure went to.
// The first failure's diagnostics are kept; kind 5 marks an abort.
__device__ __forceinline__ void record_abort(const WaitCtx& w) {
    if (w.status && *w.status == 0) {
        if (w.diag) {
            w.diag->kernel = w.kernel;
            w.diag->kind = 5;
            w.diag->problem = w.problem;
            w.diag->warp = w.warp;
            w.diag->band = w.band;
            w.diag->expect = 0;
            w.diag->seen = 0;
        }
        __threadfence_system();
        *w.status = kStatusTimeout;
    }
}

// A forward whose scores left the representable range (or met a NaN cost)
// marks its launch failed with kStatusRange; kind 6 in the diagnostics.  It
// does not raise the abort flag: no wait is affected.
__device__ __forceinline__ void record_range(const WaitCtx& w) {
    if (w.status && *w.status == 0) {
        if (w.diag) {
            w.diag->kernel = w.kernel;
            w.diag->kind = 6;
            w.diag->problem = w.problem;
            w.diag->warp = w.warp;
            w.diag->band = w.band;
            w.diag->expect = 0;
            w.diag->seen = 0;
        }
        __threadfence_system();
        *w.status = kStatusRange;
    }
}

// r as returned by backoff(): 1 = this wait ran out of time, 2 = aborted.
__device__ __forceinline__ void record_giveup(const WaitCtx& w, int r, int kind, uint32_t expect, uint32_t seen) {
    if (r == 1) record_error(w, kStatusTimeout, kind, expect, seen);
    else if (r == 2) record_abort(w);
}

// Shared back-off policy of the slow paths: poll tightly, look at the clock
// every 256 polls, at the device abort flag every 4096 polls once the wait is
// older than 20 us, and sleep between polls once it is older than 1 ms.
// Returns 0 to keep polling, 1 when the limit ran out, 2 on abort.
__device__ __forceinline__ int backoff(uint32_t it, uint64_t& t0, const WaitCtx& w) {
    if ((it & 255u) != 0u) return 0;
    const uint64_t now = globaltimer_ns();
    if (t0 == 0) {
        t0 = now;
        return 0;
    }
    const uint64_t el = now - t0;
    if (el > w.timeout_ns) return 1;
    if (el > 20000u && (it & 4095u) == 0u && w.abort_flag && *w.abort_flag) return 2;
    if (el > 1000000u) __nanosleep(256);
    return 0;
}

// Slow paths of the ring protocol.  They return their result by value (never
// through a reference), so the caller's values stay in registers: a reference
// into a non-inlined call would move them to local memory on the hot path.

// Polls the u64 at generic address `ga` until it carries `tag`; returns the
// last entry read (success iff its tag equals `tag`).
static __device__ __noinline__ uint64_t wait_tag_generic(uint64_t ga, uint32_t tag, const WaitCtx& w) {
    uint64_t t0 = 0;
    uint64_t e = 0;
    for (uint32_t it = 1;; ++it) {
        e = ld_one(ga);
        if (tag_of(e) == tag) return e;
        const int r = backoff(it, t0, w);
        record_giveup(w, r, 1, tag, tag_of(e));
        if (r) return e;
    }
}

// Polls the u32 counter at own-CTA smem address `saddr` until it is >= `need`;
// returns the last value read (success iff >= need).
static __device__ __noinline__ uint32_t wait_counter_ge(uint32_t saddr, uint32_t need, const WaitCtx& w) {
    uint64_t t0 = 0;
    uint32_t seen = 0;
    for (uint32_t it = 1;; ++it) {
        seen = ld_acquire_cluster_u32(saddr);
        if (static_cast<int32_t>(seen - need) >= 0) return seen;
        const int r = backoff(it, t0, w);
        record_giveup(w, r, 3, need, seen);
        if (r) return seen;
    }
}

}  // namespace sdtw
