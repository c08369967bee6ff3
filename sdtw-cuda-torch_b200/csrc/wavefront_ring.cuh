// wavefront_ring.cuh -- pieces shared by the wavefront kernels (wavefront.cu,
// wavefront_exp.cu): the stripe-to-stripe ring geometry, the tag of the
// global band-wrap ring, progress reporting, the layout offset of a stripe and
// the cluster launch helper.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "sdtw_plan.h"

namespace sdtw {

constexpr int kRing = 128;  // ring slots per warp (power of two)

// Byte offset of the forward's staging buffers: after the rings ([wpc][kRing][2]
// u64) and the consumption counters ([wpc] u32), 16-byte aligned for the bulk
// copies.
__host__ __device__ constexpr size_t fwd_stage_offset(int wpc) {
    return (static_cast<size_t>(wpc) * (2 * kRing * 8 + 4) + 15) / 16 * 16;
}

// Tag of a band-wrap ring slot: the launch sequence number and the band that
// wrote it.
__device__ __forceinline__ uint32_t wrap_tag(uint32_t seq, int band) {
    return (seq << 12) | (static_cast<uint32_t>(band) & 0xfffu);
}

// `done` columns consumed, PF more than after the previous group: report
// when a multiple of 32 was crossed, and at the end of the row.
__device__ __forceinline__ bool report_due(int done, int PF, int M) {
    return (done & 31) < PF || done >= M;
}

__host__ __device__ __forceinline__ size_t stripe_base(const WavePlan& P, int b, int s) {
    return (static_cast<size_t>(b) * P.n_stripes + s) * static_cast<size_t>(P.n_diag) * (32 * P.K);
}

// One launch of `fn` in thread-block clusters of `csize` CTAs along x.
// pdl: the kernel calls pdl_wait() before touching global memory, so it may
// be launched with programmatic stream serialization.
inline cudaError_t launch_cluster(const void* fn, dim3 grid, dim3 block, size_t smem, int csize,
                                  cudaStream_t stream, void** args, bool pdl = false) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace sdtw
