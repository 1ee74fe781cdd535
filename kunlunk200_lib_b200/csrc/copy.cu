// Copies done by a kernel on the library stream (k200_copy_kernel): either
// side may be pinned host memory, which the kernel reads or writes over the
// bus (pinned memory is mapped into the device's address space under unified
// addressing).  Unlike a copy-engine transfer, the kernel takes part in the
// programmatic-launch chain: the matmul after an input copy starts streaming
// its weights while the copy runs, which is what a decode step (input in,
// GEMVs, output out) needs.
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

__global__ void __launch_bounds__(256) copy_kernel(uint8_t *dst, const uint8_t *src, size_t bytes, int vec16) {
    pdl_launch_dependents();
    pdl_wait_prior();  // dst or src may belong to the previous kernel
    const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t done = 0;
    if (vec16) {
        const size_t n16 = bytes / 16;
        const uint4 *s = reinterpret_cast<const uint4 *>(src);
        uint4 *d = reinterpret_cast<uint4 *>(dst);
        for (size_t i = tid; i < n16; i += stride) d[i] = s[i];
        done = n16 * 16;
    }
    for (size_t i = done + tid; i < bytes; i += stride) dst[i] = src[i];
}

}  // namespace

cudaError_t launch_copy_kernel(void *dst, const void *src, size_t bytes, const DeviceInfo &dev, cudaStream_t stream) {
    if (bytes == 0) return cudaSuccess;
    const bool vec16 = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
    const size_t work = vec16 ? bytes / 16 + 1 : bytes;
    const size_t want = (work + 255) / 256;
    const int grid = static_cast<int>(want < static_cast<size_t>(dev.sm_count) ? (want < 1 ? 1 : want) : dev.sm_count);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, copy_kernel, static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), bytes,
                              vec16 ? 1 : 0);
}

}  // namespace k200
