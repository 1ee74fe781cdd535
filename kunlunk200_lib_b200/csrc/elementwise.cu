// kunlun::elementwise on the device (sm_100a): the step after the matmul in
// the reference's `pipeline` benchmark (bench/library-bench.cpp:113).
// Semantics of kernels/kunlun-elementwise.xpu:9-64 of the reference:
//   add       y = a + b            (b broadcast with period b_count)
//   multiply  y = a * b
//   silu      y = a / (1 + exp(-a))
//   rms_norm  y = a * (1 / sqrt(sum(a^2)/width + eps)) per row of `width`
//   scale     y = a * parameter
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

__global__ void elementwise_kernel(float *y, const float *a, const float *b, int n, int bn, int op, float p) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = a[i];
        float out;
        if (op == 0) out = v + b[bn == n ? i : i % bn];
        else if (op == 1) out = v * b[bn == n ? i : i % bn];
        else if (op == 2) out = v / (1.0f + expf(-v));
        else out = v * p;
        y[i] = out;
    }
}

__global__ void rms_kernel(float *y, const float *a, int width, float eps) {
    __shared__ float part[32];
    const float *row = a + static_cast<long long>(blockIdx.x) * width;
    float *out = y + static_cast<long long>(blockIdx.x) * width;
    float s = 0.f;
    for (int j = threadIdx.x; j < width; j += blockDim.x) s += row[j] * row[j];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) part[0] = t;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(part[0] / width + eps);
    for (int j = threadIdx.x; j < width; j += blockDim.x) out[j] = row[j] * scale;
}

}  // namespace

cudaError_t launch_elementwise(float *y, const float *a, const float *b, int n, int width, int bn, int op, float p,
                               const DeviceInfo &dev, cudaStream_t stream) {
    if (op == 3) {
        rms_kernel<<<n / width, 256, 0, stream>>>(y, a, width, p);
    } else {
        int blocks = (n + 255) / 256;
        if (blocks > dev.sm_count * 8) blocks = dev.sm_count * 8;
        elementwise_kernel<<<blocks, 256, 0, stream>>>(y, a, b, n, bn, op, p);
    }
    return cudaGetLastError();
}

}  // namespace k200
