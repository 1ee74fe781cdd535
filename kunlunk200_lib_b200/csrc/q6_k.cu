// Q6_K typed GEMV (sm_100a): Y[r] = sum over 16-value groups g of
// dot(w[r, g], q[g]) * wscale[r, g] * ascale[g / 16], the arithmetic of the
// reference's kunlun-q6-quant / kunlun-q6-onchip kernels (src/q6-k.inc):
//  * activations are quantised per 256-value chunk (symmetric A8): scale =
//    max|x| / 127, q = trunc(x * (127 / max) +- 0.5) clamped to +-127 (0 for
//    an all-zero chunk);
//  * weights are the Q6_K values q - 32 as int8 in the packed layout
//    [N32 tile][K16 group][16 values][32 rows], with one f32 scale
//    d * sub-scale (exact in f32) per row and group at
//    scale_offset + ((tile * groups + g) * 32 + row % 32) * 4;
//  * each group's int8 dot is exact; the FP32 sum runs over groups in order.
#include <cuda_fp16.h>

#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

// one CTA per 256-value chunk of one activation row
__global__ void __launch_bounds__(256) q6_quant_kernel(const void *x, int dtype, int8_t *q, float *scales) {
    __shared__ float red[8];
    const int b = blockIdx.x, j = threadIdx.x;
    const float v = dtype ? __half2float(static_cast<const __half *>(x)[b * 256 + j])
                          : static_cast<const float *>(x)[b * 256 + j];
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((j & 31) == 0) red[j >> 5] = m;
    __syncthreads();
    float mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    const float inv = mx > 0.f ? __fdiv_rn(127.f, mx) : 0.f;
    const float t = __fmul_rn(v, inv);
    int z = static_cast<int>(__fadd_rn(t, t >= 0.f ? 0.5f : -0.5f));
    z = z > 127 ? 127 : (z < -127 ? -127 : z);
    q[b * 256 + j] = static_cast<int8_t>(z);
    if (j == 0) scales[b] = mx > 0.f ? __fdiv_rn(mx, 127.f) : 0.f;
}

// warp per 32-row tile, lane = row; the chunk's quantised values and scales in shared memory
__global__ void __launch_bounds__(256) q6_gemv_kernel(float *y, const int8_t *w, const float *wscale,
                                                      const int8_t *qg, const float *ascale, int k, int n) {
    extern __shared__ __align__(16) int8_t q6s[];  // [k] int8, then [k/256] float
    float *as = reinterpret_cast<float *>(q6s + k);
    for (int i = threadIdx.x; i < k / 16; i += blockDim.x)
        reinterpret_cast<int4 *>(q6s)[i] = reinterpret_cast<const int4 *>(qg)[i];
    for (int i = threadIdx.x; i < k / 256; i += blockDim.x) as[i] = ascale[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int groups = k / 16, tiles = n / 32;
    for (int tile = blockIdx.x * warps + warp; tile < tiles; tile += gridDim.x * warps) {
        const int8_t *wt = w + static_cast<size_t>(tile) * groups * 512 + lane;
        const float *st = wscale + static_cast<size_t>(tile) * groups * 32 + lane;
        float sum = 0.f;
        for (int g = 0; g < groups; ++g) {
            const int8_t *wg = wt + static_cast<size_t>(g) * 512;
            const int8_t *qv = q6s + g * 16;
            int dot = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) dot += static_cast<int>(__ldg(wg + j * 32)) * static_cast<int>(qv[j]);
            sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(static_cast<float>(dot), as[g >> 4]), __ldg(st + g * 32)));
        }
        y[tile * 32 + lane] = sum;
    }
}

}  // namespace

cudaError_t launch_q6_quant(const void *x, int dtype, int k, int8_t *q, float *scales, cudaStream_t stream) {
    q6_quant_kernel<<<k / 256, 256, 0, stream>>>(x, dtype, q, scales);
    return cudaGetLastError();
}

cudaError_t launch_q6_gemv(float *y, const int8_t *w, const float *wscale, const int8_t *q, const float *ascale, int k,
                           int n, const DeviceInfo &dev, cudaStream_t stream) {
    const int tiles = n / 32;
    const int want = (tiles + 7) / 8;
    const int grid = want < dev.sm_count * 8 ? (want < 1 ? 1 : want) : dev.sm_count * 8;
    q6_gemv_kernel<<<grid, 256, static_cast<size_t>(k) + 4 * static_cast<size_t>(k / 256), stream>>>(y, w, wscale, q,
                                                                                                  ascale, k, n);
    return cudaGetLastError();
}

}  // namespace k200
