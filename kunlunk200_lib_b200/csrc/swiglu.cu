// kunlun::swiglu on the device (sm_100a): y = SiLU(gate) * up per element,
// rows of `width` F32 or F16 values at byte strides, with F32 intermediates
// and one final rounding (kernels/kunlun-swiglu.xpu of the reference):
//   act = g / (1 + exp(-g));  y = act * u
// and the reference's rules for non-finite inputs (g or u NaN, or g = -inf:
// NaN; g = +inf: NaN if u = 0 else +-inf with the product's sign; u = +-inf:
// NaN if act = 0 else +-inf).  F16 inputs are widened exactly; an F16 output
// is the F32 result rounded to nearest.
#include <cuda_fp16.h>

#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

__device__ __forceinline__ float swiglu_value(float g, float u) {
    const uint32_t gb = __float_as_uint(g), ub = __float_as_uint(u);
    const uint32_t ga = gb & 0x7fffffffu, ua = ub & 0x7fffffffu;
    if (ga < 0x7f800000u && ua < 0x7f800000u) return (g / (1.0f + expf(-g))) * u;
    const uint32_t sign = (gb ^ ub) & 0x80000000u;
    if (ga > 0x7f800000u || ua > 0x7f800000u || gb == 0xff800000u) return __uint_as_float(0x7fc00000u);
    if (ga == 0x7f800000u) return __uint_as_float(ua == 0 ? 0x7fc00000u : (sign | 0x7f800000u));
    const float act = g / (1.0f + expf(-g));
    return __uint_as_float((__float_as_uint(act) & 0x7fffffffu) == 0 ? 0x7fc00000u : (sign | 0x7f800000u));
}

// grid-stride over rows x width elements; strides in bytes
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(uint8_t *y, const uint8_t *gate, const uint8_t *up, int width,
                                                     int rows, int gs, int us, int ys) {
    const long long total = static_cast<long long>(width) * rows;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / width), j = static_cast<int>(i - static_cast<long long>(r) * width);
        const T gv = reinterpret_cast<const T *>(gate + static_cast<size_t>(r) * gs)[j];
        const T uv = reinterpret_cast<const T *>(up + static_cast<size_t>(r) * us)[j];
        float out;
        if constexpr (sizeof(T) == 4) {
            out = swiglu_value(gv, uv);
            reinterpret_cast<T *>(y + static_cast<size_t>(r) * ys)[j] = out;
        } else {
            out = swiglu_value(__half2float(gv), __half2float(uv));
            reinterpret_cast<T *>(y + static_cast<size_t>(r) * ys)[j] = __float2half_rn(out);
        }
    }
}

}  // namespace

cudaError_t launch_swiglu(void *y, const void *gate, const void *up, int width, int rows, int gs, int us, int ys,
                          int f16, const DeviceInfo &dev, cudaStream_t stream) {
    const long long total = static_cast<long long>(width) * rows;
    const long long want = (total + 255) / 256;
    const int grid = static_cast<int>(want < dev.sm_count * 8 ? (want < 1 ? 1 : want) : dev.sm_count * 8);
    if (f16)
        swiglu_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<uint8_t *>(y), static_cast<const uint8_t *>(gate),
                                                        static_cast<const uint8_t *>(up), width, rows, gs, us, ys);
    else
        swiglu_kernel<float><<<grid, 256, 0, stream>>>(static_cast<uint8_t *>(y), static_cast<const uint8_t *>(gate),
                                                       static_cast<const uint8_t *>(up), width, rows, gs, us, ys);
    return cudaGetLastError();
}

}  // namespace k200
