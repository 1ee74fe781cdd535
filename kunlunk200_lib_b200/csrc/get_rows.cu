// Row gathers (sm_100a): get_rows_f32 copies rows of an F32 matrix and
// common_q4_get_rows decodes rows of a common-Q4 weight (column = output row)
// to F32, for indices given on the device (src/get-rows-f32.inc,
// src/get-rows.inc of the reference).  An index outside [0, n) makes the call
// write no output: every CTA checks all indices (at most 512) before it
// writes, and CTA (0, 0) records the verdict in a status word the host reads.
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

__device__ __forceinline__ bool indices_ok(const int32_t *idx, int rows, int n) {
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
        const int v = idx[i];
        if (v < 0 || v >= n) bad = 1;
    }
    __syncthreads();
    return bad == 0;
}

// grid: (chunks of 1024 float4 of a row, rows)
__global__ void __launch_bounds__(256) get_rows_f32_kernel(float4 *out, const float4 *in, const int32_t *idx,
                                                          int *status, int k4, int n, int rows) {
    const bool ok = indices_ok(idx, rows, n);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *status = ok ? 0 : 1;
    if (!ok) return;
    const int r = blockIdx.y;
    const float4 *src = in + static_cast<size_t>(idx[r]) * k4;
    float4 *dst = out + static_cast<size_t>(r) * k4;
    const int c0 = blockIdx.x * 1024;
    for (int c = c0 + threadIdx.x; c < k4 && c < c0 + 1024; c += blockDim.x) dst[c] = __ldg(src + c);
}

// grid: (chunks of 128 blocks of a row, rows); one thread decodes one 32-value block
__global__ void __launch_bounds__(128) common_get_rows_kernel(float *out, const uint8_t *w, size_t scale_offset,
                                                            int kp, int np, const int32_t *idx, int *status, int k,
                                                            int n, int rows) {
    const bool ok = indices_ok(idx, rows, n);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *status = ok ? 0 : 1;
    if (!ok) return;
    const int r = blockIdx.y, kb = blockIdx.x * 128 + threadIdx.x;
    if (kb >= k / 32) return;
    const int col = idx[r];
    // column col's 16 bytes of block kb: elements 2p (low nibble) and 2p+1 (high) of byte p,
    // as signed 4-bit values
    const size_t tile = static_cast<size_t>(col / 32) * (kp / 32);
    const int lane = col & 31;
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(w + (tile + kb) * 512 + (lane & 15) * 32 + (lane >> 4) * 16));
    const uint16_t dbits = __ldg(reinterpret_cast<const uint16_t *>(w + scale_offset) + static_cast<size_t>(kb) * np + col);
    const float d = __half2float(__ushort_as_half(dbits));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float4 *dst = reinterpret_cast<float4 *>(out + static_cast<size_t>(r) * k + kb * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float e[8];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t byte = (u[i] >> (8 * b)) & 0xffu;
            // signed 4-bit values (q - 8 in two's complement)
            e[2 * b] = static_cast<float>(static_cast<int>((byte & 15u) ^ 8u) - 8) * d;
            e[2 * b + 1] = static_cast<float>(static_cast<int>((byte >> 4) ^ 8u) - 8) * d;
        }
        dst[2 * i] = make_float4(e[0], e[1], e[2], e[3]);
        dst[2 * i + 1] = make_float4(e[4], e[5], e[6], e[7]);
    }
}

}  // namespace

cudaError_t launch_get_rows_f32(float *out, const float *in, const int32_t *idx, int *status, int k, int n, int rows,
                                cudaStream_t stream) {
    const int k4 = k / 4;
    dim3 grid((k4 + 1023) / 1024, rows);
    get_rows_f32_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<float4 *>(out), reinterpret_cast<const float4 *>(in),
                                                  idx, status, k4, n, rows);
    return cudaGetLastError();
}

cudaError_t launch_common_get_rows(float *out, const uint8_t *w, size_t scale_offset, int kp, int np,
                                   const int32_t *idx, int *status, int k, int n, int rows, cudaStream_t stream) {
    dim3 grid((k / 32 + 127) / 128, rows);
    common_get_rows_kernel<<<grid, 128, 0, stream>>>(out, w, scale_offset, kp, np, idx, status, k, n, rows);
    return cudaGetLastError();
}

}  // namespace k200
