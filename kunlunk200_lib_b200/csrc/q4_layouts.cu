// Kernels of the native and common Q4 layouts (sm_100a): the W4A8x2 GEMV of
// native_q4_matmul and common_q4_matmul (M = 1), the exact FP32 fallback of
// native_q4_matmul, and the Row-A8 GEMM of common_q4_matmul (M > 1).
//
// Arithmetic (restated from the reference, every float step round-to-nearest
// with no contraction, so results are bit-identical to the CPU restatement):
//  * two-component A8 of one activation vector, kernels/kunlun-native-q4-
//    {max,main,residual}.xpu and kernels/native-q4/quant.h:4-10:
//      max0 = max |x| (F16 input: max of the F16 magnitudes, then widened),
//      1 if 0;  q0 = round(x * (127/max0));  r = x - (max0/127) * q0;
//      max1 = max |r| (1 if 0);  q1 = round(r * (127/max1));
//      params = {max0/127, max1/127, max0, max1}
//    (round = half away from zero, clamped to +-127);
//  * W4A8x2 block partial, kernels/kunlun-native-q4.xpu and the common GEMV
//    (src/q4-common.inc:203-238):  partial = (dot0 * s0 + dot1 * s1) * d with
//    exact int32 dots of the signed 4-bit weights and the two components,
//    then y = sum of the partials in increasing block order;
//  * exact FP32 fallback, kernels/kunlun-native-q4-fallback.xpu (the
//    kunlun-matvec arithmetic): per block acc[l] = q[l] x[l] (l < 8), then
//    acc[l] += q[j+l] x[j+l] for j = 8, 16, 24; s = serial sum of acc;
//    y += d * s;
//  * Row A8 of the common GEMM, .../quant-row-serial-fused.xpu:8-23: per
//    activation row, scale = max|x|/127, q = round(x * 127/max); then per
//    block t = dot * d, y = (sum of t in block order) * scale.
//
// Layouts (weights stay in the packed form; nothing is converted at call time):
//  * native, src/q4-layout.cpp:15-37: [N32 tile][K32 block][16 byte pairs]
//    [32 rows] of signed 4-bit pairs (element 2j low nibble, 2j+1 high), FP16
//    scales after the 256-aligned payload at (tile_block*32 + row%32)*2.  A
//    warp takes a tile with lane = row: every load of the warp is 32
//    consecutive bytes;
//  * common Micro32Bank, src/q4-common-pack.h:16-31: within a 512-byte block
//    of a 32-column tile, column c's 16 bytes are contiguous at
//    (c%16)*32 + (c/16%2)*16, so a lane (= column) reads its block with one
//    16-byte load; K-major FP16 scales at scale_offset + (kb*np + c)*2.
#include <cuda_fp16.h>

#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

__device__ __forceinline__ float half_bits(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }

__device__ __forceinline__ int round_half_away_127(float v) {
    const float t = __fadd_rn(v, v >= 0.f ? 0.5f : -0.5f);
    const int q = static_cast<int>(t);
    return q > 127 ? 127 : (q < -127 ? -127 : q);
}

__device__ __forceinline__ float load_act(const void *x, int dtype, size_t i) {
    return dtype ? __half2float(static_cast<const __half *>(x)[i]) : static_cast<const float *>(x)[i];
}

__device__ __forceinline__ uint32_t cta_max(uint32_t v, uint32_t *scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = threadIdx.x < (blockDim.x >> 5) ? scratch[threadIdx.x] : 0u;
    if (warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) scratch[0] = v;
    }
    __syncthreads();
    return scratch[0];
}

__device__ __forceinline__ int sign4(uint32_t v) { return static_cast<int>(v & 15u) - static_cast<int>((v & 8u) << 1); }

// ---- two-component A8 of one vector (one CTA) ------------------------------
// Element j of component c goes to q_c[j] (kq == 0) or, for the common
// layout's activation view, to q_c[(j/32)*64 + j%32] with every other byte of
// the first 2*kq zeroed (kq = padded K).
__device__ __forceinline__ int a8x2_index(int j, int kq) { return kq ? (j >> 5) * 64 + (j & 31) : j; }

__global__ void __launch_bounds__(1024) a8x2_kernel(const void *x, int k, int dtype, int kq, int8_t *q0, int8_t *q1,
                                                    float *params) {
    extern __shared__ float rest[];  // [k] residuals
    __shared__ uint32_t scratch[32];
    uint32_t m = 0;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const uint32_t u = dtype ? (static_cast<const uint16_t *>(x)[j] & 0x7fffu)
                                 : (__float_as_uint(static_cast<const float *>(x)[j]) & 0x7fffffffu);
        m = max(m, u);
    }
    uint32_t m0 = cta_max(m, scratch);
    if (dtype) m0 = __float_as_uint(half_bits(m0));
    const float max0 = m0 ? __uint_as_float(m0) : 1.f;
    const float scale0 = __fdiv_rn(max0, 127.f), inverse0 = __fdiv_rn(127.f, max0);
    m = 0;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const float v = load_act(x, dtype, j);
        const int q = round_half_away_127(__fmul_rn(inverse0, v));
        q0[a8x2_index(j, kq)] = static_cast<int8_t>(q);
        const float r = __fsub_rn(v, __fmul_rn(scale0, static_cast<float>(q)));
        rest[j] = r;
        m = max(m, __float_as_uint(r) & 0x7fffffffu);
    }
    const uint32_t m1 = cta_max(m, scratch);
    const float max1 = m1 ? __uint_as_float(m1) : 1.f;
    const float inverse1 = __fdiv_rn(127.f, max1);
    for (int j = threadIdx.x; j < k; j += blockDim.x)
        q1[a8x2_index(j, kq)] = static_cast<int8_t>(round_half_away_127(__fmul_rn(inverse1, rest[j])));
    if (kq) {
        for (int i = threadIdx.x; i < 2 * kq; i += blockDim.x)
            if (((i & 63) >= 32) || ((i >> 6) * 32 + (i & 31) >= k)) q0[i] = q1[i] = 0;
    }
    if (threadIdx.x == 0) {
        params[0] = scale0;
        params[1] = __fdiv_rn(max1, 127.f);
        params[2] = max0;
        params[3] = max1;
    }
}

// ---- Row A8 (one CTA per activation row) ------------------------------------
// Row scales are stored every `scale_stride` floats.
__global__ void __launch_bounds__(256) row_a8_kernel(const void *x, int k, int dtype, int kq, int8_t *q, float *row_scale,
                                                     int scale_stride) {
    __shared__ uint32_t scratch[32];
    const size_t base = static_cast<size_t>(blockIdx.x) * k;
    uint32_t m = 0;
    for (int j = threadIdx.x; j < k; j += blockDim.x) m = max(m, __float_as_uint(load_act(x, dtype, base + j)) & 0x7fffffffu);
    m = cta_max(m, scratch);
    const float mx = m ? __uint_as_float(m) : 1.f;
    const float inv = __fdiv_rn(127.f, mx);
    int8_t *out = q + static_cast<size_t>(blockIdx.x) * kq;
    for (int j = threadIdx.x; j < kq; j += blockDim.x)
        out[j] = j < k ? static_cast<int8_t>(round_half_away_127(__fmul_rn(inv, load_act(x, dtype, base + j)))) : 0;
    if (threadIdx.x == 0) row_scale[static_cast<size_t>(blockIdx.x) * scale_stride] = __fdiv_rn(mx, 127.f);
}

__device__ __forceinline__ float a8x2_partial(int dot0, int dot1, float s0, float s1, float d) {
    return __fmul_rn(__fadd_rn(__fmul_rn(static_cast<float>(dot0), s0), __fmul_rn(static_cast<float>(dot1), s1)), d);
}

// ---- native W4A8x2 GEMV: one warp per 32-row tile, lane = row ---------------
__global__ void __launch_bounds__(256) native_gemv_a8x2_kernel(const uint8_t *w, const uint16_t *scales,
                                                                const int8_t *q0g, const int8_t *q1g,
                                                                const float *params, int k, int n, float *y) {
    extern __shared__ int8_t qs[];  // [2][k]
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        qs[j] = q0g[j];
        qs[k + j] = q1g[j];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int blocks = k / 32, tiles = (n + 31) / 32;
    const float s0 = params[0], s1 = params[1];
    for (int tile = blockIdx.x * warps + warp; tile < tiles; tile += gridDim.x * warps) {
        float sum = 0.f;
        for (int b = 0; b < blocks; ++b) {
            const size_t tb = static_cast<size_t>(tile) * blocks + b;
            const uint8_t *panel = w + tb * 512 + lane;
            const float d = half_bits(__ldg(scales + tb * 32 + lane));
            const int8_t *a0 = qs + b * 32, *a1 = qs + k + b * 32;
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t v = __ldg(panel + j * 32);
                const int lo = sign4(v), hi = sign4(v >> 4);
                dot0 += lo * a0[2 * j] + hi * a0[2 * j + 1];
                dot1 += lo * a1[2 * j] + hi * a1[2 * j + 1];
            }
            sum = __fadd_rn(sum, a8x2_partial(dot0, dot1, s0, s1, d));
        }
        const int row = tile * 32 + lane;
        if (row < n) y[row] = sum;
    }
}

// ---- native exact FP32 fallback: CTA row per activation column, warp per tile ----
__global__ void __launch_bounds__(256) native_fallback_kernel(const uint8_t *w, const uint16_t *scales, const void *x,
                                                              int dtype, int k, int n, int batch, float *y) {
    extern __shared__ float xs[];  // [k] activations of this column
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int blocks = k / 32, tiles = (n + 31) / 32;
    for (int col = blockIdx.y; col < batch; col += gridDim.y) {
    __syncthreads();
    for (int j = threadIdx.x; j < k; j += blockDim.x) xs[j] = load_act(x, dtype, static_cast<size_t>(col) * k + j);
    __syncthreads();
    for (int tile = blockIdx.x * warps + warp; tile < tiles; tile += gridDim.x * warps) {
        float sum = 0.f;
        for (int b = 0; b < blocks; ++b) {
            const size_t tb = static_cast<size_t>(tile) * blocks + b;
            const uint8_t *panel = w + tb * 512 + lane;
            const float d = half_bits(__ldg(scales + tb * 32 + lane));
            float q[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t v = __ldg(panel + j * 32);
                q[2 * j] = static_cast<float>(sign4(v));
                q[2 * j + 1] = static_cast<float>(sign4(v >> 4));
            }
            const float *xb = xs + b * 32;
            float acc[8];
#pragma unroll
            for (int l = 0; l < 8; ++l) acc[l] = __fmul_rn(q[l], xb[l]);
#pragma unroll
            for (int j = 8; j < 32; j += 8)
#pragma unroll
                for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], __fmul_rn(q[j + l], xb[j + l]));
            float s = 0.f;
#pragma unroll
            for (int l = 0; l < 8; ++l) s = __fadd_rn(s, acc[l]);
            sum = __fadd_rn(sum, __fmul_rn(d, s));
        }
        const int row = tile * 32 + lane;
        if (row < n) y[static_cast<size_t>(col) * n + row] = sum;
    }
    }
}

// ---- common layout ------------------------------------------------------------
// Column c's 16 bytes of block kb: elements 2p (low nibble) and 2p+1 (high) of byte p.
__device__ __forceinline__ uint4 common_block(const uint8_t *w, int kp, int col, int kb) {
    const size_t tile = static_cast<size_t>(col / 32) * (kp / 32);
    const int lane = col & 31;
    return __ldg(reinterpret_cast<const uint4 *>(w + (tile + kb) * 512 + (lane & 15) * 32 + (lane >> 4) * 16));
}

// 4 bytes of nibble pairs -> 2 words of 4 signed int8 weights in element order.
__device__ __forceinline__ void common_unpack(uint32_t u, uint32_t &e0, uint32_t &e1) {
    const uint32_t lo = u & 0x0f0f0f0fu, hi = (u >> 4) & 0x0f0f0f0fu;
    e0 = __vsub4(__byte_perm(lo, hi, 0x5140) ^ 0x08080808u, 0x08080808u);  // lo(b0) hi(b0) lo(b1) hi(b1)
    e1 = __vsub4(__byte_perm(lo, hi, 0x7362) ^ 0x08080808u, 0x08080808u);  // lo(b2) hi(b2) lo(b3) hi(b3)
}

// M = 1: W4A8x2 GEMV, lane = column.  The components come in the activation
// view layout (block b's 32 values at b*64), zero past k.  With a second
// weight (w1, y1: the gate/up pair) the same activation records serve both:
// tiles [0, T) of the grid walk belong to w and [T, 2T) to w1.
__global__ void __launch_bounds__(256) common_gemv_a8x2_kernel(const uint8_t *w, const uint8_t *w1, size_t scale_offset,
                                                                int kp, int np, const int8_t *q0g, const int8_t *q1g,
                                                                const float *params, int k, int n, float *y,
                                                                float *y1) {
    extern __shared__ int qw[];  // [2][kp/4] int8x4 words, blocks packed densely
    const int words = kp / 4;
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
        const int src = (i >> 3) * 16 + (i & 7);  // word of block i/8 in the 64-byte view groups
        qw[i] = reinterpret_cast<const int *>(q0g)[src];
        qw[words + i] = reinterpret_cast<const int *>(q1g)[src];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int blocks = (k + 31) / 32, tiles = (n + 31) / 32, walk = w1 ? 2 * tiles : tiles;
    const float s0 = params[0], s1 = params[1];
    for (int t = blockIdx.x * warps + warp; t < walk; t += gridDim.x * warps) {
        const bool second = t >= tiles;
        const int tile = second ? t - tiles : t;
        const uint8_t *ww = second ? w1 : w;
        float *yy = second ? y1 : y;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(ww + scale_offset);
        const int col = tile * 32 + lane;
        float sum = 0.f;
        for (int kb = 0; kb < blocks; ++kb) {
            const uint4 v = common_block(ww, kp, col, kb);
            const float d = half_bits(__ldg(sc + static_cast<size_t>(kb) * np + col));
            const int *a0 = qw + kb * 8, *a1 = qw + words + kb * 8;
            int dot0 = 0, dot1 = 0;
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t e0, e1;
                common_unpack(u[i], e0, e1);
                dot0 = __dp4a(static_cast<int>(e0), a0[2 * i], dot0);
                dot0 = __dp4a(static_cast<int>(e1), a0[2 * i + 1], dot0);
                dot1 = __dp4a(static_cast<int>(e0), a1[2 * i], dot1);
                dot1 = __dp4a(static_cast<int>(e1), a1[2 * i + 1], dot1);
            }
            sum = __fadd_rn(sum, a8x2_partial(dot0, dot1, s0, s1, d));
        }
        if (col < n) yy[col] = sum;
    }
}

// M > 1: Row-A8 GEMM.  CTA = one 32-column tile x 32 activation rows (8 per warp).
constexpr int kGemmRowsPerWarp = 8;
__global__ void __launch_bounds__(128) common_gemm_a8_kernel(const uint8_t *w, size_t scale_offset, int kp, int np,
                                                             const int8_t *q, const float *row_scale, int k, int n,
                                                             int m, float *y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = blockIdx.x * 32 + lane;
    const int blocks = (k + 31) / 32;
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(w + scale_offset);
    for (int rt = blockIdx.y; rt * 32 < m; rt += gridDim.y) {
    const int r0 = rt * 32 + warp * kGemmRowsPerWarp;
    float sum[kGemmRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kGemmRowsPerWarp; ++r) sum[r] = 0.f;
    for (int kb = 0; kb < blocks; ++kb) {
        const uint4 v = common_block(w, kp, col, kb);
        const float d = half_bits(__ldg(sc + static_cast<size_t>(kb) * np + col));
        uint32_t e[8];
        common_unpack(v.x, e[0], e[1]);
        common_unpack(v.y, e[2], e[3]);
        common_unpack(v.z, e[4], e[5]);
        common_unpack(v.w, e[6], e[7]);
#pragma unroll
        for (int r = 0; r < kGemmRowsPerWarp; ++r) {
            if (r0 + r >= m) break;
            const int *a = reinterpret_cast<const int *>(q + static_cast<size_t>(r0 + r) * kp + kb * 32);
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = __dp4a(static_cast<int>(e[i]), __ldg(a + i), dot);
            sum[r] = __fadd_rn(sum[r], __fmul_rn(static_cast<float>(dot), d));
        }
    }
    if (col < n) {
#pragma unroll
        for (int r = 0; r < kGemmRowsPerWarp; ++r)
            if (r0 + r < m)
                y[static_cast<size_t>(r0 + r) * n + col] = __fmul_rn(sum[r], row_scale[static_cast<size_t>(r0 + r) * 16]);
    }
    }
}

int grid_for(int tiles, int warps, const DeviceInfo &dev) {
    const int want = (tiles + warps - 1) / warps;
    return want < dev.sm_count * 8 ? (want < 1 ? 1 : want) : dev.sm_count * 8;
}

}  // namespace

cudaError_t launch_a8x2(const void *x, int k, int dtype, int kq, int8_t *q0, int8_t *q1, float *params,
                        cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(k) * 4;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(a8x2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    a8x2_kernel<<<1, 1024, smem, stream>>>(x, k, dtype, kq, q0, q1, params);
    return cudaGetLastError();
}

cudaError_t launch_row_a8(const void *x, int m, int k, int dtype, int kq, int8_t *q, float *row_scale,
                          int scale_stride, cudaStream_t stream) {
    row_a8_kernel<<<m, 256, 0, stream>>>(x, k, dtype, kq, q, row_scale, scale_stride);
    return cudaGetLastError();
}

cudaError_t launch_native_gemv_a8x2(const uint8_t *w, const uint16_t *scales, const int8_t *q0, const int8_t *q1,
                                    const float *params, int k, int n, float *y, const DeviceInfo &dev,
                                    cudaStream_t stream) {
    const int tiles = (n + 31) / 32;
    native_gemv_a8x2_kernel<<<grid_for(tiles, 8, dev), 256, 2 * static_cast<size_t>(k), stream>>>(w, scales, q0, q1,
                                                                                                  params, k, n, y);
    return cudaGetLastError();
}

cudaError_t launch_native_fallback(const uint8_t *w, const uint16_t *scales, const void *x, int dtype, int k, int n,
                                   int batch, float *y, const DeviceInfo &dev, cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(k) * 4;
    if (smem > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(native_fallback_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int tiles = (n + 31) / 32;
    dim3 grid(grid_for(tiles, 8, dev), batch < 65535 ? batch : 65535);
    native_fallback_kernel<<<grid, 256, smem, stream>>>(w, scales, x, dtype, k, n, batch, y);
    return cudaGetLastError();
}

cudaError_t launch_common_gemv_a8x2(const uint8_t *w, size_t scale_offset, int kp, int np, const int8_t *q0,
                                    const int8_t *q1, const float *params, int k, int n, float *y,
                                    const DeviceInfo &dev, cudaStream_t stream) {
    const size_t smem = 2 * static_cast<size_t>(kp);
    const int tiles = (n + 31) / 32;
    common_gemv_a8x2_kernel<<<grid_for(tiles, 8, dev), 256, smem, stream>>>(w, nullptr, scale_offset, kp, np, q0, q1,
                                                                           params, k, n, y, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_common_gemv_pair(const uint8_t *w0, const uint8_t *w1, size_t scale_offset, int kp, int np,
                                    const int8_t *q0, const int8_t *q1, const float *params, int k, int n, float *y0,
                                    float *y1, const DeviceInfo &dev, cudaStream_t stream) {
    const size_t smem = 2 * static_cast<size_t>(kp);
    const int tiles = (n + 31) / 32;
    common_gemv_a8x2_kernel<<<grid_for(2 * tiles, 8, dev), 256, smem, stream>>>(w0, w1, scale_offset, kp, np, q0, q1,
                                                                               params, k, n, y0, y1);
    return cudaGetLastError();
}

cudaError_t launch_common_gemm_a8(const uint8_t *w, size_t scale_offset, int kp, int np, const int8_t *q,
                                  const float *row_scale, int k, int n, int m, float *y, cudaStream_t stream) {
    const int row_tiles = (m + 31) / 32;
    dim3 grid((n + 31) / 32, row_tiles < 65535 ? row_tiles : 65535);
    common_gemm_a8_kernel<<<grid, 128, 0, stream>>>(w, scale_offset, kp, np, q, row_scale, k, n, m, y);
    return cudaGetLastError();
}

}  // namespace k200
