// Q6_K typed GEMV (sm_100a): Y[c, r] = sum over 16-value groups g of
// dot(w[r, g], q[c, g]) * ascale[c, g / 16] * wscale[r, g], the arithmetic of
// the reference's kunlun-q6-quant / kunlun-q6-onchip kernels (src/q6-k.inc):
//  * activations are quantised per 256-value chunk (symmetric A8): scale =
//    max|x| / 127, q = trunc(x * (127 / max) +- 0.5) clamped to +-127 (0 for
//    an all-zero chunk);
//  * weights are the Q6_K values q - 32 as int8 in the packed layout
//    [N32 tile][K16 group][16 values][32 rows], with one f32 scale
//    d * sub-scale (exact in f32) per row and group at
//    scale_offset + ((tile * groups + g) * 32 + row % 32) * 4;
//  * each group's int8 dot is exact; the FP32 sum runs over groups in order.
//
// The packed layout is produced here too, on the device, from the raw GGML
// blocks the caller uploads (q6_unpack_kernel).
#include <cuda_fp16.h>

#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

constexpr int kQ6RawBytes = 210;    // GGML block_q6_K: ql[128] qh[64] int8 sub-scales[16] fp16 d
constexpr int kQ6RawPitch = 212;    // shared-memory row pitch: 53 words, odd, so 32 rows hit 32 banks

// GGML Q6_K block -> packed int8 values and f32 group scales, for one 32-row
// tile (blockIdx.x) and one 256-value block (blockIdx.y).  The 32 raw rows
// are staged in shared memory with coalesced byte loads; then thread (row =
// t % 32, eighth = t / 32) rebuilds 32 of the 256 values of its row, so
// every warp store covers 32 consecutive output bytes (32 rows of one value).
// Value p of a block: low four bits from byte (p / 128) * 64 + (p / 32 % 2) * 32
// + p % 32 of ql (low nibble for p % 128 < 64, high nibble otherwise), high two
// bits from byte (p / 128) * 32 + p % 32 of qh at bit 2 * (p % 128 / 32); the
// value is that six-bit number minus 32, and its scale is d * sub-scale[p / 16].
// A block whose d is Inf or NaN sets *status (the weight is rejected).
__global__ void __launch_bounds__(256) q6_unpack_kernel(const uint8_t *raw, int k, int n, int8_t *w, float *wscale,
                                                        int *status) {
    __shared__ __align__(16) uint8_t rows[32 * kQ6RawPitch];
    const int tile = blockIdx.x, blk = blockIdx.y, t = threadIdx.x;
    const int blocks_per_row = k / 256, groups = k / 16;
    for (int i = t; i < 32 * kQ6RawBytes; i += 256) {
        const int r = i / kQ6RawBytes, off = i - r * kQ6RawBytes;
        const size_t src = (static_cast<size_t>(tile * 32 + r) * blocks_per_row + blk) * kQ6RawBytes + off;
        rows[r * kQ6RawPitch + off] = raw[src];
    }
    __syncthreads();
    const int r = t & 31, eighth = t >> 5;
    const uint8_t *b = rows + r * kQ6RawPitch;
    const size_t tile_base = static_cast<size_t>(tile) * groups;
    // two sub-scales per thread: eighth and eighth + 8
    const uint16_t dbits = static_cast<uint16_t>(b[208] | (b[209] << 8));
    if (((dbits >> 10) & 31) == 31) atomicOr(status, 1);
    const float d = half_bits_to_float(dbits);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int sub = eighth + 8 * h;
        const float s = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(b[192 + sub])));
        wscale[(tile_base + blk * 16 + sub) * 32 + r] = s;
    }
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        const int p = eighth * 32 + i;
        const int half = p >> 7, quarter = (p >> 5) & 3, l = p & 31;
        const uint8_t lowbyte = b[half * 64 + (quarter & 1) * 32 + l];
        const int low4 = quarter < 2 ? (lowbyte & 15) : (lowbyte >> 4);
        const int high2 = (b[128 + half * 32 + l] >> (2 * quarter)) & 3;
        const int g = blk * 16 + (p >> 4);
        w[((tile_base + g) * 16 + (p & 15)) * 32 + r] = static_cast<int8_t>((low4 | (high2 << 4)) - 32);
    }
}

// One CTA per (256-value chunk, activation row): blockIdx.x chunk, blockIdx.y row.
__global__ void __launch_bounds__(256) q6_quant_kernel(const void *x, int dtype, int k, int8_t *q, float *scales) {
    __shared__ float red[8];
    const int j = threadIdx.x;
    const size_t at = static_cast<size_t>(blockIdx.y) * k + blockIdx.x * 256 + j;
    const float v = dtype ? __half2float(static_cast<const __half *>(x)[at]) : static_cast<const float *>(x)[at];
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
    q[at] = static_cast<int8_t>(z);
    if (j == 0) scales[static_cast<size_t>(blockIdx.y) * (k / 256) + blockIdx.x] = mx > 0.f ? __fdiv_rn(mx, 127.f) : 0.f;
}

// Warp per 32-row tile, lane = row; blockIdx.y selects the activation row,
// whose quantised values and chunk scales are staged in shared memory.
__global__ void __launch_bounds__(256) q6_gemv_kernel(float *y, const int8_t *w, const float *wscale,
                                                      const int8_t *qg, const float *ascale, int k, int n) {
    extern __shared__ __align__(16) int8_t q6s[];  // [k] int8, then [k/256] float
    float *as = reinterpret_cast<float *>(q6s + k);
    const int8_t *qrow = qg + static_cast<size_t>(blockIdx.y) * k;
    const float *arow = ascale + static_cast<size_t>(blockIdx.y) * (k / 256);
    for (int i = threadIdx.x; i < k / 16; i += blockDim.x)
        reinterpret_cast<int4 *>(q6s)[i] = reinterpret_cast<const int4 *>(qrow)[i];
    for (int i = threadIdx.x; i < k / 256; i += blockDim.x) as[i] = arow[i];
    __syncthreads();
    float *yrow = y + static_cast<size_t>(blockIdx.y) * n;
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
        yrow[tile * 32 + lane] = sum;
    }
}

}  // namespace

cudaError_t launch_q6_unpack(const uint8_t *raw, int k, int n, int8_t *w, float *wscale, int *status,
                             cudaStream_t stream) {
    q6_unpack_kernel<<<dim3(n / 32, k / 256), 256, 0, stream>>>(raw, k, n, w, wscale, status);
    return cudaGetLastError();
}

cudaError_t launch_q6_quant(const void *x, int dtype, int k, int m, int8_t *q, float *scales, cudaStream_t stream) {
    q6_quant_kernel<<<dim3(k / 256, m), 256, 0, stream>>>(x, dtype, k, q, scales);
    return cudaGetLastError();
}

cudaError_t launch_q6_gemv(float *y, const int8_t *w, const float *wscale, const int8_t *q, const float *ascale, int k,
                           int n, int m, const DeviceInfo &dev, cudaStream_t stream) {
    const int tiles = n / 32;
    const int want = (tiles + 7) / 8;
    const int grid = want < dev.sm_count * 8 ? (want < 1 ? 1 : want) : dev.sm_count * 8;
    q6_gemv_kernel<<<dim3(grid, m), 256, static_cast<size_t>(k) + 4 * static_cast<size_t>(k / 256), stream>>>(
        y, w, wscale, q, ascale, k, n);
    return cudaGetLastError();
}

}  // namespace k200
