// Quantisers of the k200 matmul path (sm_100a).  Every floating-point step is
// written with explicit round-to-nearest intrinsics (__fmul_rn, __fadd_rn,
// __fdiv_rn) so that no multiply-add is fused and the results are bit-exact
// with the reference's host code.
//
//  * a8 tensor: the rowwise-int8 path's per-tensor two-pass activation
//    quantiser, src/k200.cpp:209-229 of the reference, done on the device
//    (the reference copies X to the host and back on every call);
//  * i8 rows:   upload_i8_rows' per-row weight quantiser, src/k200.cpp:102-123;
//  * q4_0:      GGML's Q4_0 block quantiser (d = v/-8 for the element v of
//    largest magnitude, q = min(15, (int8)(x/d + 8.5))), used to build Q4_0
//    weights on the device.
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

constexpr int kErrNonFinite = 0x4b10;  // the reference aborts on non-finite X or W

// (int)(v + (v >= 0 ? .5f : -.5f)) clamped to [-127, 127]
__device__ __forceinline__ int round_away_127(float v) {
    float t = __fadd_rn(v, v >= 0.f ? 0.5f : -0.5f);
    int q = static_cast<int>(t);  // truncation toward zero, as the C cast
    return q > 127 ? 127 : (q < -127 ? -127 : q);
}

__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

__device__ __forceinline__ uint32_t block_max(uint32_t v, uint32_t *scratch) {
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

// ---- a8 tensor: one CTA for small tensors ---------------------------------
// Three passes over X (max|x|; q0 and max|r|; q1).  With X 16-byte aligned
// and count % 4 == 0 each thread reads float4s eight at a time, so a pass
// costs a few memory latencies rather than one per element.
__device__ __forceinline__ void a8_q0(float v, float inv0, float step0, int &q0, uint32_t &rbits) {
    q0 = round_away_127(__fmul_rn(v, inv0));
    rbits = abs_bits(__fsub_rn(v, __fmul_rn(static_cast<float>(q0), step0)));
}

__global__ void __launch_bounds__(1024) a8_single_kernel(const float *x, size_t count, int8_t *q, float *maxima,
                                                         int *err) {
    __shared__ uint32_t scratch[32];
    const bool vec = (count % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    const size_t count4 = vec ? count / 4 : 0;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    constexpr int U = 8;
    uint32_t m = 0;
    bool bad = false;
    // pass 1: max |x|
    for (size_t j0 = threadIdx.x; j0 < count4; j0 += U * blockDim.x) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t j = j0 + u * blockDim.x;
            v[u] = j < count4 ? __ldg(x4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t a = abs_bits(v[u].x), b = abs_bits(v[u].y), c = abs_bits(v[u].z), d = abs_bits(v[u].w);
            bad |= (a >= 0x7f800000u) | (b >= 0x7f800000u) | (c >= 0x7f800000u) | (d >= 0x7f800000u);
            m = max(m, max(max(a, b), max(c, d)));
        }
    }
    for (size_t j = 4 * count4 + threadIdx.x; j < count; j += blockDim.x) {
        const uint32_t u = abs_bits(x[j]);
        bad |= u >= 0x7f800000u;
        m = max(m, u);
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const uint32_t m0 = block_max(m, scratch);
    const float max0 = m0 ? __uint_as_float(m0) : 1.0f;
    const float inv0 = __fdiv_rn(127.0f, max0), step0 = __fdiv_rn(max0, 127.0f);
    // pass 2: q0 = round(x * 127 / max0), max |x - q0 * max0 / 127|
    m = 0;
    for (size_t j0 = threadIdx.x; j0 < count4; j0 += U * blockDim.x) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t j = j0 + u * blockDim.x;
            v[u] = j < count4 ? __ldg(x4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t j = j0 + u * blockDim.x;
            int a, b, c, d;
            uint32_t ra, rb, rc, rd;
            a8_q0(v[u].x, inv0, step0, a, ra);
            a8_q0(v[u].y, inv0, step0, b, rb);
            a8_q0(v[u].z, inv0, step0, c, rc);
            a8_q0(v[u].w, inv0, step0, d, rd);
            if (j < count4) {
                reinterpret_cast<char4 *>(q)[j] =
                    make_char4(static_cast<signed char>(a), static_cast<signed char>(b), static_cast<signed char>(c),
                               static_cast<signed char>(d));
                m = max(m, max(max(ra, rb), max(rc, rd)));
            }
        }
    }
    for (size_t j = 4 * count4 + threadIdx.x; j < count; j += blockDim.x) {
        int q0;
        uint32_t r;
        a8_q0(x[j], inv0, step0, q0, r);
        q[j] = static_cast<int8_t>(q0);
        m = max(m, r);
    }
    const uint32_t m1 = block_max(m, scratch);
    const float max1 = m1 ? __uint_as_float(m1) : 1.0f;
    const float inv1 = __fdiv_rn(127.0f, max1);
    // pass 3: q1 = round(r * 127 / max1), r recomputed from x and q0
    for (size_t j0 = threadIdx.x; j0 < count4; j0 += U * blockDim.x) {
        float4 v[U];
        char4 c0[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t j = j0 + u * blockDim.x;
            v[u] = j < count4 ? __ldg(x4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            c0[u] = j < count4 ? reinterpret_cast<const char4 *>(q)[j] : make_char4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t j = j0 + u * blockDim.x;
            const float ra = __fsub_rn(v[u].x, __fmul_rn(static_cast<float>(c0[u].x), step0));
            const float rb = __fsub_rn(v[u].y, __fmul_rn(static_cast<float>(c0[u].y), step0));
            const float rc = __fsub_rn(v[u].z, __fmul_rn(static_cast<float>(c0[u].z), step0));
            const float rd = __fsub_rn(v[u].w, __fmul_rn(static_cast<float>(c0[u].w), step0));
            if (j < count4)
                reinterpret_cast<char4 *>(q + count)[j] = make_char4(
                    static_cast<signed char>(round_away_127(__fmul_rn(ra, inv1))),
                    static_cast<signed char>(round_away_127(__fmul_rn(rb, inv1))),
                    static_cast<signed char>(round_away_127(__fmul_rn(rc, inv1))),
                    static_cast<signed char>(round_away_127(__fmul_rn(rd, inv1))));
        }
    }
    for (size_t j = 4 * count4 + threadIdx.x; j < count; j += blockDim.x) {
        const float r = __fsub_rn(x[j], __fmul_rn(static_cast<float>(q[j]), step0));
        q[count + j] = static_cast<int8_t>(round_away_127(__fmul_rn(r, inv1)));
    }
    if (threadIdx.x == 0) {
        maxima[0] = max0;
        maxima[1] = max1;
    }
}

// ---- a8 tensor: three grid-wide passes for large tensors -------------------
// words[0] = max|x| bits, words[1] = max|r| bits, words[2] = non-finite flag
__global__ void a8_max_kernel(const float *x, size_t count, uint32_t *words) {
    __shared__ uint32_t scratch[32];
    uint32_t m = 0, bad = 0;
    for (size_t j = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; j < count;
         j += static_cast<size_t>(gridDim.x) * blockDim.x) {
        uint32_t u = abs_bits(x[j]);
        bad |= u >= 0x7f800000u;
        m = max(m, u);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(&words[2], 1u);
    m = block_max(m, scratch);
    if (threadIdx.x == 0) atomicMax(&words[0], m);
}

__global__ void a8_main_kernel(const float *x, size_t count, int8_t *q, uint32_t *words) {
    __shared__ uint32_t scratch[32];
    const float max0 = words[0] ? __uint_as_float(words[0]) : 1.0f;
    const float inv0 = __fdiv_rn(127.0f, max0), step0 = __fdiv_rn(max0, 127.0f);
    uint32_t m = 0;
    for (size_t j = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; j < count;
         j += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float v = x[j];
        const int q0 = round_away_127(__fmul_rn(v, inv0));
        q[j] = static_cast<int8_t>(q0);
        m = max(m, abs_bits(__fsub_rn(v, __fmul_rn(static_cast<float>(q0), step0))));
    }
    m = block_max(m, scratch);
    if (threadIdx.x == 0) atomicMax(&words[1], m);
}

__global__ void a8_residual_kernel(const float *x, size_t count, int8_t *q, const uint32_t *words, float *maxima,
                                   int *err) {
    if (words[2]) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float max0 = words[0] ? __uint_as_float(words[0]) : 1.0f;
    const float max1 = words[1] ? __uint_as_float(words[1]) : 1.0f;
    const float step0 = __fdiv_rn(max0, 127.0f), inv1 = __fdiv_rn(127.0f, max1);
    for (size_t j = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; j < count;
         j += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float r = __fsub_rn(x[j], __fmul_rn(static_cast<float>(q[j]), step0));
        q[count + j] = static_cast<int8_t>(round_away_127(__fmul_rn(r, inv1)));
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        maxima[0] = max0;
        maxima[1] = max1;
    }
}

// ---- i8 rows -------------------------------------------------------------
__global__ void __launch_bounds__(256) i8_rows_kernel(const float *w, int k, int8_t *q, float *scales, int *err) {
    __shared__ uint32_t scratch[32];
    const int row = blockIdx.x;
    const float *src = w + static_cast<long long>(row) * k;
    uint32_t m = 0;
    bool bad = false;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        uint32_t u = abs_bits(src[j]);
        bad |= u >= 0x7f800000u;
        m = max(m, u);
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    m = block_max(m, scratch);
    const float maximum = __uint_as_float(m);
    const float inv = m ? __fdiv_rn(127.0f, maximum) : 0.0f;
    if (threadIdx.x == 0) scales[row] = m ? __fdiv_rn(maximum, 127.0f) : 1.0f;
    int8_t *dst = q + static_cast<long long>(row) * k;
    for (int j = threadIdx.x; j < k; j += blockDim.x) dst[j] = static_cast<int8_t>(round_away_127(__fmul_rn(src[j], inv)));
}

// ---- q4_0 ----------------------------------------------------------------
__global__ void q4_0_quantize_kernel(const float *w, long long blocks, uint8_t *q4) {
    const long long b = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    if (b >= blocks) return;
    const float4 *src = reinterpret_cast<const float4 *>(w + b * 32);
    float x[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float4 t = src[i];
        x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
    }
    float amax = 0.f, vmax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(x[j]);
        if (amax < a) { amax = a; vmax = x[j]; }
    }
    const float d = __fdiv_rn(vmax, -8.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint8_t out[18];
    const uint16_t hd = __half_as_ushort(__float2half_rn(d));
    out[0] = static_cast<uint8_t>(hd & 255u);
    out[1] = static_cast<uint8_t>(hd >> 8);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        int xi0 = static_cast<int8_t>(static_cast<int>(__fadd_rn(__fmul_rn(x[j], id), 8.5f)));
        int xi1 = static_cast<int8_t>(static_cast<int>(__fadd_rn(__fmul_rn(x[16 + j], id), 8.5f)));
        xi0 = xi0 > 15 ? 15 : xi0;
        xi1 = xi1 > 15 ? 15 : xi1;
        out[2 + j] = static_cast<uint8_t>(xi0 | (xi1 << 4));
    }
    uint8_t *dst = q4 + b * 18;
#pragma unroll
    for (int j = 0; j < 18; ++j) dst[j] = out[j];
}

}  // namespace

size_t a8_tensor_scratch_bytes(size_t) { return 64; }

cudaError_t launch_a8_tensor(const float *x, size_t count, int8_t *q, float *maxima, void *scratch,
                             const DeviceInfo &dev, cudaStream_t stream) {
    if (count <= 65536) {
        a8_single_kernel<<<1, 1024, 0, stream>>>(x, count, q, maxima, dev.err);
        return cudaGetLastError();
    }
    uint32_t *words = static_cast<uint32_t *>(scratch);
    cudaError_t e = cudaMemsetAsync(words, 0, 16, stream);
    if (e != cudaSuccess) return e;
    const int threads = 512;
    long long want = static_cast<long long>((count + threads * 8 - 1) / (threads * 8));
    const int grid = static_cast<int>(want < dev.sm_count * 4 ? (want < 1 ? 1 : want) : dev.sm_count * 4);
    a8_max_kernel<<<grid, threads, 0, stream>>>(x, count, words);
    a8_main_kernel<<<grid, threads, 0, stream>>>(x, count, q, words);
    a8_residual_kernel<<<grid, threads, 0, stream>>>(x, count, q, words, maxima, dev.err);
    return cudaGetLastError();
}

cudaError_t launch_i8_rows(const float *w, int k, int rows, int8_t *q, float *scales, const DeviceInfo &dev,
                           cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    i8_rows_kernel<<<rows, 256, 0, stream>>>(w, k, q, scales, dev.err);
    return cudaGetLastError();
}

cudaError_t launch_q4_0_quantize(const float *w, int n, int k, uint8_t *q4, cudaStream_t stream) {
    const long long blocks = static_cast<long long>(n) * (k / 32);
    if (blocks <= 0) return cudaSuccess;
    const int threads = 256;
    q4_0_quantize_kernel<<<static_cast<unsigned>((blocks + threads - 1) / threads), threads, 0, stream>>>(w, blocks,
                                                                                                         q4);
    return cudaGetLastError();
}

}  // namespace k200
