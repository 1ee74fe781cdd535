// Streaming matrix-vector kernels for the k200 matmul path (sm_100a).
//
// Y[c, r] = sum_j W[r, j] * X[c, j] for a few activation columns c, where W is
// stored row-major in one of the legacy kunlun::WeightType encodings:
//   f32   4 bytes/element                       (WeightType::f32  = 0)
//   f16   2 bytes/element, IEEE binary16          (WeightType::f16  = 1)
//   q4_0  18-byte blocks: fp16 d, 16 nibble bytes (WeightType::q4_0 = 2)
//   i8    int8 rows + per-row f32 scale           (WeightType::rowwise_i8 = 3)
// The arithmetic follows kernels/kunlun-matvec.xpu:37-77 of the reference
// (decoded weight times f32 activation, f32 accumulation) for f32/f16/q4_0,
// and the exact int32 dot + combine of src/k200.cpp:231-232 and
// kernels/kunlun-combine.xpu:19 for rowwise_i8.
//
// Design (one persistent CTA per SM):
//  * every CTA owns a contiguous range of output rows, i.e. one contiguous
//    range of weight bytes; a single thread streams it through an S-stage ring
//    of shared-memory chunks with 1-D bulk copies (cp.async.bulk + mbarrier),
//    so each weight byte crosses HBM exactly once, fully coalesced;
//  * each thread owns a fixed K-segment (64 elements for q4_0/f16/i8, 32 for
//    f32) and keeps the matching activation values in registers for the whole
//    CTA, so X is read once per CTA and never again;
//  * a row is reduced across the threads of its "row slot" with warp shuffles,
//    then across warps through shared memory in a fixed order (results are
//    bitwise reproducible run to run);
//  * q4_0 nibbles are turned into exact floats with one PRMT each
//    (0x4B0000vv = 2^23 + v) and one packed f32x2 subtract of 2^23 + 8, and
//    multiplied with packed f32x2 FMAs.
#include <cstdint>
#include <cstdio>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

// Threads per CTA: 512 when the activation registers of a segment fit in
// 64 registers, 256 otherwise (keeps the CTA inside the 64K register file).
template <int WT, int B>
constexpr int max_threads() {
    return ((WT == 0 || WT == 3) ? 32 * B : 64 * B) <= 64 ? 512 : 256;
}

struct GemvArgs {
    const uint8_t *w;
    const float *x;          // f32 activations [batch][x_stride]            (types 0..2)
    const int8_t *q;         // int8 activations [2][batch][q_stride]        (type 3)
    const float *act_max;    // {max0, max1} of the quantised activations   (type 3)
    const float *row_scale;  // per-row f32 scales [n]                       (type 3)
    float *y;
    long long row_bytes;
    int k, n, batch;
    int x_stride, q_stride, y_stride;
    int rows_per_cta, chunk_rows, tpr, slots, stages;
    uint32_t chunk_bytes;
    long long q_comp;        // elements between the two int8 components (type 3)
    int *err;
};

template <int WT>
struct Seg;  // activation elements owned by one thread (its segment of K)
template <> struct Seg<0> { static constexpr int elems = 32; };  // 128 bytes of a row
template <> struct Seg<1> { static constexpr int elems = 64; };  // 128 bytes
template <> struct Seg<2> { static constexpr int elems = 64; };  // 36 bytes (two blocks)
template <> struct Seg<3> { static constexpr int elems = 64; };  // 64 bytes

// ---------------------------------------------------------------------------
// per-segment arithmetic
// ---------------------------------------------------------------------------
// Builds two exact floats (v0 - 8, v1 - 8) from nibble bytes of `nib`.
__device__ __forceinline__ unsigned long long q4_pair(uint32_t nib, uint32_t sel0, uint32_t sel1) {
    constexpr unsigned long long kNegMagic = 0xCB000008CB000008ull;  // -(2^23 + 8) twice
    uint32_t a = __byte_perm(nib, 0x4B000000u, sel0);
    uint32_t b = __byte_perm(nib, 0x4B000000u, sel1);
    unsigned long long v = (static_cast<unsigned long long>(b) << 32) | a;
    return f2_add(v, kNegMagic);
}

// One Q4_0 block: 4 data words (byte j = element j low nibble, element j+16
// high nibble) against 16 packed activation pairs per column.
template <int B>
__device__ __forceinline__ void q4_block(const uint32_t (&dw)[4], float d, const unsigned long long (*xp)[16],
                                         float (&acc)[B]) {
    unsigned long long s[B][2];
#pragma unroll
    for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t lo = dw[j] & 0x0F0F0F0Fu;
        uint32_t hi = (dw[j] >> 4) & 0x0F0F0F0Fu;
        // elements 4j..4j+3 (low nibbles) and 16+4j..16+4j+3 (high nibbles)
        unsigned long long l01 = q4_pair(lo, 0x7440, 0x7441), l23 = q4_pair(lo, 0x7442, 0x7443);
        unsigned long long h01 = q4_pair(hi, 0x7440, 0x7441), h23 = q4_pair(hi, 0x7442, 0x7443);
#pragma unroll
        for (int c = 0; c < B; ++c) {
            s[c][0] = f2_fma(l01, xp[c][2 * j], s[c][0]);
            s[c][1] = f2_fma(l23, xp[c][2 * j + 1], s[c][1]);
            s[c][0] = f2_fma(h01, xp[c][8 + 2 * j], s[c][0]);
            s[c][1] = f2_fma(h23, xp[c][8 + 2 * j + 1], s[c][1]);
        }
    }
#pragma unroll
    for (int c = 0; c < B; ++c) {
        unsigned long long t = f2_add(s[c][0], s[c][1]);
        float blk = f2_lo(t) + f2_hi(t);
        acc[c] = fmaf(d, blk, acc[c]);
    }
}

// Thread-resident activation registers for one segment.
template <int WT, int B>
struct XRegs;

template <int B>
struct XRegs<2, B> {  // q4_0: two blocks of 32 activations, as f32 pairs
    unsigned long long v[2][B][16];
};
template <int B>
struct XRegs<1, B> {  // f16: 64 activations as f32 pairs
    unsigned long long v[B][32];
};
template <int B>
struct XRegs<0, B> {  // f32: 32 activations as f32 pairs
    unsigned long long v[B][16];
};
template <int B>
struct XRegs<3, B> {  // i8: 64 activations per component, packed 4 per word
    uint32_t v[2][B][16];
};

template <int WT, int B>
__device__ __forceinline__ void load_x(XRegs<WT, B> &xr, const GemvArgs &a, int seg) {
    const int e0 = seg * Seg<WT>::elems;
    if constexpr (WT == 3) {
#pragma unroll
        for (int comp = 0; comp < 2; ++comp)
#pragma unroll
            for (int c = 0; c < B; ++c) {
                const int8_t *src = a.q + comp * a.q_comp + static_cast<long long>(c) * a.q_stride + e0;
                bool col = c < a.batch;
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    int4 t = make_int4(0, 0, 0, 0);
                    if (col && e0 + 16 * v < a.k) t = __ldg(reinterpret_cast<const int4 *>(src) + v);
                    xr.v[comp][c][4 * v + 0] = static_cast<uint32_t>(t.x);
                    xr.v[comp][c][4 * v + 1] = static_cast<uint32_t>(t.y);
                    xr.v[comp][c][4 * v + 2] = static_cast<uint32_t>(t.z);
                    xr.v[comp][c][4 * v + 3] = static_cast<uint32_t>(t.w);
                }
            }
    } else {
        constexpr int P = Seg<WT>::elems / 2;  // pairs per segment
#pragma unroll
        for (int c = 0; c < B; ++c) {
            const float *src = a.x + static_cast<long long>(c) * a.x_stride + e0;
            bool col = c < a.batch;
#pragma unroll
            for (int v = 0; v < P / 2; ++v) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (col && e0 + 4 * v < a.k) t = __ldg(reinterpret_cast<const float4 *>(src) + v);
                unsigned long long p0 = f2_pack(t.x, t.y), p1 = f2_pack(t.z, t.w);
                if constexpr (WT == 2) {
                    xr.v[(2 * v) / 16][c][(2 * v) % 16] = p0;
                    xr.v[(2 * v + 1) / 16][c][(2 * v + 1) % 16] = p1;
                } else {
                    xr.v[c][2 * v] = p0;
                    xr.v[c][2 * v + 1] = p1;
                }
            }
        }
    }
}

// Partial result of one row for one thread: float sums (types 0..2) or the
// two exact int32 component dots (type 3).
template <int WT, int B>
struct Partial {
    float f[B];
};
template <int B>
struct Partial<3, B> {
    int d0[B], d1[B];
};

template <int WT, int B>
__device__ __forceinline__ void segment_dot(Partial<WT, B> &out, const uint8_t *row, int seg, int k,
                                            const XRegs<WT, B> &xr) {
    const int e0 = seg * Seg<WT>::elems;
    if constexpr (WT == 2) {
#pragma unroll
        for (int c = 0; c < B; ++c) out.f[c] = 0.f;
        const uint32_t *p = reinterpret_cast<const uint32_t *>(row + 36 * seg);
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = p[i];
        // block 2*seg: scale in bytes 0..1, data in bytes 2..17 (2-byte offset)
        uint32_t d0[4] = {__funnelshift_r(w[0], w[1], 16), __funnelshift_r(w[1], w[2], 16),
                          __funnelshift_r(w[2], w[3], 16), __funnelshift_r(w[3], w[4], 16)};
        q4_block<B>(d0, half_bits_to_float(static_cast<uint16_t>(w[0] & 0xffffu)), xr.v[0], out.f);
        if (e0 + 32 < k) {
            // block 2*seg+1: scale in bytes 18..19, data in bytes 20..35
            uint32_t d1[4] = {w[5], w[6], w[7], w[8]};
            q4_block<B>(d1, half_bits_to_float(static_cast<uint16_t>(w[4] >> 16)), xr.v[1], out.f);
        }
    } else if constexpr (WT == 1) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + 128 * seg);
        unsigned long long s[B][2];
#pragma unroll
        for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
        const int vmax = (e0 + 32 < k) ? 8 : 4;  // K % 64 == 32: upper half lies past the row
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            if (v >= vmax) break;
            uint4 t = p[v];
            uint32_t h[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[i]));
                unsigned long long wp = f2_pack(f.x, f.y);
#pragma unroll
                for (int c = 0; c < B; ++c) s[c][i & 1] = f2_fma(wp, xr.v[c][4 * v + i], s[c][i & 1]);
            }
        }
#pragma unroll
        for (int c = 0; c < B; ++c) {
            unsigned long long t = f2_add(s[c][0], s[c][1]);
            out.f[c] = f2_lo(t) + f2_hi(t);
        }
    } else if constexpr (WT == 0) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + 128 * seg);
        unsigned long long s[B][2];
#pragma unroll
        for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            uint4 t = p[v];
            unsigned long long w0 = (static_cast<unsigned long long>(t.y) << 32) | t.x;
            unsigned long long w1 = (static_cast<unsigned long long>(t.w) << 32) | t.z;
#pragma unroll
            for (int c = 0; c < B; ++c) {
                s[c][0] = f2_fma(w0, xr.v[c][2 * v], s[c][0]);
                s[c][1] = f2_fma(w1, xr.v[c][2 * v + 1], s[c][1]);
            }
        }
#pragma unroll
        for (int c = 0; c < B; ++c) {
            unsigned long long t = f2_add(s[c][0], s[c][1]);
            out.f[c] = f2_lo(t) + f2_hi(t);
        }
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + 64 * seg);
#pragma unroll
        for (int c = 0; c < B; ++c) out.d0[c] = out.d1[c] = 0;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint4 t = p[v];
            uint32_t wv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < B; ++c) {
                    out.d0[c] = __dp4a(static_cast<int>(wv[i]), static_cast<int>(xr.v[0][c][4 * v + i]), out.d0[c]);
                    out.d1[c] = __dp4a(static_cast<int>(wv[i]), static_cast<int>(xr.v[1][c][4 * v + i]), out.d1[c]);
                }
        }
    }
    (void)k;
}

// Reduction of a partial across `width` lanes (power of two <= 32).
template <int WT, int B>
__device__ __forceinline__ void reduce_lanes(Partial<WT, B> &p, int width) {
    for (int o = width >> 1; o > 0; o >>= 1) {
#pragma unroll
        for (int c = 0; c < B; ++c) {
            if constexpr (WT == 3) {
                p.d0[c] += __shfl_xor_sync(0xffffffffu, p.d0[c], o);
                p.d1[c] += __shfl_xor_sync(0xffffffffu, p.d1[c], o);
            } else {
                p.f[c] += __shfl_xor_sync(0xffffffffu, p.f[c], o);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// the streaming kernel
// ---------------------------------------------------------------------------
template <int WT, int B>
__global__ void __launch_bounds__(max_threads<WT, B>(), 1) gemv_stream_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int row_begin = blockIdx.x * a.rows_per_cta;
    const int row_end = min(a.n, row_begin + a.rows_per_cta);
    if (row_begin >= row_end) return;
    const int nchunks = (row_end - row_begin + a.chunk_rows - 1) / a.chunk_rows;

    // shared memory: [stages][chunk_bytes] ring | mbarriers | reduction buffer
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + static_cast<size_t>(a.stages) * a.chunk_bytes);
    const int wps = a.tpr >= 32 ? a.tpr / 32 : 1;  // partial writers per row slot
    using P = Partial<WT, B>;
    P *red = reinterpret_cast<P *>(full + a.stages);  // [2][chunk_rows][wps]

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    const uint64_t policy = policy_evict_first();
    auto issue = [&](int c) {
        const int r0 = row_begin + c * a.chunk_rows;
        const int rows = min(a.chunk_rows, row_end - r0);
        const uint32_t bytes = static_cast<uint32_t>(rows * a.row_bytes);
        uint64_t *bar = &full[c % a.stages];
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s_stream(ring + static_cast<size_t>(c % a.stages) * a.chunk_bytes, a.w + r0 * a.row_bytes,
                        bytes, bar, policy);
    };
    if (tid == 0)
        for (int c = 0; c < min(a.stages, nchunks); ++c) issue(c);

    const int slot = tid / a.tpr;
    const int seg = tid % a.tpr;
    const int nseg = (a.k + Seg<WT>::elems - 1) / Seg<WT>::elems;
    const bool active = slot < a.slots;
    const bool has_seg = active && seg < nseg;
    const int lane_width = a.tpr >= 32 ? 32 : a.tpr;

    XRegs<WT, B> xr;
    if (has_seg) load_x<WT, B>(xr, a, seg);

    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
        const int stage = c % a.stages;
        const uint32_t parity = (c / a.stages) & 1;
        const int r0 = row_begin + c * a.chunk_rows;
        const int rows = min(a.chunk_rows, row_end - r0);
        if (!mbar_wait(&full[stage], parity, a.err, kErrBulkTimeout)) ok = false;
        const uint8_t *chunk = ring + static_cast<size_t>(stage) * a.chunk_bytes;
        P *rb = red + (c & 1) * a.chunk_rows * wps;
        // warp-uniform trip count: every lane takes part in the shuffles
        for (int i0 = 0; i0 < rows; i0 += a.slots) {
            const int i = i0 + slot;
            const bool live = ok && active && i < rows;
            P part;
            if (live && has_seg) {
                segment_dot<WT, B>(part, chunk + static_cast<size_t>(i) * a.row_bytes, seg, a.k, xr);
            } else {
#pragma unroll
                for (int cc = 0; cc < B; ++cc) {
                    if constexpr (WT == 3) { part.d0[cc] = part.d1[cc] = 0; }
                    else { part.f[cc] = 0.f; }
                }
            }
            reduce_lanes<WT, B>(part, lane_width);
            if (live && (seg & (lane_width - 1)) == 0) rb[i * wps + seg / 32] = part;
        }
        if (__syncthreads_or(!ok)) { ok = false; break; }
        // the stage is free again: refill it while the partials are combined
        if (tid == 0 && c + a.stages < nchunks) issue(c + a.stages);
        if (tid < rows * B) {
            const int i = tid / B, cc = tid % B;
            if (cc < a.batch) {
                const P *src = rb + i * wps;
                float result;
                if constexpr (WT == 3) {
                    int s0 = 0, s1 = 0;
                    for (int wv = 0; wv < wps; ++wv) { s0 += src[wv].d0[cc]; s1 += src[wv].d1[cc]; }
                    const float scale0 = __fdiv_rn(a.act_max[0], 127.0f);
                    const float scale1 = __fdiv_rn(a.act_max[1], 127.0f);
                    float t0 = __fmul_rn(static_cast<float>(s0), scale0);
                    float t1 = __fmul_rn(static_cast<float>(s1), scale1);
                    result = __fmul_rn(__fadd_rn(t0, t1), a.row_scale[r0 + i]);
                } else {
                    float s = 0.f;
                    for (int wv = 0; wv < wps; ++wv) s += src[wv].f[cc];
                    result = s;
                }
                a.y[static_cast<long long>(cc) * a.y_stride + r0 + i] = result;
            }
        }
    }
    // drain: never leave a bulk copy in flight into shared memory of an exited CTA
    if (!ok && tid == 0) {
        // bounded: wait for outstanding copies of each stage's latest phase
        for (int s2 = 0; s2 < min(a.stages, nchunks); ++s2)
            for (uint32_t t = 0; t < kWaitBudget; ++t)
                if (mbar_try_wait(&full[s2], 0) || mbar_try_wait(&full[s2], 1)) break;
    }
}

// ---------------------------------------------------------------------------
// generic fallback: any alignment, any K%32 == 0 (one warp per row and column)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t ldb(const uint8_t *p) { return __ldg(p); }

__global__ void gemv_generic_kernel(const uint8_t *w, int wt, const float *x, float *y, int k, int n, int batch,
                                    long long row_bytes, int x_stride, int y_stride) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (warp >= n * batch) return;
    const int r = warp % n, c = warp / n;
    const uint8_t *row = w + r * row_bytes;
    const float *xv = x + static_cast<long long>(c) * x_stride;
    float sum = 0.f;
    for (int j = lane; j < k; j += 32) {
        float wv;
        if (wt == 0) {
            uint32_t b = ldb(row + 4 * j) | (ldb(row + 4 * j + 1) << 8) | (ldb(row + 4 * j + 2) << 16) |
                         (static_cast<uint32_t>(ldb(row + 4 * j + 3)) << 24);
            wv = __uint_as_float(b);
        } else if (wt == 1) {
            wv = half_bits_to_float(static_cast<uint16_t>(ldb(row + 2 * j) | (ldb(row + 2 * j + 1) << 8)));
        } else {
            const uint8_t *blk = row + (j / 32) * 18;
            float d = half_bits_to_float(static_cast<uint16_t>(ldb(blk) | (ldb(blk + 1) << 8)));
            int e = j % 32;
            int nib = (ldb(blk + 2 + (e % 16)) >> (e < 16 ? 0 : 4)) & 15;
            wv = static_cast<float>(nib - 8) * d;
        }
        sum = fmaf(wv, xv[j], sum);
    }
    sum = warp_sum(sum);
    if (lane == 0) y[static_cast<long long>(c) * y_stride + r] = sum;
}

__global__ void gemv_i8_generic_kernel(const int8_t *w, const int8_t *q, long long q_comp, const float *act_max,
                                       const float *scale, float *y, int k, int n, int batch, int q_stride,
                                       int y_stride) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (warp >= n * batch) return;
    const int r = warp % n, c = warp / n;
    const int8_t *row = w + static_cast<long long>(r) * k;
    const int8_t *q0 = q + static_cast<long long>(c) * q_stride;
    const int8_t *q1 = q + q_comp + static_cast<long long>(c) * q_stride;
    int s0 = 0, s1 = 0;
    for (int j = lane; j < k; j += 32) {
        s0 += static_cast<int>(row[j]) * q0[j];
        s1 += static_cast<int>(row[j]) * q1[j];
    }
    s0 = warp_sum_int(s0);
    s1 = warp_sum_int(s1);
    if (lane == 0) {
        const float scale0 = __fdiv_rn(act_max[0], 127.0f), scale1 = __fdiv_rn(act_max[1], 127.0f);
        float t0 = __fmul_rn(static_cast<float>(s0), scale0);
        float t1 = __fmul_rn(static_cast<float>(s1), scale1);
        y[static_cast<long long>(c) * y_stride + r] = __fmul_rn(__fadd_rn(t0, t1), scale[r]);
    }
}

// ---------------------------------------------------------------------------
// launch planning
// ---------------------------------------------------------------------------
template <int WT>
constexpr int seg_elems() { return Seg<WT>::elems; }

struct Plan {
    int tpr, slots, chunk_rows, stages, threads, grid, rows_per_cta;
    uint32_t chunk_bytes;
    size_t smem;
};

template <int WT, int B>
bool make_plan(Plan &p, int k, int n, long long row_bytes, const DeviceInfo &dev) {
    const int nseg = (k + Seg<WT>::elems - 1) / Seg<WT>::elems;
    if (nseg <= 32) {
        p.tpr = 1;
        while (p.tpr < nseg) p.tpr <<= 1;
    } else {
        p.tpr = (nseg + 31) / 32 * 32;
    }
    constexpr int kThreads = max_threads<WT, B>();
    if (p.tpr > kThreads) return false;
    p.slots = kThreads / p.tpr;
    // chunk: a whole number of rows, about 24 KB, at least one row per slot
    int rows = static_cast<int>((24 * 1024) / row_bytes);
    if (rows < 1) rows = 1;
    if (rows > 64) rows = 64;
    p.grid = dev.sm_count;
    p.rows_per_cta = (n + p.grid - 1) / p.grid;
    if (p.rows_per_cta < 1) p.rows_per_cta = 1;
    if (rows > p.rows_per_cta) rows = p.rows_per_cta;
    if (p.slots > rows) p.slots = rows;
    p.chunk_rows = rows;
    p.chunk_bytes = static_cast<uint32_t>(rows * row_bytes);
    p.threads = p.tpr * p.slots;
    if (p.threads < 32) p.threads = 32;
    const int wps = p.tpr >= 32 ? p.tpr / 32 : 1;
    const size_t red = 2 * static_cast<size_t>(rows) * wps * sizeof(Partial<WT, B>);
    const size_t budget = static_cast<size_t>(dev.smem_optin) - 1024;
    int stages = 6;
    while (stages > 2 && stages * static_cast<size_t>(p.chunk_bytes) + 8 * stages + red > budget) --stages;
    if (stages * static_cast<size_t>(p.chunk_bytes) + 8 * stages + red > budget) return false;
    p.stages = stages;
    p.smem = stages * static_cast<size_t>(p.chunk_bytes) + 8 * stages + red;
    p.grid = (n + p.rows_per_cta - 1) / p.rows_per_cta;
    return true;
}

template <int WT, int B>
cudaError_t launch_stream(const GemvArgs &base, const Plan &p, cudaStream_t stream) {
    GemvArgs a = base;
    a.rows_per_cta = p.rows_per_cta;
    a.chunk_rows = p.chunk_rows;
    a.tpr = p.tpr;
    a.slots = p.slots;
    a.stages = p.stages;
    a.chunk_bytes = p.chunk_bytes;
    auto kern = gemv_stream_kernel<WT, B>;
    static int configured[64] = {0};  // largest dynamic smem already granted, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || configured[dev] < static_cast<int>(p.smem)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(p.smem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = static_cast<int>(p.smem);
    }
    kern<<<p.grid, p.threads, p.smem, stream>>>(a);
    return cudaGetLastError();
}

template <int WT>
cudaError_t launch_batch_group(const GemvArgs &a, const DeviceInfo &dev, cudaStream_t stream, int bgroup) {
    Plan p;
    if (bgroup == 1) {
        if (!make_plan<WT, 1>(p, a.k, a.n, a.row_bytes, dev)) return cudaErrorInvalidConfiguration;
        return launch_stream<WT, 1>(a, p, stream);
    }
    if (!make_plan<WT, 2>(p, a.k, a.n, a.row_bytes, dev)) return cudaErrorInvalidConfiguration;
    return launch_stream<WT, 2>(a, p, stream);
}

}  // namespace

bool gemv_fast_path_ok(int wt, const void *w, const void *x, const void *y, int k, long long row_bytes) {
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (row_bytes & 15)) return false;
    if (wt != 3 && (reinterpret_cast<uintptr_t>(x) & 15)) return false;
    if (wt != 3 && (k % 4)) return false;
    (void)y;
    return true;
}

cudaError_t launch_gemv(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    const long long row_bytes = r.wt == 0 ? 4ll * r.k : r.wt == 1 ? 2ll * r.k : r.wt == 2 ? 18ll * (r.k / 32) : r.k;
    const bool fast = gemv_fast_path_ok(r.wt, r.w, r.x, r.y, r.k, row_bytes);
    for (int c0 = 0; c0 < r.batch; c0 += 2) {
        const int cols = r.batch - c0 < 2 ? r.batch - c0 : 2;
        if (!fast) {
            const int warps = r.n * cols;
            const int threads = 256;
            const int blocks = (warps * 32 + threads - 1) / threads;
            if (r.wt == 3) {
                gemv_i8_generic_kernel<<<blocks, threads, 0, stream>>>(
                    static_cast<const int8_t *>(r.w), r.q + static_cast<long long>(c0) * r.q_stride, r.q_comp,
                    r.act_max, r.row_scale, r.y + static_cast<long long>(c0) * r.y_stride, r.k, r.n, cols,
                    r.q_stride, r.y_stride);
            } else {
                gemv_generic_kernel<<<blocks, threads, 0, stream>>>(
                    static_cast<const uint8_t *>(r.w), r.wt, r.x + static_cast<long long>(c0) * r.x_stride,
                    r.y + static_cast<long long>(c0) * r.y_stride, r.k, r.n, cols, row_bytes, r.x_stride,
                    r.y_stride);
            }
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return e;
            continue;
        }
        GemvArgs a{};
        a.w = static_cast<const uint8_t *>(r.w);
        a.x = r.x ? r.x + static_cast<long long>(c0) * r.x_stride : nullptr;
        a.q = r.q ? r.q + static_cast<long long>(c0) * r.q_stride : nullptr;
        a.act_max = r.act_max;
        a.row_scale = r.row_scale;
        a.y = r.y + static_cast<long long>(c0) * r.y_stride;
        a.row_bytes = row_bytes;
        a.k = r.k;
        a.n = r.n;
        a.batch = cols;
        a.x_stride = r.x_stride;
        a.q_stride = r.q_stride;
        a.y_stride = r.y_stride;
        a.q_comp = r.q_comp;
        a.err = dev.err;
        cudaError_t e;
        switch (r.wt) {
            case 0: e = launch_batch_group<0>(a, dev, stream, cols); break;
            case 1: e = launch_batch_group<1>(a, dev, stream, cols); break;
            case 2: e = launch_batch_group<2>(a, dev, stream, cols); break;
            default: e = launch_batch_group<3>(a, dev, stream, cols); break;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace k200
