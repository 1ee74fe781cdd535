// Streaming matrix-vector kernels for the k200 matmul path (sm_100a).
//
// Y[c, r] = sum_j W[r, j] * X[c, j] for a few activation columns c, where W is
// stored row-major in one of the legacy kunlun::WeightType encodings:
//   f32   4 bytes/element                       (WeightType::f32  = 0)
//   f16   2 bytes/element, IEEE binary16          (WeightType::f16  = 1)
//   q4_0  18-byte blocks: fp16 d, 16 nibble bytes (WeightType::q4_0 = 2)
//   i8    int8 rows + per-row f32 scale           (WeightType::rowwise_i8 = 3)
// The arithmetic follows kernels/kunlun-matvec.xpu:37-77 of the reference
// (exactly decoded weight times f32 activation, f32 accumulation) for
// f32/f16/q4_0, and the exact int32 dot + combine of src/k200.cpp:231-232 and
// kernels/kunlun-combine.xpu:19 for rowwise_i8.
//
// Design (one persistent CTA per SM, warp-specialised):
//  * every CTA owns a contiguous range of output rows, i.e. one contiguous
//    range of weight bytes.  A producer warp streams it through an S-stage
//    ring of shared-memory chunks (whole rows) with 1-D bulk copies
//    (cp.async.bulk + mbarrier "full"), refilling a stage as soon as the row
//    slot that owns it has released it (mbarrier "empty").  Each weight byte
//    crosses HBM exactly once, fully coalesced, with no CTA-wide barrier;
//  * each consumer thread owns a fixed K-segment (64 elements for
//    q4_0/f16/i8, 32 for f32) and keeps the matching activations in
//    registers for the whole CTA, so X is read once per CTA; f32/f16/int8
//    segments are 16-byte vectors interleaved across lanes (conflict-free
//    shared-memory reads), q4_0 segments are two consecutive 18-byte blocks
//    (a 36-byte stride, also conflict-free);
//  * a row slot processes whole chunks of rows, two rows at a time
//    (instruction-level parallelism); each row is reduced across the slot's
//    lanes with shuffles and across its warps through shared memory behind
//    one named barrier per chunk, summing in fixed warp order, so results are
//    bitwise reproducible run to run;
//  * q4_0 nibbles become exact floats without byte shuffles: a nibble at bit
//    offset s <= 16 of a data word is OR-ed into the bits of 2^23, giving
//    2^23 + v*2^s exactly; one packed f32x2 add of -(2^23 + 8*2^s) leaves
//    (v-8)*2^s, and the activation registers hold x*2^-s, so the f32x2 FMA
//    forms the same product (v-8)*x as the reference.  (Activations below
//    2^-106 in magnitude lose precision to this pre-scaling.)
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

struct GemvArgs {
    const uint8_t *w;
    const float *x;          // f32 activations [batch][x_stride]            (types 0..2)
    const int8_t *q;         // int8 activations: component c of column j at q + c*q_comp + j*q_stride
    const float *act_max;    // {max0, max1} of the quantised activations   (type 3)
    const float *row_scale;  // per-row f32 scales [n]                       (type 3)
    float *y;
    long long row_bytes;
    long long q_comp;
    int k, n, batch;
    int x_stride, q_stride, y_stride;
    int rows_per_cta, chunk_rows, tpr, slots, stages, consumers;
    int prefetch;            // chunks the producer may load before the previous kernel completes
    uint32_t chunk_bytes;
    int *err;
};

template <int WT>
struct Seg;  // activation elements owned by one thread (its segment of K)
template <> struct Seg<0> { static constexpr int elems = 32; };  // 128 bytes of a row
template <> struct Seg<1> { static constexpr int elems = 64; };  // 128 bytes
template <> struct Seg<2> { static constexpr int elems = 64; };  // 36 bytes (two blocks)
template <> struct Seg<3> { static constexpr int elems = 64; };  // 64 bytes

// f32 / f16 / int8 rows are read as 16-byte vectors.  Thread `seg` of a row
// slot owns V vectors, interleaved across the lanes of its warp so that a
// warp-wide 16-byte shared-memory load touches 512 consecutive bytes (no bank
// conflicts): vector v of the thread is  ((seg / lw) * V + v) * lw + seg % lw,
// lw = min(32, threads per row).
template <int WT>
struct Vec { static constexpr int per_thread = 8, elems = 4; };   // f32: 8 x 4
template <> struct Vec<1> { static constexpr int per_thread = 8, elems = 8; };   // f16: 8 x 8
template <> struct Vec<3> { static constexpr int per_thread = 4, elems = 16; };  // int8: 4 x 16
__device__ __forceinline__ int vec_index(int seg, int lw, int per_thread, int v) {
    return ((seg / lw) * per_thread + v) * lw + seg % lw;
}

// Rows in flight per thread (1 or 2) and consumer threads per CTA, chosen so
// the activation registers, two rows of weight words and the accumulators fit
// the register file with one CTA per SM.
template <int WT, int B>
struct Shape {
    static constexpr int xregs = (WT == 0 || WT == 3) ? 32 * B : 64 * B;
    static constexpr int consumers = xregs <= 64 ? 448 : 256;
    static constexpr int threads = consumers + 32;  // + one producer warp
    // registers per thread that still fit one CTA in the 64K register file
    static constexpr int maxreg = (65536 / threads) / 8 * 8 > 255 ? 255 : (65536 / threads) / 8 * 8;
};

// ---------------------------------------------------------------------------
// activation registers
// ---------------------------------------------------------------------------
// Q4_0: bit offset s of element e (0..31) of a block inside its 32-bit data
// word after q4_word's extraction (see there); the activation is held as x*2^-s.
__host__ __device__ constexpr int q4_shift(int e) {
    return e < 16 ? ((e & 3) == 0 ? 0 : (e & 3) == 1 ? 8 : (e & 3) == 2 ? 16 : 12)
                  : ((e & 3) == 0 ? 4 : (e & 3) == 1 ? 12 : (e & 3) == 2 ? 8 : 16);
}
__device__ __forceinline__ float pow2_neg(int s) { return __uint_as_float(static_cast<uint32_t>(127 - s) << 23); }

template <int WT, int B>
struct XRegs;
template <int B>
struct XRegs<2, B> {  // q4_0: two blocks of 32 pre-scaled activations, as f32 pairs
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
__device__ __forceinline__ void load_x(XRegs<WT, B> &xr, const GemvArgs &a, int seg, int lw) {
    if constexpr (WT == 3) {
        constexpr int V = Vec<3>::per_thread;
#pragma unroll
        for (int comp = 0; comp < 2; ++comp)
#pragma unroll
            for (int c = 0; c < B; ++c) {
                const int8_t *src = a.q + comp * a.q_comp + static_cast<long long>(c) * a.q_stride;
                const bool col = c < a.batch;
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const int j = vec_index(seg, lw, V, v);
                    int4 t = make_int4(0, 0, 0, 0);
                    if (col && j * 16 < a.k) t = __ldg(reinterpret_cast<const int4 *>(src) + j);
                    xr.v[comp][c][4 * v + 0] = static_cast<uint32_t>(t.x);
                    xr.v[comp][c][4 * v + 1] = static_cast<uint32_t>(t.y);
                    xr.v[comp][c][4 * v + 2] = static_cast<uint32_t>(t.z);
                    xr.v[comp][c][4 * v + 3] = static_cast<uint32_t>(t.w);
                }
            }
    } else if constexpr (WT == 2) {
        (void)lw;
        const int e0 = seg * Seg<2>::elems;
#pragma unroll
        for (int c = 0; c < B; ++c) {
            const float *src = a.x + static_cast<long long>(c) * a.x_stride + e0;
            const bool col = c < a.batch;
#pragma unroll
            for (int v = 0; v < 16; ++v) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (col && e0 + 4 * v < a.k) t = __ldg(reinterpret_cast<const float4 *>(src) + v);
                // elements e..e+3 of block `blk` of this segment, pre-scaled by 2^-s
                const int blk = (4 * v) / 32, e = (4 * v) % 32;
                t.x = __fmul_rn(t.x, pow2_neg(q4_shift(e)));
                t.y = __fmul_rn(t.y, pow2_neg(q4_shift(e + 1)));
                t.z = __fmul_rn(t.z, pow2_neg(q4_shift(e + 2)));
                t.w = __fmul_rn(t.w, pow2_neg(q4_shift(e + 3)));
                xr.v[blk][c][e / 2] = f2_pack(t.x, t.y);
                xr.v[blk][c][e / 2 + 1] = f2_pack(t.z, t.w);
            }
        }
    } else {
        constexpr int V = Vec<WT>::per_thread, E = Vec<WT>::elems;
#pragma unroll
        for (int c = 0; c < B; ++c) {
            const float *src = a.x + static_cast<long long>(c) * a.x_stride;
            const bool col = c < a.batch;
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const int j = vec_index(seg, lw, V, v);
#pragma unroll
                for (int h = 0; h < E / 4; ++h) {
                    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (col && j * E < a.k) t = __ldg(reinterpret_cast<const float4 *>(src + j * E) + h);
                    xr.v[c][(E / 2) * v + 2 * h] = f2_pack(t.x, t.y);
                    xr.v[c][(E / 2) * v + 2 * h + 1] = f2_pack(t.z, t.w);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// per-segment arithmetic
// ---------------------------------------------------------------------------
template <int WT, int B>
struct Partial {
    float f[B];
};
template <int B>
struct Partial<3, B> {
    int d0[B], d1[B];
};

template <int WT, int B>
__device__ __forceinline__ void zero(Partial<WT, B> &p) {
#pragma unroll
    for (int c = 0; c < B; ++c) {
        if constexpr (WT == 3) { p.d0[c] = p.d1[c] = 0; }
        else { p.f[c] = 0.f; }
    }
}

// (w & mask) | m in one LOP3 (the mask is an immediate, m a register).
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or(uint32_t w, uint32_t m) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(MASK), "r"(m));
    return d;
}

// One 32-bit Q4_0 data word (bytes 4j..4j+3 of a block: element 4j+k in the
// low nibble of byte k, element 16+4j+k in its high nibble) against the
// pre-scaled activation pairs; accumulates into s[c][0..1].  With u = w >> 12
// every nibble sits at a bit offset s <= 16, inside the 23-bit mantissa:
//   element  4j   : w bits  0..3  (s = 0)     16+4j : w bits  4..7  (s = 4)
//   element  4j+1 : w bits  8..11 (s = 8)     17+4j : w bits 12..15 (s = 12)
//   element  4j+2 : w bits 16..19 (s = 16)    18+4j : u bits  8..11 (s = 8)
//   element  4j+3 : u bits 12..15 (s = 12)    19+4j : u bits 16..19 (s = 16)
template <int B>
__device__ __forceinline__ void q4_word(uint32_t w, uint32_t m, const unsigned long long (*xp)[16], int j,
                                        unsigned long long (&s)[B][2]) {
    // -(2^23 + 8*2^s) for the offset pairs (0,8), (16,12), (4,12), (8,16)
    constexpr unsigned long long kNeg0_8 = (0xCB000800ull << 32) | 0xCB000008ull;
    constexpr unsigned long long kNeg16_12 = (0xCB008000ull << 32) | 0xCB080000ull;
    constexpr unsigned long long kNeg4_12 = (0xCB008000ull << 32) | 0xCB000080ull;
    constexpr unsigned long long kNeg8_16 = (0xCB080000ull << 32) | 0xCB000800ull;
    const uint32_t u = w >> 12;
    const unsigned long long a01 = f2_add(u2_pack(and_or<0x0000000Fu>(w, m), and_or<0x00000F00u>(w, m)), kNeg0_8);
    const unsigned long long a23 = f2_add(u2_pack(and_or<0x000F0000u>(w, m), and_or<0x0000F000u>(u, m)), kNeg16_12);
    const unsigned long long b01 = f2_add(u2_pack(and_or<0x000000F0u>(w, m), and_or<0x0000F000u>(w, m)), kNeg4_12);
    const unsigned long long b23 = f2_add(u2_pack(and_or<0x00000F00u>(u, m), and_or<0x000F0000u>(u, m)), kNeg8_16);
#pragma unroll
    for (int c = 0; c < B; ++c) {
        s[c][0] = f2_fma(a01, xp[c][2 * j], s[c][0]);
        s[c][1] = f2_fma(a23, xp[c][2 * j + 1], s[c][1]);
        s[c][0] = f2_fma(b01, xp[c][8 + 2 * j], s[c][0]);
        s[c][1] = f2_fma(b23, xp[c][8 + 2 * j + 1], s[c][1]);
    }
}

template <int B>
__device__ __forceinline__ void q4_block(const uint32_t (&dw)[4], float d, const unsigned long long (*xp)[16],
                                         float (&acc)[B]) {
    unsigned long long s[B][2];
#pragma unroll
    for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
    const uint32_t m = 0x4B000000u;  // 2^23
#pragma unroll
    for (int j = 0; j < 4; ++j) q4_word<B>(dw[j], m, xp, j, s);
#pragma unroll
    for (int c = 0; c < B; ++c) acc[c] = fmaf(d, f2_sum(f2_add(s[c][0], s[c][1])), acc[c]);
}

template <int WT, int B>
__device__ __forceinline__ void segment_dot(Partial<WT, B> &out, const uint8_t *row, int seg, int lw, int k,
                                            const XRegs<WT, B> &xr) {
    zero(out);
    if constexpr (WT == 2) {
        const int e0 = seg * Seg<2>::elems;
        const uint32_t *p = reinterpret_cast<const uint32_t *>(row + 36 * seg);
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = p[i];
        // block 2*seg: scale in bytes 0..1, data in bytes 2..17 (2-byte offset)
        const uint32_t d0[4] = {__funnelshift_r(w[0], w[1], 16), __funnelshift_r(w[1], w[2], 16),
                                __funnelshift_r(w[2], w[3], 16), __funnelshift_r(w[3], w[4], 16)};
        q4_block<B>(d0, half_bits_to_float(static_cast<uint16_t>(w[0] & 0xffffu)), xr.v[0], out.f);
        // block 2*seg+1: scale in bytes 18..19, data in bytes 20..35.  Past the
        // row (odd K/32) its bytes belong to the next row: the scale is dropped
        // and the activations are zero, so it adds exactly 0 (even for a
        // non-finite foreign scale or nibble pattern).
        const uint32_t d1[4] = {w[5], w[6], w[7], w[8]};
        const float s1 = e0 + 32 < k ? half_bits_to_float(static_cast<uint16_t>(w[4] >> 16)) : 0.f;
        q4_block<B>(d1, s1, xr.v[1], out.f);
        (void)lw;
    } else if constexpr (WT == 1) {
        constexpr int V = Vec<1>::per_thread;
        const uint4 *p = reinterpret_cast<const uint4 *>(row);
        unsigned long long s[B][2];
#pragma unroll
        for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const int j = vec_index(seg, lw, V, v);
            if (j * 8 >= k) break;  // past the row (K % 64 == 32, or a short K)
            const uint4 t = p[j];
            const uint32_t h[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[i]));
                const unsigned long long wp = f2_pack(f.x, f.y);
#pragma unroll
                for (int c = 0; c < B; ++c) s[c][i & 1] = f2_fma(wp, xr.v[c][4 * v + i], s[c][i & 1]);
            }
        }
#pragma unroll
        for (int c = 0; c < B; ++c) out.f[c] = f2_sum(f2_add(s[c][0], s[c][1]));
    } else if constexpr (WT == 0) {
        constexpr int V = Vec<0>::per_thread;
        const uint4 *p = reinterpret_cast<const uint4 *>(row);
        unsigned long long s[B][2];
#pragma unroll
        for (int c = 0; c < B; ++c) s[c][0] = s[c][1] = 0ull;
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const int j = vec_index(seg, lw, V, v);
            if (j * 4 >= k) break;
            const uint4 t = p[j];
            const unsigned long long w0 = u2_pack(t.x, t.y);
            const unsigned long long w1 = u2_pack(t.z, t.w);
#pragma unroll
            for (int c = 0; c < B; ++c) {
                s[c][0] = f2_fma(w0, xr.v[c][2 * v], s[c][0]);
                s[c][1] = f2_fma(w1, xr.v[c][2 * v + 1], s[c][1]);
            }
        }
#pragma unroll
        for (int c = 0; c < B; ++c) out.f[c] = f2_sum(f2_add(s[c][0], s[c][1]));
    } else {
        constexpr int V = Vec<3>::per_thread;
        const uint4 *p = reinterpret_cast<const uint4 *>(row);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const int j = vec_index(seg, lw, V, v);
            if (j * 16 >= k) break;
            const uint4 t = p[j];
            const uint32_t wv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < B; ++c) {
                    out.d0[c] = __dp4a(static_cast<int>(wv[i]), static_cast<int>(xr.v[0][c][4 * v + i]), out.d0[c]);
                    out.d1[c] = __dp4a(static_cast<int>(wv[i]), static_cast<int>(xr.v[1][c][4 * v + i]), out.d1[c]);
                }
        }
    }
}

// Reduction of a partial across `width` lanes (power of two <= 32).
template <int WT, int B>
__device__ __forceinline__ void reduce_lanes(Partial<WT, B> &p, int width) {
    if (width == 32) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
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
        return;
    }
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

// Final value of output (row, column c) from its complete partial.
template <int WT, int B>
__device__ __forceinline__ float finish(const Partial<WT, B> &p, int c, int row, const GemvArgs &a) {
    if constexpr (WT == 3) {
        const float scale0 = __fdiv_rn(a.act_max[0], 127.0f);
        const float scale1 = __fdiv_rn(a.act_max[1], 127.0f);
        const float t0 = __fmul_rn(static_cast<float>(p.d0[c]), scale0);
        const float t1 = __fmul_rn(static_cast<float>(p.d1[c]), scale1);
        return __fmul_rn(__fadd_rn(t0, t1), a.row_scale[row]);
    } else {
        (void)row;
        (void)a;
        return p.f[c];
    }
}

template <int WT, int B>
__device__ __forceinline__ void accumulate(Partial<WT, B> &acc, const Partial<WT, B> &p) {
#pragma unroll
    for (int c = 0; c < B; ++c) {
        if constexpr (WT == 3) { acc.d0[c] += p.d0[c]; acc.d1[c] += p.d1[c]; }
        else { acc.f[c] += p.f[c]; }
    }
}

// ---------------------------------------------------------------------------
// the streaming kernel
// ---------------------------------------------------------------------------
// Work decomposition inside a CTA (rows [row_begin, row_end)):
//   * the K dimension of a row is split into nseg segments; `tpr` threads
//     (a multiple of 32, or a power of two below 32) form a row slot and
//     thread `seg` of a slot owns segment `seg`;
//   * below 32 threads per row, a warp hosts 32/tpr lane groups that work on
//     different rows of the same chunk;
//   * the row range is cut into chunks of `chunk_rows` rows; chunk c lives in
//     ring stage c % stages and belongs to slot c % slots (stages is a
//     multiple of slots, so a stage always serves the same slot);
//   * a slot computes all rows of its chunk two at a time, reduces each row
//     across its lanes with shuffles and across its warps through shared
//     memory behind one named barrier per chunk, then releases the stage
//     with a single arrival on "empty".
template <int WT, int B>
__global__ void __maxnreg__((Shape<WT, B>::maxreg)) gemv_stream_kernel(const GemvArgs a) {
    using P = Partial<WT, B>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int row_begin = blockIdx.x * a.rows_per_cta;
    const int row_end = min(a.n, row_begin + a.rows_per_cta);
    if (row_begin >= row_end) return;
    const int nchunks = (row_end - row_begin + a.chunk_rows - 1) / a.chunk_rows;
    const int consumer_warps = a.consumers >> 5;
    const int wps = a.tpr >= 32 ? a.tpr / 32 : 1;        // warps per slot
    const int groups = a.tpr >= 32 ? 1 : 32 / a.tpr;     // row groups per warp

    // shared memory: ring | full[S] | empty[S] | red[S][wps][chunk_rows]
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + static_cast<size_t>(a.stages) * a.chunk_bytes);
    uint64_t *empty = full + a.stages;
    P *red = reinterpret_cast<P *>(empty + a.stages);

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == consumer_warps) {
        // ---------------- producer warp ----------------
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            int issued = 0;
            for (int c = 0; c < nchunks; ++c) {
                const int s = c % a.stages;
                if (c >= a.stages && !mbar_wait_sleep(&empty[s], ((c / a.stages) - 1) & 1, a.err, kErrBulkTimeout, 64))
                    break;
                if (c == (a.prefetch < a.stages ? a.prefetch : a.stages)) pdl_wait_prior();
                const int r0 = row_begin + c * a.chunk_rows;
                const int rows = min(a.chunk_rows, row_end - r0);
                const uint32_t bytes = static_cast<uint32_t>(rows * a.row_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s_stream(ring + static_cast<size_t>(s) * a.chunk_bytes, a.w + r0 * a.row_bytes, bytes,
                                &full[s], policy);
                ++issued;
            }
            if (issued <= (a.prefetch < a.stages ? a.prefetch : a.stages)) pdl_wait_prior();
            // never exit with a bulk copy still writing into this CTA's shared memory
            for (int c = issued > a.stages ? issued - a.stages : 0; c < issued; ++c)
                (void)mbar_wait_sleep(&full[c % a.stages], (c / a.stages) & 1, a.err, kErrBulkTimeout, 64);
        }
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait_prior();  // X (and Y) may belong to the previous kernel on the stream
    const int slot = a.tpr >= 32 ? tid / a.tpr : warp;
    const int tis = a.tpr >= 32 ? tid % a.tpr : lane;    // thread index within the slot
    const int seg = a.tpr >= 32 ? tis : (lane % a.tpr);
    const int grp = a.tpr >= 32 ? 0 : (lane / a.tpr);
    const int wis = a.tpr >= 32 ? seg >> 5 : 0;          // warp index within the slot
    const int nseg = (a.k + Seg<WT>::elems - 1) / Seg<WT>::elems;
    const bool active = slot < a.slots;
    // q4_0 segments are contiguous (padding threads own nothing); the vector
    // types interleave across all lanes of the slot and bound-check each vector
    const bool has_seg = active && (WT != 2 || seg < nseg);
    const int lane_width = a.tpr >= 32 ? 32 : a.tpr;
    const int per_group = a.chunk_rows / groups;         // rows of a chunk one lane group computes

    XRegs<WT, B> xr;
    if (has_seg) load_x<WT, B>(xr, a, seg, lane_width);
    if (!active) return;

    for (int c = slot; c < nchunks; c += a.slots) {
        const int s = c % a.stages;
        const int r0 = row_begin + c * a.chunk_rows;
        const int rows = min(a.chunk_rows, row_end - r0);
        if (!mbar_wait(&full[s], (c / a.stages) & 1, a.err, kErrBulkTimeout)) return;
        const uint8_t *chunk = ring + static_cast<size_t>(s) * a.chunk_bytes;
        P *rb = red + static_cast<size_t>(s) * wps * a.chunk_rows;
        // rows grp + groups*j of the chunk, two at a time (warp-uniform trip count)
        for (int j = 0; j < per_group; j += 2) {
            const int i0 = grp + groups * j, i1 = i0 + groups;
            const bool l0 = i0 < rows, l1 = j + 1 < per_group && i1 < rows;
            P p0, p1;
            if (has_seg && l0) segment_dot<WT, B>(p0, chunk + static_cast<size_t>(i0) * a.row_bytes, seg, lane_width, a.k, xr);
            else zero(p0);
            if (has_seg && l1) segment_dot<WT, B>(p1, chunk + static_cast<size_t>(i1) * a.row_bytes, seg, lane_width, a.k, xr);
            else zero(p1);
            reduce_lanes<WT, B>(p0, lane_width);
            reduce_lanes<WT, B>(p1, lane_width);
            if ((seg & (lane_width - 1)) == 0) {
                if (wps == 1) {
#pragma unroll
                    for (int cc = 0; cc < B; ++cc)
                        if (cc < a.batch) {
                            if (l0) a.y[static_cast<long long>(cc) * a.y_stride + r0 + i0] = finish<WT, B>(p0, cc, r0 + i0, a);
                            if (l1) a.y[static_cast<long long>(cc) * a.y_stride + r0 + i1] = finish<WT, B>(p1, cc, r0 + i1, a);
                        }
                } else {
                    if (l0) rb[wis * a.chunk_rows + i0] = p0;
                    if (l1) rb[wis * a.chunk_rows + i1] = p1;
                }
            }
        }
        // order this thread's reads of the stage before the next TMA write into it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (wps > 1) {
            // all warps of the slot have deposited: sum each row in warp order
            asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(a.tpr) : "memory");
            if (tis < rows) {
                P total = rb[tis];
                for (int wv = 1; wv < wps; ++wv) accumulate<WT, B>(total, rb[wv * a.chunk_rows + tis]);
#pragma unroll
                for (int cc = 0; cc < B; ++cc)
                    if (cc < a.batch)
                        a.y[static_cast<long long>(cc) * a.y_stride + r0 + tis] = finish<WT, B>(total, cc, r0 + tis, a);
            }
            if (tis == 0) mbar_arrive(&empty[s]);
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
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
            const uint32_t b = ldb(row + 4 * j) | (ldb(row + 4 * j + 1) << 8) | (ldb(row + 4 * j + 2) << 16) |
                               (static_cast<uint32_t>(ldb(row + 4 * j + 3)) << 24);
            wv = __uint_as_float(b);
        } else if (wt == 1) {
            wv = half_bits_to_float(static_cast<uint16_t>(ldb(row + 2 * j) | (ldb(row + 2 * j + 1) << 8)));
        } else {
            const uint8_t *blk = row + (j / 32) * 18;
            const float d = half_bits_to_float(static_cast<uint16_t>(ldb(blk) | (ldb(blk + 1) << 8)));
            const int e = j % 32;
            const int nib = (ldb(blk + 2 + (e % 16)) >> (e < 16 ? 0 : 4)) & 15;
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
        const float t0 = __fmul_rn(static_cast<float>(s0), scale0);
        const float t1 = __fmul_rn(static_cast<float>(s1), scale1);
        y[static_cast<long long>(c) * y_stride + r] = __fmul_rn(__fadd_rn(t0, t1), scale[r]);
    }
}

// ---------------------------------------------------------------------------
// launch planning
// ---------------------------------------------------------------------------
struct Plan {
    int tpr, slots, chunk_rows, stages, consumers, threads, grid, rows_per_cta;
    uint32_t chunk_bytes;
    size_t smem;
};

// Threads a launch of gemv_stream_kernel<WT, B> may use on this device (its
// register footprint as reported by the runtime), cached per device.
template <int WT, int B>
int kernel_thread_limit() {
    static int limit[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 0;
    if (!limit[dev]) {
        cudaFuncAttributes attr{};
        if (cudaFuncGetAttributes(&attr, gemv_stream_kernel<WT, B>) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        limit[dev] = attr.maxThreadsPerBlock;
        if (std::getenv("KUNLUN_DEBUG"))
            std::fprintf(stderr, "k200 gemv<%d,%d>: %d registers, %d threads max\n", WT, B, attr.numRegs,
                         attr.maxThreadsPerBlock);
    }
    return limit[dev];
}

template <int WT, int B>
bool make_plan(Plan &p, int k, int n, long long row_bytes, const DeviceInfo &dev) {
    using S = Shape<WT, B>;
    const int thread_limit = kernel_thread_limit<WT, B>();
    int consumer_limit = (thread_limit - 32) / 32 * 32;
    if (consumer_limit > S::consumers) consumer_limit = S::consumers;
    if (consumer_limit < 32) return false;
    const int nseg = (k + Seg<WT>::elems - 1) / Seg<WT>::elems;
    if (nseg <= 32) {
        p.tpr = 1;
        while (p.tpr < nseg) p.tpr <<= 1;
    } else {
        p.tpr = (nseg + 31) / 32 * 32;
    }
    if (p.tpr > consumer_limit) return false;
    const int groups = p.tpr >= 32 ? 1 : 32 / p.tpr;
    const int slot_threads = p.tpr >= 32 ? p.tpr : 32;
    p.grid = dev.sm_count;
    p.rows_per_cta = (n + p.grid - 1) / p.grid;
    // rows per chunk: a multiple of 2*groups (two rows per lane group), about
    // 8-24 KB, never more than the CTA's rows
    int rows = 2 * groups;
    while (rows * 2 * row_bytes <= 16 * 1024 && rows * 2 <= 32 * groups) rows *= 2;
    if (rows > p.rows_per_cta) rows = (p.rows_per_cta + 2 * groups - 1) / (2 * groups) * (2 * groups);
    p.chunk_rows = rows;
    p.chunk_bytes = static_cast<uint32_t>(rows * row_bytes);
    const int chunks = (p.rows_per_cta + rows - 1) / rows;
    p.slots = consumer_limit / slot_threads;
    if (p.slots > chunks) p.slots = chunks;
    if (p.slots > 14) p.slots = 14;  // named barriers 1..14 (15: q4_0 prologue)
    if (p.slots < 1) p.slots = 1;
    const int wps = p.tpr >= 32 ? p.tpr / 32 : 1;
    const size_t budget = static_cast<size_t>(dev.smem_optin) - 1024;
    const size_t table = 0;
    auto need = [&](int stages) {
        return stages * static_cast<size_t>(p.chunk_bytes) + 16 * stages +
               stages * static_cast<size_t>(wps) * rows * sizeof(Partial<WT, B>) + 64 + table;
    };
    // stages: a multiple of the slot count.  A slot with several warps reuses
    // a stage's reduction buffer only after one more named barrier, so it
    // needs at least two stages.
    int per_slot = 3;
    const int min_per_slot = wps > 1 ? 2 : 1;
    while (per_slot > min_per_slot && need(per_slot * p.slots) > budget) --per_slot;
    while (p.slots > 1 && need(per_slot * p.slots) > budget) --p.slots;
    if (need(per_slot * p.slots) > budget) return false;
    p.stages = per_slot * p.slots;
    p.smem = need(p.stages);
    p.consumers = p.slots * slot_threads;
    p.threads = p.consumers + 32;
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
    a.consumers = p.consumers;
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
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(p.threads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
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

namespace {
cudaError_t launch_generic(const GemvRequest &r, int c0, int cols, long long row_bytes, cudaStream_t stream) {
    const int warps = r.n * cols;
    const int threads = 256;
    const int blocks = (warps * 32 + threads - 1) / threads;
    if (r.wt == 3) {
        gemv_i8_generic_kernel<<<blocks, threads, 0, stream>>>(
            static_cast<const int8_t *>(r.w), r.q + static_cast<long long>(c0) * r.q_stride, r.q_comp, r.act_max,
            r.row_scale, r.y + static_cast<long long>(c0) * r.y_stride, r.k, r.n, cols, r.q_stride, r.y_stride);
    } else {
        gemv_generic_kernel<<<blocks, threads, 0, stream>>>(
            static_cast<const uint8_t *>(r.w), r.wt, r.x + static_cast<long long>(c0) * r.x_stride,
            r.y + static_cast<long long>(c0) * r.y_stride, r.k, r.n, cols, row_bytes, r.x_stride, r.y_stride);
    }
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemv(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    if (r.tensor_cores && gemm_tc_supported(r.wt, r.k, r.n, r.batch)) {
        const cudaError_t e = launch_gemm_tc(r, dev, stream);
        if (e != cudaErrorNotSupported) return e;
    }
    if (r.fixup) {
        const cudaError_t e = launch_q4_mma_gemv(r, dev, stream);
        if (e != cudaErrorNotSupported) return e;
    }
    if (r.wt == 0 && gemm_f32_supported(r)) return launch_gemm_f32(r, dev, stream);
    const long long row_bytes = r.wt == 0 ? 4ll * r.k : r.wt == 1 ? 2ll * r.k : r.wt == 2 ? 18ll * (r.k / 32) : r.k;
    const bool fast = gemv_fast_path_ok(r.wt, r.w, r.x, r.y, r.k, row_bytes);
    for (int c0 = 0; c0 < r.batch; c0 += 2) {
        const int cols = r.batch - c0 < 2 ? r.batch - c0 : 2;
        GemvArgs a{};
        a.w = static_cast<const uint8_t *>(r.w);
        a.x = r.x ? r.x + static_cast<long long>(c0) * r.x_stride : nullptr;
        a.q = r.q ? r.q + static_cast<long long>(c0) * r.q_stride : nullptr;
        a.q_comp = r.q_comp;
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
        a.prefetch = r.prefetch_weights ? 1 << 30 : 0;  // clamped to the ring size by the producer
        a.err = dev.err;
        cudaError_t e = cudaErrorInvalidConfiguration;  // "no streaming plan fits": take the generic kernel
        if (fast) {
            switch (r.wt) {
                case 0: e = launch_batch_group<0>(a, dev, stream, cols); break;
                case 1: e = launch_batch_group<1>(a, dev, stream, cols); break;
                case 2: e = launch_batch_group<2>(a, dev, stream, cols); break;
                default: e = launch_batch_group<3>(a, dev, stream, cols); break;
            }
        }
        if (e == cudaErrorInvalidConfiguration) e = launch_generic(r, c0, cols, row_bytes, stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace k200
