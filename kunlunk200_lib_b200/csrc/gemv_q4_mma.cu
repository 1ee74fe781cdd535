// Q4_0 matrix-vector product for one activation column on the tensor cores
// (sm_100a): Y[r] = sum_b d[r,b] * sum_j (q[r,b,j] - 8) * x[32b + j], the
// arithmetic of kernels/kunlun-matvec.xpu:37-77 of the reference.
//
// Why this kernel exists: at batch 1 a Q4_0 GEMV is bounded by how fast the
// SMs can turn nibbles into numbers, not by HBM, unless the decode costs
// about one instruction per weight.  Here two nibbles become two exact f16
// values (v - 8) with one LOP3 (OR the nibble into the mantissa of 1024.0)
// plus one HADD2/HFMA2, and mma.sync m16n8k16 does the multiply-add.  The
// activations are split into f16 hi + lo halves (x = hi + lo to about 22
// bits) after a power-of-two scaling per 32-element block, the fp16 block
// scale d is applied in f32 to each block's dot product, and partial sums
// are f32.  Results agree with the reference's FP32 arithmetic to within its
// rounding (the products (v-8)*hi and (v-8)*lo are exact; the error is the
// hi/lo truncation, about 2^-22 relative per term, plus f32 summation).
//
// Layout and work split:
//  * the unit of work is 16 rows x 144 bytes of the weight matrix (eight
//    Q4_0 blocks of each row, two "groups" of four blocks).  K is cut into
//    parts of at most 16 units (4096 values; one part up to K = 4096), the
//    CTAs (one per SM) are shared out to the parts in proportion to their
//    units, and within a part the units are numbered row-tile-major and
//    every CTA takes a contiguous range of them, so the bytes per CTA are
//    balanced to within about one unit and a CTA prepares at most 16 KiB of
//    X.  The last part's CTA that finishes a row tile adds the other parts'
//    sums of it in part order;
//  * a producer thread streams the CTA's range as "boxes" of 16 rows x 1-4
//    units (2-D TMA tensor copies, cp.async.bulk.tensor + mbarriers): each
//    row tile's part of the range is cut into boxes of four units (576-byte
//    rows, read as 592 so that the row pitch in shared memory is bank-
//    conflict-free) and one narrower box for the remainder;
//  * the ring has 16 stages and box j lands in stage j mod 16.  Unit slot q
//    of box j goes to consumer warp 4 (j mod Q) + q (Q quads of warps), so
//    each warp meets its boxes' phases in order and the work per warp is
//    balanced to within about one unit.  A warp
//    computes its unit (one m16 tile per group of four blocks) and releases
//    its slot with one mbarrier arrival (the producer arrives for the slots a
//    narrow box lacks).  The producer records each box's position in a small
//    table before its copy is issued, so the consumers need no box
//    arithmetic;
//  * within a group the four blocks use the four column pairs of the n8
//    MMA: column pair i holds (hi, lo) of block beta(i)'s activations and
//    zero elsewhere, so after the 8 MMAs of a group the accumulator holds
//    four separate block dots and lane c of each quad finds block beta(c)
//    in its own columns.  Each lane then applies d and the activation scale
//    of one block per row and accumulates in f32;
//  * activations are prepared once per CTA into "fragment records" in shared
//    memory (544 bytes per group: the B fragments of the four column pairs,
//    16 zero bytes and the four block scales), so the main loop reads them
//    with one 16-byte load per block;
//  * each warp keeps running row sums of its current row tile in registers
//    and adds them to its own partial sums of that tile in shared memory when
//    the tile changes; after the last box the CTA's warps meet at
//    one barrier and finish the CTA's tiles (one warp per tile): sum the
//    warps' partials in warp order and store Y.  A tile shared with other
//    CTAs is finished by the CTA that holds its first units, which adds the
//    higher CTAs' sums in CTA order, so results do not depend on timing.
//    Those sums move early: every consumer warp signals when it is past its
//    first row tile, and the producer warp (idle once its boxes are issued)
//    then publishes the CTA's sum of that tile and collects the higher CTAs'
//    sums of the CTA's last tile into shared memory while the consumers are
//    still working, so the finish does not wait on another CTA's loop.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "device_common.cuh"
#include "k200_internal.h"
#include "exchange.cuh"

namespace k200 {

namespace {

constexpr int kTileRows = 16;                          // rows of a box: one m16 tile
constexpr int kPairBytes = 144;                        // a unit's bytes per row: two groups of four blocks
constexpr int kPairWords = kPairBytes / 4;
constexpr int kMaxBoxPairs = 4;                        // widest box: 16 rows x 4 units
// Words a box row of w units occupies in shared memory: the units, plus four
// words of the next bytes of the row when w is even, so that the row pitch
// is 4 mod 8 words and the eight rows a load instruction touches (lane
// pattern below) fall in different banks.
__host__ __device__ constexpr int box_words(int w) { return kPairWords * w + ((w & 1) ? 0 : 4); }
constexpr int kStageBytes = kTileRows * 4 * box_words(kMaxBoxPairs);  // 9472
constexpr int kRecBytes = 544;                         // fragment record of one group
constexpr int kZeroOff = 512, kScaleOff = 528;
#ifndef K200_Q4_GEMV_WARPS
#define K200_Q4_GEMV_WARPS 16
#endif
constexpr int kWarps = K200_Q4_GEMV_WARPS;             // consumer warps, four per box
constexpr int kQuads = kWarps / 4;                     // box j is read by quad j mod kQuads
constexpr int kStages = 16;                            // ring stages (box j in stage j mod 16)
constexpr int kThreads = (kWarps + 1) * 32;
// K is cut into at most kMaxParts parts of at most kPartPairs pairs (256
// values): a CTA works on one part, so it reads and converts at most 16 KiB of
// X, and a row tile of a part has at most 16 units, so at most 15 later CTAs
// share a CTA's last tile.
constexpr int kPartPairs = 16;
constexpr int kMaxParts = 4;
constexpr int kMaxPeers = kPartPairs;
static_assert(kWarps % 4 == 0 && kWarps >= 16, "consumer warps come in quads, at least one per four stages");

struct Q4MmaArgs {
    const float *x;
    float *y;
    unsigned long long *slot;  // [grid][16] tagged partial sums of row tiles shared with other CTAs
    unsigned long long *vt;    // [tiles][parts - 1][16] tagged sums of a row tile over K parts 0 .. parts-2
    int *err;
    int k, n, tiles, grid, prefetch;
    int parts;                       // K parts (units of part s: row tiles x pairs [part_pair[s], part_pair[s+1]))
    int part_pair[kMaxParts + 1];    // first pair of each part (and ppr at the end)
    int part_cta[kMaxParts + 1];     // first CTA of each part (and grid at the end), in proportion to its units
    int rec_groups;                  // activation records held (2 x the pairs of the largest part)
    int max_tiles;      // row tiles any CTA touches (partial-sum slots in shared memory)
    int max_boxes;      // boxes any CTA streams (entries of the box table)
};

// Tensor maps over the weight rows viewed as 32-bit words [n][row_bytes/4],
// with boxes of 16 rows x 1, 2, 3 and 4 units (box[w - 1] for width w).
struct Q4MmaMaps {
    CUtensorMap box[kMaxBoxPairs];
};

// The CTA's units [u, end) covered by boxes, segment by segment (a segment
// is one row tile's part of the range): boxes of four units, then one box
// for the rest of the segment.
struct BoxWalk {
    int u, end;
    int tile, pair, width, ppr;
    __device__ BoxWalk(int begin, int end_, int ppr_) : u(begin), end(end_), ppr(ppr_) {
        tile = begin / ppr;
        pair = begin - tile * ppr;
        fit();
    }
    __device__ void fit() { width = min(kMaxBoxPairs, min(ppr - pair, end - u)); }
    __device__ void next() {
        u += width;
        pair += width;
        if (pair == ppr) { pair = 0; ++tile; }
        fit();
    }
};

// Boxes that cover a segment of L units.
__host__ __device__ constexpr int boxes_in(int L) { return (L + kMaxBoxPairs - 1) / kMaxBoxPairs; }

// Column pair c of the MMA carries block beta(c) of a group, beta = (3, 1, 2, 0),
// and lane c of a quad finishes that block; beta_inv is the inverse.
__host__ __device__ constexpr int beta_inv(int b) { return b == 0 ? 3 : b == 1 ? 1 : b == 2 ? 2 : 0; }

// Bytes (qs indices 0..15) of block position p (0..3 in its group) that
// lane c of a quad decodes.  Groups are 72 bytes (18 words) and start
// 8-byte aligned; blocks 1 and 3 have their 16 nibble bytes on word
// boundaries, blocks 0 and 2 are offset by two bytes, so three lanes take
// aligned words and the fourth combines the two-byte ends of the block.
__host__ __device__ constexpr void lane_bytes(int p, int c, int (&q)[4]) {
    if (p & 1) {
        for (int i = 0; i < 4; ++i) q[i] = 4 * c + i;
    } else if (p == 0) {
        if (c < 3) { for (int i = 0; i < 4; ++i) q[i] = 2 + 4 * c + i; }
        else { q[0] = 0; q[1] = 1; q[2] = 14; q[3] = 15; }
    } else {
        if (c == 0) { q[0] = 0; q[1] = 1; q[2] = 14; q[3] = 15; }
        else { for (int i = 0; i < 4; ++i) q[i] = 4 * c - 2 + i; }
    }
}

// Lane c's bytes of block position p come in two adjacent pairs starting at
// pair_first and pair_second (the activation loader reads them as float2s).
__host__ __device__ constexpr int pair_first(int p, int c) {
    return (p & 1) ? 4 * c : p == 0 ? (c < 3 ? 2 + 4 * c : 0) : (c == 0 ? 0 : 4 * c - 2);
}
__host__ __device__ constexpr int pair_second(int p, int c) {
    return (p & 1) ? 4 * c + 2 : p == 0 ? (c < 3 ? 4 + 4 * c : 14) : (c == 0 ? 14 : 4 * c);
}
constexpr bool pairs_match_lane_bytes() {
    for (int p = 0; p < 4; ++p)
        for (int c = 0; c < 4; ++c) {
            int q[4] = {0, 0, 0, 0};
            lane_bytes(p, c, q);
            const int a0 = pair_first(p, c), a1 = pair_second(p, c);
            if (q[0] != a0 || q[1] != a0 + 1 || q[2] != a1 || q[3] != a1 + 1) return false;
        }
    return true;
}
static_assert(pairs_match_lane_bytes(), "activation pairs disagree with the lane byte map");

template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or(uint32_t w, uint32_t m) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(MASK), "r"(m));
    return d;
}
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One 32-bit word of nibble bytes (b0, b1, b2, b3) -> four f16x2 registers of
// exact (v - 8) values: t0 = {lo(b0), lo(b2)}, t1 = {hi(b0), hi(b2)},
// t2 = {lo(b1), lo(b3)}, t3 = {hi(b1), hi(b3)}.
//   lo nibble: (w & 0x000f000f) | 0x6400 pairs = 1024 + v;  + (-1032)      = v - 8
//   hi nibble: (w & 0x00f000f0) | 0x6400 pairs = 1024 + 16v; * 1/16 + (-72) = v - 8
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t (&t)[4]) {
    const uint32_t m = 0x64006400u;
    const uint32_t w8 = w >> 8;
    t[0] = hadd2_u(and_or<0x000F000Fu>(w, m), 0xE408E408u);
    t[1] = hfma2_u(and_or<0x00F000F0u>(w, m), 0x2C002C00u, 0xD480D480u);
    t[2] = hadd2_u(and_or<0x000F000Fu>(w8, m), 0xE408E408u);
    t[3] = hfma2_u(and_or<0x00F000F0u>(w8, m), 0x2C002C00u, 0xD480D480u);
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

template <int OFF>
__device__ __forceinline__ uint32_t lds_at(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(OFF));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory");
}

// CTA that processes unit u (CTA i owns units [i*U/G, (i+1)*U/G)).
__device__ __forceinline__ int cta_of(uint32_t u, uint32_t units, int grid) {
    return static_cast<int>(((u + 1) * static_cast<uint32_t>(grid) - 1) / units);
}

// One B-fragment slot pair of an activation block is built by the four
// threads of a quad together (thread c writes the hi and lo slots of lane c).
// load_slot fetches lane c's eight activations: x[a0], x[a0+1], x[a1],
// x[a1+1] and the same +16 (see lane_bytes); store_slot scales the block by
// 2^-e so that its largest magnitude lies in [2^14, 2^15), splits the values
// into f16 hi + lo and stores them (all 32 lanes of the warp must call it).
__device__ __forceinline__ void load_slot(const float *xb, int p, int c, float (&v)[8]) {
    const int a0 = pair_first(p, c), a1 = pair_second(p, c);
    const float2 *q0 = reinterpret_cast<const float2 *>(xb + a0), *q1 = reinterpret_cast<const float2 *>(xb + a1);
    const float2 l0 = __ldg(q0);
    const float2 l1 = __ldg(q1);
    const float2 h0 = __ldg(q0 + 8);
    const float2 h1 = __ldg(q1 + 8);
    // register order = fragment order: {q0, q2}, {q0+16, q2+16}, {q1, q3}, {q1+16, q3+16}
    v[0] = l0.x; v[1] = l1.x; v[2] = h0.x; v[3] = h1.x;
    v[4] = l0.y; v[5] = l1.y; v[6] = h0.y; v[7] = h1.y;
}

// The same eight activations when X is another exchange's output: tagged
// words {f32, epoch} (exchange.cuh) for the block's first `lim` elements,
// plain floats after them (the zeroed padding past the exchange's rows).
// issue_slot_tagged starts the loads of the tagged words.
__device__ __forceinline__ void issue_slot_tagged(const unsigned long long *tb, int lim, int p, int c,
                                                  unsigned long long (&w)[8]) {
    const int a0 = pair_first(p, c), a1 = pair_second(p, c);
    const int e[4] = {a0, a1, a0 + 16, a1 + 16};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        w[2 * q] = 0ull;
        w[2 * q + 1] = 0ull;
        if (e[q] + 1 < lim) ld_tag2(tb + e[q], w[2 * q], w[2 * q + 1]);
        else if (e[q] < lim) w[2 * q] = ld_tag(tb + e[q]);
    }
}
// One round of the wait for a slot's tagged words: re-issues the loads of
// the words that do not carry `epoch` yet and returns whether there were any
// (their new values are checked in the next round, so the rounds of all of a
// thread's slots share one round trip).
__device__ __forceinline__ bool refresh_slot_tagged(const unsigned long long *tb, int lim, int p, int c,
                                                    unsigned long long (&w)[8], unsigned epoch) {
    const int a0 = pair_first(p, c), a1 = pair_second(p, c);
    const int e[4] = {a0, a1, a0 + 16, a1 + 16};
    bool any = false;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const bool stale = (e[q] < lim && tag_epoch(w[2 * q]) != epoch) ||
                           (e[q] + 1 < lim && tag_epoch(w[2 * q + 1]) != epoch);
        if (!stale) continue;
        any = true;
        if (e[q] + 1 < lim) ld_tag2(tb + e[q], w[2 * q], w[2 * q + 1]);
        else w[2 * q] = ld_tag(tb + e[q]);
    }
    return any;
}
// The slot's eight activations once its words are current, in load_slot's order.
__device__ __forceinline__ void values_slot_tagged(const float *xb, int lim, int p, int c,
                                                   const unsigned long long (&w)[8], float (&v)[8]) {
    const int a0 = pair_first(p, c), a1 = pair_second(p, c);
    const int e[4] = {a0, a1, a0 + 16, a1 + 16};
    float2 f[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (e[q] + 1 < lim) {
            f[q].x = tag_value(w[2 * q]);
            f[q].y = tag_value(w[2 * q + 1]);
        } else if (e[q] >= lim) {
            f[q] = __ldcg(reinterpret_cast<const float2 *>(xb + e[q]));
        } else {  // the last tagged element, then padding
            f[q].x = tag_value(w[2 * q]);
            f[q].y = __ldcg(xb + e[q] + 1);
        }
    }
    v[0] = f[0].x; v[1] = f[1].x; v[2] = f[2].x; v[3] = f[3].x;
    v[4] = f[0].y; v[5] = f[1].y; v[6] = f[2].y; v[7] = f[3].y;
}

__device__ __forceinline__ void store_slot(const float (&v)[8], uint8_t *rec, int p, int c, bool store) {
    uint32_t mx = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = max(mx, __float_as_uint(v[i]) & 0x7fffffffu);
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    int e = 0;  // x = 2^e * x'
    const bool finite = mx < 0x7f800000u;
    if (mx != 0 && finite) {
        int ex = static_cast<int>(mx >> 23) - 127;                                 // floor(log2(max))
        if (mx < 0x00800000u) ex = (31 - __clz(static_cast<int>(mx))) - 149;       // subnormal max
        e = min(max(ex - 14, -126), 113);
    }
    const float scale = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e, a normal float
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float u = __fmul_rn(v[2 * i], scale), w = __fmul_rn(v[2 * i + 1], scale);
        const __half2 h = __floats2half2_rn(u, w);
        const float2 hf = __half22float2(h);
        __half2 l = __floats2half2_rn(__fsub_rn(u, hf.x), __fsub_rn(w, hf.y));
        if (!finite) {
            // a non-finite hi keeps its Inf/NaN alone (lo = 0), as v*x would
            if (!((__float_as_uint(hf.x) & 0x7fffffffu) < 0x7f800000u)) l.x = __ushort_as_half(0);
            if (!((__float_as_uint(hf.y) & 0x7fffffffu) < 0x7f800000u)) l.y = __ushort_as_half(0);
        }
        hi[i] = *reinterpret_cast<const uint32_t *>(&h);
        lo[i] = *reinterpret_cast<const uint32_t *>(&l);
    }
    if (!store) return;
    const int col = beta_inv(p);  // column pair that carries this block
    *reinterpret_cast<uint4 *>(rec + col * 128 + c * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(rec + col * 128 + 64 + c * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    if (c == 0) *reinterpret_cast<float *>(rec + kScaleOff + 4 * col) = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
    if (c == 0 && p == 0) *reinterpret_cast<uint4 *>(rec + kZeroOff) = make_uint4(0, 0, 0, 0);
}

// Partial sums of a row tile shared between CTAs travel as 64-bit words
// {1, f32 bits}: value and "present" tag in one single-copy-atomic access,
// so the reader needs no fence.  The reader clears each word after use, so
// every launch starts from zeros.
__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
constexpr unsigned long long kPresent = 1ull << 32;
constexpr uint32_t kPeerBudget = 1u << 20;   // polls of a partial sum (with 64 ns sleeps)

// kGather: the fused all-gather (xg.ranks > 0) and the wait for X
// (xg.wait_flags), in a separate instantiation with its own parameter, so that
// the plain GEMV carries none of its code or registers.
template <bool kGather>
__global__ void __launch_bounds__(kThreads, 1)
    q4_mma_gemv_kernel(const __grid_constant__ Q4MmaMaps maps, const Q4MmaArgs a, const __grid_constant__ GatherLaunch xg) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint8_t *xrec = ring + kStages * kStageBytes;  // [rec_groups] records, by group within the K part
    float *part = reinterpret_cast<float *>(xrec + a.rec_groups * kRecBytes);  // [max_tiles][kWarps][16]
    float *peer = part + a.max_tiles * kWarps * kTileRows;  // [kMaxPeers][16]: later CTAs' sums of the last tile
    uint64_t *full = reinterpret_cast<uint64_t *>(peer + kMaxPeers * kTileRows);
    uint64_t *empty = full + kStages;
    uint64_t *first_done = empty + kStages;  // every consumer lane is past the first row tile
    uint64_t *peers_in = first_done + 1;     // the producer warp has collected the last tile's peer sums
    volatile uint32_t *box_tab = reinterpret_cast<volatile uint32_t *>(peers_in + 1);  // [max_boxes]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // This CTA's K part: CTAs cta0 .. cta0 + grid_p - 1 share its units, the
    // row tiles x its pairs [pair0, pair0 + ppr), numbered row-tile-major;
    // CTA `cta` of the part takes a contiguous, balanced range of them.
    int part_s = 0, cta0 = a.part_cta[0], cta_end = a.part_cta[1], pair0 = a.part_pair[0], pair_end = a.part_pair[1];
#pragma unroll
    for (int s = 1; s < kMaxParts; ++s)  // constant indices: the parameter arrays stay in the constant bank
        if (s < a.parts && static_cast<int>(blockIdx.x) >= a.part_cta[s]) {
            part_s = s;
            cta0 = a.part_cta[s];
            cta_end = a.part_cta[s + 1];
            pair0 = a.part_pair[s];
            pair_end = a.part_pair[s + 1];
        }
    const int grid_p = cta_end - cta0, cta = static_cast<int>(blockIdx.x) - cta0, ppr = pair_end - pair0;
    const uint32_t units = static_cast<uint32_t>(a.tiles) * static_cast<uint32_t>(ppr);
    const int u0 = static_cast<int>(static_cast<uint32_t>(cta) * units / static_cast<uint32_t>(grid_p));
    const int u1 = static_cast<int>(static_cast<uint32_t>(cta + 1) * units / static_cast<uint32_t>(grid_p));
    const int t_first = u0 / ppr;
    const int t_last = (u1 - 1) / ppr;

    if (tid < kStages) {
        mbar_init(&full[tid], 1);
        mbar_init(&empty[tid], kMaxBoxPairs);  // one arrival per unit slot of a box
        if (tid == 0) {
            mbar_init(first_done, kWarps * 32);
            mbar_init(peers_in, 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    // Row tiles shared with other CTAs: this CTA's first tile began in a lower
    // CTA (which finishes it) when p_first > 0; its last tile continues in
    // higher CTAs (whose sums this CTA collects) when collect_last.
    const int p_first = u0 - t_first * ppr;
    const int p_end = u1 - t_last * ppr;
    const bool collect_last = (t_last + 1) * ppr > u1 && t_last * ppr >= u0;

    if (warp == kWarps) {
        // ---------------- producer ----------------
        int issued = 0;
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < kMaxBoxPairs; ++m)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.box[m])) : "memory");
            const uint64_t policy = policy_evict_first();
            const int early = a.prefetch < kStages ? a.prefetch : kStages;
            const uint32_t ring_u = smem_u32(ring);
            int j = 0;
            for (BoxWalk bw(u0, u1, ppr); bw.u < u1 && j < a.max_boxes; bw.next(), ++j) {
                const int s = j % kStages;
                if (j >= kStages && !mbar_wait_sleep(&empty[s], ((j / kStages) & 1) ^ 1, a.err, kErrBulkTimeout, 128))
                    break;
                if (j == early) pdl_wait_prior();
                // published to the consumer by the arrive below (release) and its wait (acquire)
                box_tab[j] = static_cast<uint32_t>(bw.tile - t_first) | (static_cast<uint32_t>(bw.pair) << 16) |
                             (static_cast<uint32_t>(bw.width) << 24);
                mbar_arrive_expect_tx(&full[s], kTileRows * 4 * box_words(bw.width));
                tma_load_2d(ring_u + s * kStageBytes, &maps.box[bw.width - 1], (pair0 + bw.pair) * kPairWords,
                            bw.tile * kTileRows, &full[s], policy);
                // the unit slots a narrow box lacks are released here
                if (bw.width < kMaxBoxPairs) mbar_arrive_count(&empty[s], kMaxBoxPairs - bw.width);
            }
            if (j <= early) pdl_wait_prior();
            issued = j;
        }
        __syncwarp();
        pdl_wait_prior();  // the partial-sum words were cleared by the previous launch's collectors
        // Publish the sum of the first row tile as soon as the consumers are
        // past it (the lower CTA that finishes the tile then finds it early),
        // and collect the higher CTAs' sums of the last row tile while the
        // consumers still work, so neither waits at the end.
        if (p_first > 0) {
            bool ok = false;
            for (uint32_t i = 0; i < kWaitBudget && !ok; ++i) ok = mbar_try_wait(first_done, 0);
            if (!ok) atomicExch(a.err, kErrBulkTimeout);
            if (lane < kTileRows) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) v += part[w * kTileRows + lane];
                st_relaxed(a.slot + static_cast<size_t>(blockIdx.x) * kTileRows + lane, kPresent | __float_as_uint(v));
            }
        }
        if (collect_last) {
            const int last = cta_of(static_cast<uint32_t>((t_last + 1) * ppr - 1), units, grid_p);
            if (lane < kTileRows) {
                for (int j0 = cta + 1; j0 <= last; ++j0) {
                    unsigned long long *src = a.slot + static_cast<size_t>(cta0 + j0) * kTileRows + lane;
                    unsigned long long w = ld_relaxed(src);
                    for (uint32_t spin = 0; !(w & kPresent); ++spin) {
                        if (spin >= kPeerBudget) {
                            atomicExch(a.err, kErrPeerTimeout);
                            break;
                        }
                        __nanosleep(64);
                        w = ld_relaxed(src);
                    }
                    peer[(j0 - cta - 1) * kTileRows + lane] = __uint_as_float(static_cast<uint32_t>(w));
                    st_relaxed(src, 0ull);
                }
            }
            mbar_arrive(peers_in);
        }
        if (lane == 0) {
            // never exit with a copy still writing into this CTA's shared memory
            for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
                (void)mbar_wait_sleep(&full[i % kStages], (i / kStages) & 1, a.err, kErrBulkTimeout, 128);
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait_prior();  // x, y, the partial-sum words and the exchange counters may belong to earlier kernels
    // X from another exchange (its tagged words, as every rank's rows arrive)
    const bool peer_x = kGather && xg.wait_tags != nullptr;
    const unsigned wait_epoch = peer_x ? exchange_epoch(xg.wait_counter) : 0u;
    // this launch's epoch of its own exchange
    const unsigned epoch = kGather && xg.ranks > 0 ? exchange_epoch(xg.counter) + 1u : 0u;
    {
        // fragment records: four threads per activation block; every load of a
        // thread is issued before the first conversion.  Only the unit pairs
        // (256-element K ranges, 32 slots each) of the CTA's K part that its
        // units touch are built: the pairs p_first .. ppr-1 and 0 .. p_end-1
        // of its first and last row tiles, i.e. every pair of the part once
        // the range covers a whole row tile.  (At most kPartPairs pairs.)
        constexpr int kPasses = (kPartPairs * 32 + kWarps * 32 - 1) / (kWarps * 32);
        const int pf = u0 - t_first * ppr, pe = u1 - t_last * ppr;
        int p_start = 0, npairs = ppr;
        if (t_first == t_last) {
            p_start = pf;
            npairs = pe - pf;
        } else if (t_last == t_first + 1 && pe <= pf) {
            p_start = pf;
            npairs = ppr - pf + pe;
        }
        const int count = 32 * npairs;  // a multiple of 32: whole warps are inside or past the range
        float xv[kPasses][8];
        if (kGather && peer_x) {
            // tagged words: every load of the thread is issued before the first wait
            unsigned long long xw[kPasses][8];
#pragma unroll
            for (int k = 0; k < kPasses; ++k)
                if (k * kWarps * 32 < count) {
                    const int t = min(k * kWarps * 32 + tid, count - 1);
                    const int pr = p_start + (t >> 5);
                    const int b = (((pr < ppr ? pr : pr - ppr) * 32 + (t & 31)) >> 2) + 8 * pair0;
                    issue_slot_tagged(xg.wait_tags + 32 * b, xg.wait_tagged - 32 * b, b & 3, lane & 3, xw[k]);
                }
            // every pass's stale words are re-loaded together: one round trip per round
            for (uint32_t spin = 0;; ++spin) {
                bool any = false;
#pragma unroll
                for (int k = 0; k < kPasses; ++k)
                    if (k * kWarps * 32 < count) {
                        const int t = min(k * kWarps * 32 + tid, count - 1);
                        const int pr = p_start + (t >> 5);
                        const int b = (((pr < ppr ? pr : pr - ppr) * 32 + (t & 31)) >> 2) + 8 * pair0;
                        any |= refresh_slot_tagged(xg.wait_tags + 32 * b, xg.wait_tagged - 32 * b, b & 3, lane & 3,
                                                   xw[k], wait_epoch);
                    }
                if (!any) break;
                if (spin >= kTagBudget ||
                    ((spin & 255u) == 255u && *reinterpret_cast<volatile int *>(a.err) == kErrPeerTimeout)) {
                    atomicExch(a.err, kErrPeerTimeout);
                    break;
                }
                __nanosleep(64);
            }
#pragma unroll
            for (int k = 0; k < kPasses; ++k)
                if (k * kWarps * 32 < count) {
                    const int t = min(k * kWarps * 32 + tid, count - 1);
                    const int pr = p_start + (t >> 5);
                    const int b = (((pr < ppr ? pr : pr - ppr) * 32 + (t & 31)) >> 2) + 8 * pair0;
                    values_slot_tagged(a.x + 32 * b, xg.wait_tagged - 32 * b, b & 3, lane & 3, xw[k], xv[k]);
                }
        } else {
#pragma unroll
            for (int k = 0; k < kPasses; ++k)
                if (k * kWarps * 32 < count) {
                    const int t = min(k * kWarps * 32 + tid, count - 1);
                    const int pr = p_start + (t >> 5);
                    const int b = (((pr < ppr ? pr : pr - ppr) * 32 + (t & 31)) >> 2) + 8 * pair0;
                    load_slot(a.x + 32 * b, b & 3, lane & 3, xv[k]);
                }
        }
#pragma unroll
        for (int k = 0; k < kPasses; ++k)
            if (k * kWarps * 32 < count) {
                const int t0 = k * kWarps * 32 + tid, t = min(t0, count - 1);
                const int pr = p_start + (t >> 5);
                const int br = ((pr < ppr ? pr : pr - ppr) * 32 + (t & 31)) >> 2;  // block within the part
                store_slot(xv[k], xrec + (br >> 2) * kRecBytes, br & 3, lane & 3, t0 < count);
            }
    }
    for (int i = tid; i < a.max_tiles * kWarps * kTileRows; i += kWarps * 32) part[i] = 0.f;
    consumer_sync();
    // every consumer thread has read this launch's epoch: count the block in
    // now (the last one raises the exchange's epoch, which only kernels after
    // this launch read), so the count's round trip is not on the launch's tail
    if (kGather && xg.ranks > 0 && tid == 0) count_launch(xg.counter, a.grid, epoch);

    const int g = lane >> 2, c = lane & 3;
    // The five words lane c loads from each of its rows, as byte offsets in
    // a 72-byte group: A = 4c+4 (block 0; lane 3: block 1's first word, the
    // partner of its block-0 ends), B = 4c+20 (block 1), C = 4c+36 (block 2;
    // lane 0: the word holding block 2's first two nibble bytes), D = 4c+56
    // (block 3) and E = 52, 16, 36, 0 for lanes 0..3 (the other half of a
    // split block-0/block-2 word, and the word holding the scale d of the
    // lane's block beta(c)).  A-D are one base register plus immediates.
    const uint32_t offE = (c == 0 ? 52u : c == 1 ? 16u : c == 2 ? 36u : 0u) - 4u * c;  // relative to 4c
    const uint32_t selA = c == 3 ? 0x1076u : 0x3210u;  // lane 3: {w0.b2, w0.b3, w4.b0, w4.b1}
    const uint32_t selC = c == 0 ? 0x5432u : 0x3210u;  // lane 0: {w9.b2, w9.b3, w13.b0, w13.b1}
    const uint32_t selD = c >= 2 ? 0x1010u : 0x3232u;  // scale half: lanes 2, 3 low, 0, 1 high
    // B-fragment offsets inside a record for the MMAs of blocks 0..3
    uint32_t boff[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) boff[b] = (g >> 1) == beta_inv(b) ? (g >> 1) * 128 + (g & 1) * 64 + c * 16 : kZeroOff;

    // A row tile is finished by one warp after every warp's partial sums are
    // in shared memory.  The finishing warp (lanes 0-15, one row each) sums
    // the warps' partials in warp order, then
    //  * stores Y if this CTA holds all of the tile's units;
    //  * publishes the sum if a lower CTA holds the tile's first units (that
    //    CTA finishes the tile; for this CTA it is always its first tile);
    //  * otherwise (the tile continues in higher CTAs) adds the sums those
    //    CTAs published, in CTA order, and stores Y.
    auto finish_tile = [&](int ts) {
        if (lane >= kTileRows) return;
        const int t = t_first + ts;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += part[(ts * kWarps + w) * kTileRows + lane];
        const int tb = t * ppr, te = tb + ppr;
        const int row = t * kTileRows + lane;
        if (tb < u0) return;  // the producer warp published this CTA's sum of the tile
        if (te > u1) {
            // the sums of the higher CTAs that hold the rest of the tile, in CTA order
            bool ok = false;
            for (uint32_t i = 0; i < kWaitBudget && !ok; ++i) ok = mbar_try_wait(peers_in, 0);
            if (!ok) atomicExch(a.err, kErrPeerTimeout);
            const int last = cta_of(static_cast<uint32_t>(te - 1), units, grid_p);
            for (int q = 0; q < last - cta; ++q) v += peer[q * kTileRows + lane];
        }
        if (a.parts > 1) {
            // the row tile's sum over K parts: parts 0 .. parts-2 publish theirs,
            // the last part's finishing CTA adds them in part order, then its own
            unsigned long long *vt = a.vt + static_cast<size_t>(t) * (a.parts - 1) * kTileRows + lane;
            if (part_s + 1 < a.parts) {
                st_relaxed(vt + part_s * kTileRows, kPresent | __float_as_uint(v));
                return;
            }
            float sum = 0.f;
            for (int q = 0; q + 1 < a.parts; ++q) {
                unsigned long long w = ld_relaxed(vt + q * kTileRows);
                for (uint32_t spin = 0; !(w & kPresent); ++spin) {
                    if (spin >= kPeerBudget) {
                        atomicExch(a.err, kErrPeerTimeout);
                        break;
                    }
                    __nanosleep(64);
                    w = ld_relaxed(vt + q * kTileRows);
                }
                const float f = __uint_as_float(static_cast<uint32_t>(w));
                sum = q == 0 ? f : sum + f;
                st_relaxed(vt + q * kTileRows, 0ull);
            }
            v = sum + v;
        }
        if (row < a.n) {
            a.y[row] = v;
            // fused all-gather: the row as a tagged word into every rank's tag array
            if (kGather) {
                const unsigned long long w = tag_word(v, epoch);
                for (int r = 0; r < xg.ranks; ++r) st_tag(xg.tags[r] + row, w);
            }
        }
    };

    // boxes of this CTA: the first segment, the full row tiles, the last segment
    const int nboxes = t_first == t_last ? boxes_in(p_end - p_first)
                                         : boxes_in(ppr - p_first) + (t_last - t_first - 1) * boxes_in(ppr) +
                                               boxes_in(p_end);
    const uint32_t ring_u = smem_u32(ring), xrec_u = smem_u32(xrec);
    // Warp 4r + q takes unit slot q of boxes r, r + Q, r + 2Q, ... (Q quads):
    // box j sits in stage j mod 16.  A warp never meets a stage two phases
    // behind the box it waits for: its previous box was issued after box
    // j - 16 (Q < 16), whose stage reuse needed box j - 32 consumed.
    const int quad_r = warp >> 2, slot_q = warp & 3;  // quad of the warp, its unit slot in a box
    float acc0 = 0.f, acc1 = 0.f;  // rows g and g + 8 of the current row tile
    int cur = -1;
    bool past_first = false;  // arrived on first_done
    auto flush = [&](int t) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if (c == 0) {
            float *dst = part + (t * kWarps + warp) * kTileRows;
            dst[g] += acc0;
            dst[g + 8] += acc1;
        }
        acc0 = 0.f;
        acc1 = 0.f;
    };
    for (int j = quad_r; j < nboxes && j < a.max_boxes; j += kQuads) {
        const int s = j % kStages;
        if (!mbar_wait(&full[s], (j / kStages) & 1, a.err, kErrBulkTimeout)) break;
        const uint32_t info = box_tab[j];
        const int width = static_cast<int>(info >> 24);
        if (!past_first && (info & 0xffffu) != 0) {
            // this warp is done with the first row tile: its sums go to shared
            // memory now, for the producer warp's early publish
            if (cur == 0) {
                flush(0);
                cur = -1;
            }
            past_first = true;
            mbar_arrive(first_done);
        }
        if (slot_q < width) {
            const int tile_l = static_cast<int>(info & 0xffffu), pair = static_cast<int>((info >> 16) & 0xffu) + slot_q;
            if (tile_l != cur) {
                if (cur >= 0) flush(cur);
                cur = tile_l;
            }
            const uint32_t pitch = 4 * box_words(width);
            // this lane's rows g and g+8 of the unit, at byte 4c of each group
            const uint32_t ra = ring_u + s * kStageBytes + slot_q * kPairBytes + g * pitch + 4 * c;
            const uint32_t rows[2] = {ra, ra + 8 * pitch};
            const uint32_t recp = xrec_u + pair * 2 * kRecBytes;
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
                const uint32_t rec = recp + grp * kRecBytes;
                uint32_t wq[2][4], dh[2];  // [row][block] nibble words, scale halves
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const uint32_t ro = rows[r];
                    const uint32_t A = grp ? lds_at<72 + 4>(ro) : lds_at<4>(ro);
                    const uint32_t B = grp ? lds_at<72 + 20>(ro) : lds_at<20>(ro);
                    const uint32_t C = grp ? lds_at<72 + 36>(ro) : lds_at<36>(ro);
                    const uint32_t D = grp ? lds_at<72 + 56>(ro) : lds_at<56>(ro);
                    const uint32_t E = grp ? lds_at<72>(ro + offE) : lds_at<0>(ro + offE);
                    wq[r][0] = __byte_perm(A, E, selA);
                    wq[r][1] = B;
                    wq[r][2] = __byte_perm(C, E, selC);
                    wq[r][3] = D;
                    dh[r] = __byte_perm(E, E, selD);
                }
                float d0[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint4 xf = lds128(rec + boff[b]);
                    uint32_t t0[4], t1[4];
                    decode_word(wq[0][b], t0);
                    decode_word(wq[1][b], t1);
                    mma16816(d0, t0[0], t1[0], t0[1], t1[1], xf.x, xf.y);
                    mma16816(d0, t0[2], t1[2], t0[3], t1[3], xf.z, xf.w);
                }
                const float sig = ldsf(rec + kScaleOff + 4 * c);
                const float s0 = __fmul_rn(half_bits_to_float(static_cast<uint16_t>(dh[0])), sig);
                const float s1 = __fmul_rn(half_bits_to_float(static_cast<uint16_t>(dh[1])), sig);
                acc0 = fmaf(s0, d0[0] + d0[1], acc0);
                acc1 = fmaf(s1, d0[2] + d0[3], acc1);
            }
            // release this unit's slot of the stage; the proxy fence orders
            // this warp's reads before the next TMA write into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    if (cur >= 0) flush(cur);
    if (!past_first) mbar_arrive(first_done);
    consumer_sync();  // every warp's partials are in shared memory
    for (int ts = warp; ts <= t_last - t_first; ts += kWarps) finish_tile(ts);
}

// The end of a sharded sequence (launch_gather_wait): waits for the first
// `count` words of this rank's tag array of an exchange to carry this rank's
// current epoch of it, and stores their values as the exchange's plain rows.
__global__ void __launch_bounds__(256) gather_wait_kernel(const unsigned long long *tags, float *y, long long count,
                                                          const unsigned *counter, int *err) {
    pdl_wait_prior();  // the counter belongs to the kernels that stored into the exchange
    const unsigned epoch = exchange_epoch(counter);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = await_tag(tags + i, ld_tag(tags + i), epoch, err);
}

struct Q4MmaPlan {
    int grid, tiles, ppr, parts, max_tiles, max_boxes, rec_groups;
    int part_pair[kMaxParts + 1], part_cta[kMaxParts + 1];
    long long units;
    size_t smem;
};

bool q4_mma_plan(Q4MmaPlan &p, int k, int n, const DeviceInfo &dev) {
    if (k % 256 != 0 || n <= 0) return false;
    p.tiles = (n + kTileRows - 1) / kTileRows;
    p.ppr = k / 256;
    p.units = static_cast<long long>(p.tiles) * p.ppr;
    p.grid = static_cast<int>(p.units < dev.sm_count ? p.units : dev.sm_count);
    if (p.units * (p.grid + 1) >= (1ll << 32)) return false;  // the kernel's index math is 32-bit
    if (p.tiles >= (1 << 16)) return false;                    // box table: 16-bit tile index
    // K parts of at most kPartPairs pairs, their boundaries on multiples of
    // four pairs where that keeps every part within kPartPairs (a row tile's
    // part is then streamed as full 4-unit boxes, but for the last one), and
    // CTAs in proportion to the parts' units
    p.parts = (p.ppr + kPartPairs - 1) / kPartPairs;
    if (p.parts > kMaxParts) return false;
    bool aligned = true;
    for (int s = 0; s <= p.parts; ++s) {
        p.part_pair[s] = s == p.parts ? p.ppr : (2 * s * p.ppr + 4 * p.parts) / (8 * p.parts) * 4;
        if (s > 0 && (p.part_pair[s] - p.part_pair[s - 1] < 1 || p.part_pair[s] - p.part_pair[s - 1] > kPartPairs))
            aligned = false;
    }
    for (int s = 0; s <= p.parts; ++s) {
        if (!aligned) p.part_pair[s] = s * p.ppr / p.parts;
        p.part_cta[s] = static_cast<int>(static_cast<long long>(p.grid) * p.part_pair[s] / p.ppr);
    }
    long long per = 0;  // units of the largest CTA range
    int min_ppr = p.ppr, max_ppr = 0;
    for (int s = 0; s < p.parts; ++s) {
        const int g = p.part_cta[s + 1] - p.part_cta[s], pp = p.part_pair[s + 1] - p.part_pair[s];
        const long long u = static_cast<long long>(p.tiles) * pp;
        if (g < 1 || pp < 1 || g > u) return false;  // every CTA holds at least one unit
        per = std::max(per, (u + g - 1) / g);
        min_ppr = std::min(min_ppr, pp);
        max_ppr = std::max(max_ppr, pp);
    }
    p.max_tiles = static_cast<int>((per + min_ppr - 1) / min_ppr + 1);
    p.max_boxes = static_cast<int>(per / kMaxBoxPairs + p.max_tiles + 1);  // >= the boxes of any range
    p.rec_groups = 2 * max_ppr;
    p.smem = static_cast<size_t>(kStages) * kStageBytes + static_cast<size_t>(p.rec_groups) * kRecBytes +
             sizeof(float) * (p.max_tiles * kWarps + kMaxPeers) * kTileRows + 16 * kStages + 16 +
             4 * static_cast<size_t>(p.max_boxes);
    return p.smem + 1024 <= static_cast<size_t>(dev.smem_optin);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// Tensor maps of a weight matrix, cached by (pointer, k, n): enough entries
// for the weights a serving loop or a sharded bench rotates through, so that
// the maps are encoded once per weight.  Called with the library's runtime
// mutex held.
constexpr int kMapCache = 128;
bool weight_maps(Q4MmaMaps &out, const void *w, int k, int n) {
    struct Entry {
        const void *w = nullptr;
        int k = 0, n = 0;
        Q4MmaMaps maps;
    };
    static Entry cache[kMapCache];
    static int next = 0;
    for (const Entry &e : cache)
        if (e.w == w && e.k == k && e.n == n) {
            out = e.maps;
            return true;
        }
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t row_bytes = static_cast<cuuint64_t>(k / 32) * 18;
    cuuint64_t dims[2] = {row_bytes / 4, static_cast<cuuint64_t>(n)};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t estr[2] = {1, 1};
    Q4MmaMaps maps;
    for (int width = 1; width <= kMaxBoxPairs; ++width) {
        cuuint32_t box[2] = {static_cast<cuuint32_t>(box_words(width)), kTileRows};
        if (fn(&maps.box[width - 1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    cache[next].w = w;
    cache[next].k = k;
    cache[next].n = n;
    cache[next].maps = maps;
    next = (next + 1) % kMapCache;
    out = maps;
    return true;
}

}  // namespace

size_t q4_mma_scratch_bytes(int k, int n, int batch, const DeviceInfo &dev) {
    Q4MmaPlan p;
    if (batch != 1 || !q4_mma_plan(p, k, n, dev)) return 0;
    // per CTA the sums of a shared row tile, per row tile the sums of K parts 0 .. parts-2
    return (static_cast<size_t>(p.grid) + static_cast<size_t>(p.tiles) * (p.parts - 1)) * kTileRows *
           sizeof(unsigned long long);
}

cudaError_t launch_q4_mma_gemv(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    Q4MmaPlan p;
    if (r.wt != 2 || r.batch != 1 || !r.fixup || !q4_mma_plan(p, r.k, r.n, dev)) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(r.w) & 15) || (reinterpret_cast<uintptr_t>(r.x) & 15))
        return cudaErrorNotSupported;
    if (r.fixup_bytes < q4_mma_scratch_bytes(r.k, r.n, 1, dev)) return cudaErrorNotSupported;
    Q4MmaMaps maps;
    if (!weight_maps(maps, r.w, r.k, r.n)) return cudaErrorNotSupported;
    Q4MmaArgs a{};
    a.x = r.x;
    a.y = r.y;
    a.slot = static_cast<unsigned long long *>(r.fixup);
    a.vt = a.slot + static_cast<size_t>(p.grid) * kTileRows;
    a.err = dev.err;
    a.k = r.k;
    a.n = r.n;
    a.tiles = p.tiles;
    a.grid = p.grid;
    a.parts = p.parts;
    for (int s = 0; s <= kMaxParts; ++s) {
        a.part_pair[s] = s <= p.parts ? p.part_pair[s] : p.ppr;
        a.part_cta[s] = s <= p.parts ? p.part_cta[s] : p.grid;
    }
    a.rec_groups = p.rec_groups;
    a.prefetch = r.prefetch_weights ? 1 << 30 : 0;
    a.max_tiles = p.max_tiles;
    a.max_boxes = p.max_boxes;
    const bool gather = r.gather != nullptr;
    void (*kernel)(const Q4MmaMaps, const Q4MmaArgs, const GatherLaunch) =
        gather ? q4_mma_gemv_kernel<true> : q4_mma_gemv_kernel<false>;
    const GatherLaunch xg = gather ? *r.gather : GatherLaunch{};
    static int configured[2][64] = {};
    int devno = 0;
    cudaGetDevice(&devno);
    if (devno < 0 || devno >= 64 || configured[gather][devno] < static_cast<int>(p.smem)) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(p.smem));
        if (e != cudaSuccess) return e;
        if (devno >= 0 && devno < 64) configured[gather][devno] = static_cast<int>(p.smem);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, maps, a, xg);
}

cudaError_t launch_gather_wait(const unsigned long long *tags, float *y, long long count, const unsigned *counter,
                               const DeviceInfo &dev, cudaStream_t stream) {
    if (!tags || !y || !counter || count < 1) return cudaErrorInvalidValue;
    const long long want = (count + 255) / 256;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(want < dev.sm_count * 2LL ? want : dev.sm_count * 2LL));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gather_wait_kernel, tags, y, count, counter, dev.err);
}

}  // namespace k200
