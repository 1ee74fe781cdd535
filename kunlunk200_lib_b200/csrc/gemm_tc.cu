// Batched matmul on the 5th-generation tensor cores (tcgen05, sm_100a):
// Y[b, n] = X[b, :] . W[n, :] for batches of activation columns, the
// "matmul" of src/k200.cpp:268-279 when batch is large enough that the
// weight rows are reused across columns (the streaming GEMV kernels re-read W
// once per pair of columns).
//
// One CTA computes a tile of 128 weight rows x NB activation columns:
//  * warp 0 (one thread) streams the K dimension through a ring of stages
//    with 2-D TMA copies in the 128-byte-swizzled K-major layout the MMA reads
//    directly: the weight tile (128 rows x 128 bytes) and up to two
//    activation operands (NB rows x 128 bytes);
//  * warp 1 allocates tensor memory, and one of its threads issues the
//    tcgen05.mma instructions (M = 128, N = NB) for every 128-byte K step and
//    releases each stage with tcgen05.commit when its MMAs are done;
//  * warps 2-5 wait for the last commit, read the accumulators from tensor
//    memory (tcgen05.ld, 32 lanes = 32 weight rows per warp) and write Y,
//    consecutive lanes writing consecutive outputs of a column.
//
// Operand sets:
//  * rowwise-int8 (gemm_i8_kernel): weights x the two int8 activation components of the
//    per-tensor two-pass quantiser (src/k200.cpp:209-239), kind::i8 with two
//    int32 accumulators; the epilogue is the combine of
//    kernels/kunlun-combine.xpu:19, so results are bit-exact with the
//    reference's integer dot products.
//  * f16 weights (gemm_f16_kernel): exact f16 weights x the activations split
//    into f16 hi + lo parts after a power-of-two scaling per activation row
//    (split_rows below; x = 2^e * (hi + lo) to about 22 bits), kind::f16.
//    The tensor cores' f32 accumulation aligns each MMA to the running sum,
//    which over K = 8192 costs ~2^-21 of sum|w*x| (measured); so the MMAs
//    of every 4 K steps go to one of two tensor-memory slots and the
//    epilogue warps add each finished slot into f32 registers while the
//    other slot fills.  The reference computes these products in FP32
//    (kernels/kunlun-matvec.xpu); the difference is the ~2^-22 split plus
//    the order of the f32 sums.
//  * Q4_0 weights (gemm_q4_kernel): four dequantiser warps, one weight row
//    per thread, read each K step's two blocks (36 bytes) straight from
//    global memory and write W' = d*(q-8) into shared memory as exact f16
//    hi + lo halves (hi = f16(d*(q-8)), lo = fma(d, q-8, -hi): the residual
//    has at most 3 significant bits) in the swizzled layout the MMA reads.
//    The raw blocks arrive by TMA in boxes of 128 rows x 288 bytes (eight
//    K steps) through a ring of 2-3 slots filled by a dedicated producer
//    warp; each dequantiser reads its row's bytes with 16-byte shared loads.
//    (Per-thread global loads of the 36-byte row pieces touch 32 sectors per
//    instruction and saturate L1; a TMA box costs the copy engine about the
//    same per row whatever the row's width, so rows are made wide.)
//    Three products per K slice: hi*x_hi + hi*x_lo + lo*x_hi (lo*x_lo is
//    below 2^-21 of the term), issued as two MMAs: W hi against the x hi and
//    x lo tiles as one 2NB-row operand, and W lo against x hi.  (An MMA of
//    M = 128, K = 16 occupies the tensor pipe for at least ~45 cycles
//    whatever N is below 128, so fewer, wider MMAs are what small batches
//    need.)  Each 16-byte chunk holds one decoded nibble
//    word in the order the decode produces, and the activations are split
//    into the same permuted K order (q4_pos below), so the sums are those of
//    the natural order.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

constexpr int kTileM = 128;       // weight rows per CTA (MMA M)
constexpr int kStepBytes = 128;   // K bytes per pipeline step (one 128-byte swizzle atom)
constexpr int kThreadsTc = 192;   // 6 warps: TMA, MMA, 4 x epilogue

struct TcMaps {
    CUtensorMap a;    // weights [n][k] (bytes)
    CUtensorMap b0;   // activation operand 0 [batch][k]
    CUtensorMap b1;   // activation operand 1 [batch][k]
};

struct TcArgs {
    const uint8_t *w;        // q4_0: weight rows (read by the dequantisers)
    long long row_bytes;     // q4_0: bytes per weight row
    float *y;
    const float *row_scale;  // rowwise-int8: per weight row scale
    const float *act_max;    // rowwise-int8: {max0, max1}
    const float *col_scale;  // f16: 2^e of each activation row
    int *err;
    int k, n, batch, y_stride;
    int nb;                  // activation columns per CTA (MMA N, multiple of 16)
    int stages;
    int ksteps;
    uint32_t tmem_cols;      // allocated tensor-memory columns (power of two >= 32)
    int raw_slots;           // q4: raw weight boxes in flight
    // Persistent schedule over the (tile, chunk) space, chunk = kChunkSteps K
    // steps: CTA c takes iterations [c * iters / grid, (c + 1) * iters / grid).
    // Tile t is row tile t / ncolt, column tile t % ncolt.  With grid = tiles
    // every CTA owns one whole tile; with grid = the SM count (stream-K) a tile
    // can be split between consecutive CTAs, whose partial accumulators go to
    // `partials` (two slots per CTA: its first and its last tile) and are
    // summed in CTA order by the CTA that arrives last (`counters`, zero
    // between launches).
    long long iters;
    int grid, chunks, ncolt;
    int *counters;
    void *partials;
};

constexpr int kChunkSteps = 4;  // K steps per schedule iteration (and per f16/q4 tensor-memory chunk)

// One CTA's run of chunks inside one tile.
struct Seg {
    int t, mt, nt;    // tile, its row tile and column tile
    int ks0, ks1;     // K steps [ks0, ks1)
    bool whole;       // the CTA computes the whole tile
    int slot;         // partial slot when not whole
};

__device__ __forceinline__ long long sk_begin(const TcArgs &a, int cta) { return cta * a.iters / a.grid; }
// CTA whose range holds iteration it
__device__ __forceinline__ int sk_owner(const TcArgs &a, long long it) {
    return static_cast<int>(((it + 1) * a.grid - 1) / a.iters);
}
// Partial slot of CTA c's segment of tile t: slot 0 for its first tile, 1 for its last.
__device__ __forceinline__ int sk_slot(const TcArgs &a, int c, int t) {
    return 2 * c + (t == static_cast<int>(sk_begin(a, c) / a.chunks) ? 0 : 1);
}

struct SkWalk {
    long long i, i1;
    __device__ explicit SkWalk(const TcArgs &a) : i(sk_begin(a, blockIdx.x)), i1(sk_begin(a, blockIdx.x + 1)) {}
    __device__ bool next(const TcArgs &a, Seg &s) {
        if (i >= i1) return false;
        const long long t = i / a.chunks;
        const long long e = min(i1, (t + 1) * a.chunks);
        const int ca = static_cast<int>(i - t * a.chunks), cb = static_cast<int>(e - t * a.chunks);
        s.t = static_cast<int>(t);
        s.mt = s.t / a.ncolt;
        s.nt = s.t - s.mt * a.ncolt;
        s.ks0 = ca * kChunkSteps;
        s.ks1 = min(a.ksteps, cb * kChunkSteps);
        s.whole = ca == 0 && cb == a.chunks;
        s.slot = sk_slot(a, blockIdx.x, s.t);
        i = e;
        return true;
    }
};

// The four epilogue warps (2..5) meet here.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// After this CTA's epilogue threads stored their partials of a split tile:
// counts the segment in and returns true in every epilogue thread of the CTA
// that arrived last (it then owns the tile's final sum; the count is reset).
// Every epilogue thread calls it for every split segment, also after a wait
// that ran out (ok false: nothing is counted), so the named barriers always
// meet.
__device__ __forceinline__ bool sk_arrive(const TcArgs &a, const Seg &s, int *flag, bool ok) {
    __threadfence();  // this thread's partial stores before the count (device scope)
    epi_sync();
    if (threadIdx.x == 64) *flag = 0;
    if (threadIdx.x == 64 && ok) {
        const long long it0 = static_cast<long long>(s.t) * a.chunks;
        const int nseg = sk_owner(a, it0 + a.chunks - 1) - sk_owner(a, it0) + 1;
        __threadfence();
        const int prev = atomicAdd(a.counters + s.t, 1);
        const int last = prev + 1 == nseg;
        if (last) {
            __threadfence();
            a.counters[s.t] = 0;
        }
        *flag = last;
    }
    epi_sync();
    return *flag != 0;
}

// ---- tcgen05 primitives ----------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the
// 128-byte swizzled layout TMA writes (8-row groups of 1024 bytes): start
// address, leading offset 16 B (unused for swizzled K-major), stride 1024 B
// between 8-row groups, descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3fff);
    d |= static_cast<uint64_t>(1) << 16;                 // LBO = 16 B
    d |= static_cast<uint64_t>(1024 >> 4) << 32;         // SBO = 1024 B
    d |= static_cast<uint64_t>(1) << 46;                 // version
    d |= static_cast<uint64_t>(2) << 61;                 // SWIZZLE_128B
    return d;
}

// Instruction descriptor: D format (0 f16, 1 f32, 2 s32), A/B formats, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, int m, int n) {
    return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ---- rowwise int8 --------------------------------------------------------------
// Accumulators of one segment: p0 = W . q0 in columns [0, nb), p1 = W . q1 in
// [nb, 2 nb).  The next segment's first MMA waits until the epilogue has
// read them (accfree).
__global__ void __launch_bounds__(kThreadsTc, 1) gemm_i8_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned stages: [A 128 x 128 B][B0 nb x 128 B][B1 nb x 128 B]
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t a_bytes = kTileM * kStepBytes, b_bytes = a.nb * kStepBytes;
    const uint32_t stage_bytes = a_bytes + 2 * b_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.stages * stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *accum = empty + a.stages;  // a segment's accumulators are final
    uint64_t *accfree = accum + 1;       // the epilogue has read them (4 arrivals)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accfree + 1);
    int *flag = reinterpret_cast<int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        mbar_init(accfree, 4);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            pdl_wait_prior();
            SkWalk walk(a);
            Seg sg;
            int g = 0;  // K steps issued by this CTA (ring position)
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                const int m0 = sg.mt * kTileM, n0 = sg.nt * a.nb;
                for (int ks = sg.ks0; ks < sg.ks1; ++ks, ++g) {
                    const int s = g % a.stages;
                    if (g >= a.stages &&
                        !mbar_wait_sleep(&empty[s], ((g / a.stages) - 1) & 1, a.err, kErrBulkTimeout, 64)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = base + s * stage_bytes;
                    mbar_arrive_expect_tx(&full[s], stage_bytes);
                    tma_2d(st, &maps.a, ks * kStepBytes, m0, &full[s]);
                    tma_2d(st + a_bytes, &maps.b0, ks * kStepBytes, n0, &full[s]);
                    tma_2d(st + a_bytes + b_bytes, &maps.b1, ks * kStepBytes, n0, &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = instr_desc(2, 1, 1, kTileM, a.nb);  // s32 <- s8 x s8
            // the two activation components are adjacent nb-row tiles: one 2nb-wide MMA when it fits
            const bool merged = 2 * a.nb <= 256;
            const uint32_t idesc2 = instr_desc(2, 1, 1, kTileM, merged ? 2 * a.nb : a.nb);
            SkWalk walk(a);
            Seg sg;
            int g = 0, seg = 0;
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                if (seg > 0 && !mbar_wait(accfree, (seg - 1) & 1, a.err, kErrMmaTimeout)) break;
                tc_fence_after();
                for (int ks = sg.ks0; ks < sg.ks1; ++ks, ++g) {
                    const int s = g % a.stages;
                    if (!mbar_wait(&full[s], (g / a.stages) & 1, a.err, kErrBulkTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = base + s * stage_bytes;
                    const uint64_t da = sw128_desc(st), db0 = sw128_desc(st + a_bytes),
                                   db1 = sw128_desc(st + a_bytes + b_bytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K per 128-byte step: +2 in the address field
                        const uint32_t acc = (ks != sg.ks0) || kk != 0;
                        if (merged) {
                            mma_i8(taddr, da + 2 * kk, db0 + 2 * kk, idesc2, acc);
                        } else {
                            mma_i8(taddr, da + 2 * kk, db0 + 2 * kk, idesc, acc);
                            mma_i8(taddr + a.nb, da + 2 * kk, db1 + 2 * kk, idesc, acc);
                        }
                    }
                    mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
                }
                mma_commit(accum);
                ++seg;
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warps 2..5 -> TMEM lane quarters 2,3,0,1 ----------------
        const int quarter = warp & 3;
        const int rt = quarter * 32 + lane;  // row of the tile
        const uint32_t lane_addr = taddr + (static_cast<uint32_t>(quarter * 32) << 16);
        const float s0 = __fdiv_rn(a.act_max[0], 127.0f), s1 = __fdiv_rn(a.act_max[1], 127.0f);
        SkWalk walk(a);
        Seg sg;
        int seg = 0;
        bool ok = true;  // false once a wait ran out: the rest only keeps the barriers in step
        while (walk.next(a, sg)) {
            ok = __all_sync(0xffffffffu, ok && mbar_wait_sleep(accum, seg & 1, a.err, kErrMmaTimeout, 128));
            tc_fence_after();
            const int row = sg.mt * kTileM + rt, n0 = sg.nt * a.nb;
            const float rs = row < a.n ? a.row_scale[row] : 0.f;
            int *part = static_cast<int *>(a.partials) + static_cast<size_t>(sg.slot) * 2 * a.nb * kTileM + rt;
            for (int c0 = 0; ok && c0 < a.nb; c0 += 16) {
                uint32_t p0[16], p1[16];
                tmem_ld16(lane_addr + c0, p0);
                tmem_ld16(lane_addr + a.nb + c0, p1);
                tmem_ld_wait();
                if (sg.whole) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int col = n0 + c0 + i;
                        if (row < a.n && col < a.batch) {
                            const float t0 = __fmul_rn(static_cast<float>(static_cast<int>(p0[i])), s0);
                            const float t1 = __fmul_rn(static_cast<float>(static_cast<int>(p1[i])), s1);
                            a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(__fadd_rn(t0, t1), rs);
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        part[(c0 + i) * kTileM] = static_cast<int>(p0[i]);
                        part[(a.nb + c0 + i) * kTileM] = static_cast<int>(p1[i]);
                    }
                }
            }
            // the accumulators are in registers or memory: the next segment may overwrite them
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accfree);
            if (!sg.whole && sk_arrive(a, sg, flag, ok)) {
                // the exact int32 sums of every CTA's segment (CTA order), then the combine;
                // 16 columns at a time so that the loads of a group are in flight together
                const long long it0 = static_cast<long long>(sg.t) * a.chunks;
                const int c_first = sk_owner(a, it0), c_last = sk_owner(a, it0 + a.chunks - 1);
                for (int c0 = 0; c0 < a.nb; c0 += 16) {
                    int q0[16], q1[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) q0[i] = q1[i] = 0;
                    for (int c = c_first; c <= c_last; ++c) {
                        const int *pp = static_cast<const int *>(a.partials) +
                                        static_cast<size_t>(sk_slot(a, c, sg.t)) * 2 * a.nb * kTileM + rt;
                        int v0[16], v1[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            v0[i] = __ldcg(pp + (c0 + i) * kTileM);
                            v1[i] = __ldcg(pp + (a.nb + c0 + i) * kTileM);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            q0[i] += v0[i];
                            q1[i] += v1[i];
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int col = n0 + c0 + i;
                        if (row < a.n && col < a.batch) {
                            const float t0 = __fmul_rn(static_cast<float>(q0[i]), s0);
                            const float t1 = __fmul_rn(static_cast<float>(q1[i]), s1);
                            a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(__fadd_rn(t0, t1), rs);
                        }
                    }
                }
            }
            ++seg;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, a.tmem_cols);
    }
}

// f16 weights, chunked accumulation; NB activation columns per CTA.
// Epilogue of the f16 and q4 kernels for one finished segment: sum[] holds
// the f32 sums of its chunks for this thread's row rt.  A whole tile is
// written (times each column's 2^e); a split one goes to the partial slot,
// and the CTA that completes the tile adds every segment's partial in CTA
// order and writes it.  sum[] is left zero.
template <int NB>
__device__ __forceinline__ void f32_segment_out(const TcArgs &a, const Seg &sg, int rt, float (&sum)[NB], int *flag,
                                                bool ok) {
    const int row = sg.mt * kTileM + rt, n0 = sg.nt * NB;
    if (sg.whole) {
        if (ok && row < a.n) {
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int col = n0 + i;
                if (col < a.batch) a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(sum[i], a.col_scale[col]);
            }
        }
    } else {
        float *part = static_cast<float *>(a.partials) + static_cast<size_t>(sg.slot) * NB * kTileM + rt;
        if (ok) {
#pragma unroll
            for (int i = 0; i < NB; ++i) part[i * kTileM] = sum[i];
        }
        if (sk_arrive(a, sg, flag, ok)) {
            const long long it0 = static_cast<long long>(sg.t) * a.chunks;
            const int c_first = sk_owner(a, it0), c_last = sk_owner(a, it0 + a.chunks - 1);
#pragma unroll
            for (int i = 0; i < NB; ++i) sum[i] = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
                const float *pp = static_cast<const float *>(a.partials) +
                                  static_cast<size_t>(sk_slot(a, c, sg.t)) * NB * kTileM + rt;
#pragma unroll
                for (int i = 0; i < NB; ++i) sum[i] = __fadd_rn(sum[i], __ldcg(pp + i * kTileM));
            }
            if (row < a.n) {
#pragma unroll
                for (int i = 0; i < NB; ++i) {
                    const int col = n0 + i;
                    if (col < a.batch)
                        a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(sum[i], a.col_scale[col]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) sum[i] = 0.f;
}

// Epilogue warps of the f16 and q4 kernels: drain every finished chunk of
// the two tensor-memory slots into sum[] and close each segment.
template <int NB>
__device__ __forceinline__ void f32_chunk_epilogue(const TcArgs &a, uint32_t taddr, uint64_t *tfull, uint64_t *tfree,
                                                   int *flag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3;
    const int rt = quarter * 32 + lane;
    const uint32_t lane_addr = taddr + (static_cast<uint32_t>(quarter * 32) << 16);
    float sum[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) sum[i] = 0.f;
    bool ok = true;  // false once a wait ran out: the rest only keeps the barriers in step
    SkWalk walk(a);
    Seg sg;
    int gc = 0;  // chunks drained by this CTA (slot and phase)
    while (walk.next(a, sg)) {
        const int nch = (sg.ks1 - sg.ks0 + kChunkSteps - 1) / kChunkSteps;
        for (int c = 0; c < nch; ++c, ++gc) {
            const int slot = gc & 1;
            ok = __all_sync(0xffffffffu, ok && mbar_wait_sleep(&tfull[slot], (gc >> 1) & 1, a.err, kErrMmaTimeout, 32));
            tc_fence_after();
            if (ok) {
#pragma unroll
                for (int c0 = 0; c0 < 2 * NB; c0 += 16) {
                    uint32_t p[16];
                    tmem_ld16(lane_addr + slot * 2 * NB + c0, p);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        sum[(c0 % NB) + i] = __fadd_rn(sum[(c0 % NB) + i], __uint_as_float(p[i]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfree[slot]);
        }
        f32_segment_out<NB>(a, sg, rt, sum, flag, ok);
    }
}

template <int NB>
__global__ void __launch_bounds__(kThreadsTc, 1) gemm_f16_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - smem_u32(smem_raw));
    // stage: [A 128 x 128 B][B0 NB x 128 B][B1 NB x 128 B]
    constexpr uint32_t a_bytes = kTileM * kStepBytes, b_bytes = NB * kStepBytes;
    constexpr uint32_t a_total = a_bytes;
    constexpr uint32_t stage_bytes = a_total + 2 * b_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.stages * stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *tfull = empty + a.stages;  // [2] a tensor-memory slot holds a finished chunk
    uint64_t *tfree = tfull + 2;         // [2] the epilogue has read a slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + 2);
    int *flag = reinterpret_cast<int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&tfull[t], 1);
            mbar_init(&tfree[t], 4);  // one arrival per epilogue warp
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait_prior();
            SkWalk walk(a);
            Seg sg;
            int g = 0;
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                const int m0 = sg.mt * kTileM, n0 = sg.nt * NB;
                for (int ks = sg.ks0; ks < sg.ks1; ++ks, ++g) {
                    const int s = g % a.stages;
                    if (g >= a.stages &&
                        !mbar_wait_sleep(&empty[s], ((g / a.stages) - 1) & 1, a.err, kErrBulkTimeout, 64)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = base + s * stage_bytes;
                    mbar_arrive_expect_tx(&full[s], stage_bytes);
                    tma_2d(st, &maps.a, ks * kStepBytes, m0, &full[s]);
                    tma_2d(st + a_total, &maps.b0, ks * kStepBytes, n0, &full[s]);
                    tma_2d(st + a_total + b_bytes, &maps.b1, ks * kStepBytes, n0, &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // f32 <- f16 x f16; x hi and x lo are adjacent NB-row tiles: one 2NB-wide MMA
            const uint32_t idesc = instr_desc(1, 0, 0, kTileM, 2 * NB);
            SkWalk walk(a);
            Seg sg;
            int g = 0, gc = 0;
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                for (int c0 = sg.ks0; ok && c0 < sg.ks1; c0 += kChunkSteps, ++gc) {
                    const int slot = gc & 1;
                    if (gc >= 2 && !mbar_wait(&tfree[slot], ((gc >> 1) - 1) & 1, a.err, kErrMmaTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = taddr + slot * 2 * NB;  // [W*x hi | W*x lo]
                    const int ks_end = min(sg.ks1, c0 + kChunkSteps);
                    for (int ks = c0; ks < ks_end; ++ks, ++g) {
                        const int s = g % a.stages;
                        if (!mbar_wait(&full[s], (g / a.stages) & 1, a.err, kErrBulkTimeout)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = base + s * stage_bytes;
                        const uint64_t da = sw128_desc(st);
                        const uint64_t db = sw128_desc(st + a_total);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) mma_f16(d, da + 2 * kk, db + 2 * kk, idesc, (ks != c0) || kk != 0);
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&tfull[slot]);
                }
            }
        }
        __syncwarp();
    } else {
        f32_chunk_epilogue<NB>(a, taddr, tfull, tfree, flag);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, a.tmem_cols);
    }
}

// ---- q4_0 with in-kernel dequantisation -------------------------------------
constexpr int kThreadsQ4 = 352;  // x TMA, MMA, 4 x epilogue, 4 x dequantiser, weight TMA
constexpr int kRawSteps = 8;                // K steps (pairs of blocks) per raw box
constexpr int kRawRow = 36 * kRawSteps;     // 288 bytes of one weight row per raw box
constexpr int kRawBox = kTileM * kRawRow;   // 36 KB
constexpr int kBarBytesQ4 = 1024;          // mbarriers and the TMEM slot

// Position of element e (0..31) of a block inside the block's 32 K positions
// after dequantisation: 16-byte chunk q (nibble bytes 4q..4q+3) holds
// elements 4q, 4q+2, 16+4q, 18+4q, 4q+1, 4q+3, 17+4q, 19+4q.
__host__ __device__ constexpr int q4_pos(int e) {
    const int hi = e >= 16, j = e & 15, q = j >> 2, b = j & 3;
    return 8 * q + ((b & 1) ? 4 : 0) + (hi ? 2 : 0) + (b >> 1);
}

// One nibble word (bytes b0..b3) -> the chunk's 8 values as f16 pairs of
// (v - 8): {lo(b0), lo(b2)}, {hi(b0), hi(b2)}, {lo(b1), lo(b3)}, {hi(b1), hi(b3)}.
__device__ __forceinline__ void q4_word_f16(uint32_t w, uint32_t (&t)[4]) {
    const uint32_t m = 0x64006400u;
    uint32_t a0, a1, a2, a3;
    const uint32_t w8 = w >> 8;
    asm("lop3.b32 %0, %1, 0x000F000F, %2, 0xEA;" : "=r"(a0) : "r"(w), "r"(m));
    asm("lop3.b32 %0, %1, 0x00F000F0, %2, 0xEA;" : "=r"(a1) : "r"(w), "r"(m));
    asm("lop3.b32 %0, %1, 0x000F000F, %2, 0xEA;" : "=r"(a2) : "r"(w8), "r"(m));
    asm("lop3.b32 %0, %1, 0x00F000F0, %2, 0xEA;" : "=r"(a3) : "r"(w8), "r"(m));
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(t[0]) : "r"(a0), "r"(0xE408E408u));                  // 1024+v - 1032
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(t[1]) : "r"(a1), "r"(0x2C002C00u), "r"(0xD480D480u));  // /16 - 72
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(t[2]) : "r"(a2), "r"(0xE408E408u));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(t[3]) : "r"(a3), "r"(0x2C002C00u), "r"(0xD480D480u));
}

// d*(v-8) for 8 values -> hi and lo chunks
__device__ __forceinline__ void q4_chunk(uint32_t w, uint32_t d2, uint4 &hi, uint4 &lo) {
    uint32_t t[4], h[4], l[4];
    q4_word_f16(w, t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(h[i]) : "r"(d2), "r"(t[i]));
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(l[i]) : "r"(d2), "r"(t[i]), "r"(h[i] ^ 0x80008000u));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <int NB>
__global__ void __launch_bounds__(kThreadsQ4, 1) gemm_q4_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - smem_u32(smem_raw));
    // stage: [W hi 128 x 128 B][W lo 128 x 128 B][x hi NB x 128 B][x lo NB x 128 B]
    constexpr uint32_t a_bytes = kTileM * kStepBytes, b_bytes = NB * kStepBytes;
    constexpr uint32_t stage_bytes = 2 * a_bytes + 2 * b_bytes;
    uint64_t *full_x = reinterpret_cast<uint64_t *>(smem + a.stages * stage_bytes);
    uint64_t *full_w = full_x + a.stages;
    uint64_t *empty = full_w + a.stages;
    uint64_t *tfull = empty + a.stages;
    uint64_t *tfree = tfull + 2;
    uint64_t *full_r = tfree + 2;         // raw box landed (TMA)
    uint64_t *empty_r = full_r + a.raw_slots;  // raw box read by all 128 dequantisers
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(empty_r + a.raw_slots);
    int *flag = reinterpret_cast<int *>(tmem_slot + 1);
    const uint32_t raw_u = base + a.stages * stage_bytes + kBarBytesQ4;  // raw ring [slot][row][288 B]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&full_w[s], 128);  // one arrival per dequantiser thread
            mbar_init(&empty[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&tfull[t], 1);
            mbar_init(&tfree[t], 4);
        }
        for (int r = 0; r < a.raw_slots; ++r) {
            mbar_init(&full_r[r], 1);
            mbar_init(&empty_r[r], 128);
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;

    if (warp == 10) {
        // ---------------- raw weight boxes by TMA ----------------
        // A segment's K steps [ks0, ks1) are covered by boxes of kRawSteps
        // steps from ks0 (ks0 is a multiple of four, so a box starts on a
        // 16-byte boundary: 144 bytes per four steps); the last box may run
        // past the segment (the dequantisers skip those steps) or past the
        // row (zero fill).
        if (lane == 0) {
            pdl_wait_prior();
            SkWalk walk(a);
            Seg sg;
            int gr = 0;  // boxes issued by this CTA (raw ring position)
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                const int m0 = sg.mt * kTileM;
                for (int ks = sg.ks0; ks < sg.ks1; ks += kRawSteps, ++gr) {
                    const int rs = gr % a.raw_slots;
                    if (gr >= a.raw_slots &&
                        !mbar_wait_sleep(&empty_r[rs], ((gr / a.raw_slots) - 1) & 1, a.err, kErrBulkTimeout, 64)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_r[rs], kRawBox);
                    tma_2d(raw_u + rs * kRawBox, &maps.a, ks * (kRawRow / kRawSteps / 4), m0, &full_r[rs]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 0) {
        // ---------------- activations by TMA ----------------
        if (lane == 0) {
            pdl_wait_prior();
            SkWalk walk(a);
            Seg sg;
            int g = 0;
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                const int n0 = sg.nt * NB;
                for (int ks = sg.ks0; ks < sg.ks1; ++ks, ++g) {
                    const int s = g % a.stages;
                    if (g >= a.stages &&
                        !mbar_wait_sleep(&empty[s], ((g / a.stages) - 1) & 1, a.err, kErrBulkTimeout, 64)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = base + s * stage_bytes;
                    mbar_arrive_expect_tx(&full_x[s], 2 * b_bytes);
                    tma_2d(st + 2 * a_bytes, &maps.b0, ks * kStepBytes, n0, &full_x[s]);
                    tma_2d(st + 2 * a_bytes + b_bytes, &maps.b1, ks * kStepBytes, n0, &full_x[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // x hi and x lo are adjacent NB-row tiles: one 2NB-row operand
            const uint32_t idesc2 = instr_desc(1, 0, 0, kTileM, 2 * NB), idesc1 = instr_desc(1, 0, 0, kTileM, NB);
            SkWalk walk(a);
            Seg sg;
            int g = 0, gc = 0;
            bool ok = true;
            while (ok && walk.next(a, sg)) {
                for (int c0 = sg.ks0; ok && c0 < sg.ks1; c0 += kChunkSteps, ++gc) {
                    const int slot = gc & 1;
                    if (gc >= 2 && !mbar_wait(&tfree[slot], ((gc >> 1) - 1) & 1, a.err, kErrMmaTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = taddr + slot * 2 * NB;  // [W*x hi | W hi*x lo]
                    const int ks_end = min(sg.ks1, c0 + kChunkSteps);
                    for (int ks = c0; ks < ks_end; ++ks, ++g) {
                        const int s = g % a.stages;
                        const uint32_t par = (g / a.stages) & 1;
                        if (!mbar_wait(&full_x[s], par, a.err, kErrBulkTimeout) ||
                            !mbar_wait(&full_w[s], par, a.err, kErrBulkTimeout)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = base + s * stage_bytes;
                        const uint64_t dh = sw128_desc(st), dl = sw128_desc(st + a_bytes);
                        const uint64_t xh = sw128_desc(st + 2 * a_bytes);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            mma_f16(d, dh + 2 * kk, xh + 2 * kk, idesc2, (ks != c0) || kk != 0);
                            mma_f16(d, dl + 2 * kk, xh + 2 * kk, idesc1, 1);
                        }
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&tfull[slot]);
                }
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- epilogue: chunk sums in f32 registers ----------------
        f32_chunk_epilogue<NB>(a, taddr, tfull, tfree, flag);
    } else {
        // ---------------- dequantisers: one weight row per thread ----------------
        const int rt = threadIdx.x - 192;  // row in the tile
        const uint32_t row_off = (rt >> 3) * 1024 + (rt & 7) * 128;  // swizzled tile row
        const uint32_t sw = rt & 7;
        SkWalk walk(a);
        Seg sg;
        int g = 0, gr = 0;
        bool ok = true;
        while (ok && walk.next(a, sg)) {
            for (int kb = sg.ks0; ok && kb < sg.ks1; kb += kRawSteps, ++gr) {
                const int rs = gr % a.raw_slots;
                if (!mbar_wait(&full_r[rs], (gr / a.raw_slots) & 1, a.err, kErrBulkTimeout)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int half = 0; half < kRawSteps / 4; ++half) {
                    uint32_t w[36];  // four K steps of this row: per step two blocks (2-byte scale + 16 nibble bytes)
                    const uint32_t rp = raw_u + rs * kRawBox + rt * kRawRow + half * 144;
#pragma unroll
                    for (int c = 0; c < 9; ++c)
                        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                     : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                                     : "r"(rp + 16 * c));
                    if (half == kRawSteps / 4 - 1) {
                        // order these generic reads before the copy engine's next write into the slot
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        mbar_arrive(&empty_r[rs]);
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int ks = kb + half * 4 + j;
                        if (!ok || ks >= sg.ks1) break;
                        const int s = g % a.stages;
                        if (g >= a.stages &&
                            !mbar_wait_sleep(&empty[s], ((g / a.stages) - 1) & 1, a.err, kErrBulkTimeout, 64)) {
                            ok = false;
                            break;
                        }
                        const uint32_t th = base + s * stage_bytes + row_off, tl = th + a_bytes;
                        const uint32_t *v = w + 9 * j;
                        // block 0: scale in bytes 0-1, nibbles in bytes 2-17; block 1: scale 18-19, nibbles 20-35
                        const uint32_t d0 = __byte_perm(v[0], v[0], 0x1010), d1 = __byte_perm(v[4], v[4], 0x3232);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint4 h, l;
                            q4_chunk(__byte_perm(v[q], v[q + 1], 0x5432), d0, h, l);
                            sts128(th + ((q ^ sw) << 4), h);
                            sts128(tl + ((q ^ sw) << 4), l);
                            q4_chunk(v[5 + q], d1, h, l);
                            sts128(th + (((4 + q) ^ sw) << 4), h);
                            sts128(tl + (((4 + q) ^ sw) << 4), l);
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
                        mbar_arrive(&full_w[s]);
                        ++g;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, a.tmem_cols);
    }
}

// Activation rows for the f16 kernel: x[b, :] = 2^e[b] * (hi + lo), e chosen so that the
// row's largest magnitude lies in [2^14, 2^15) (f16 hi/lo keep ~22 bits for
// values down to ~2^-28 of it).  One CTA per row and one thread per 32-element
// block of it (K <= 16384: at most 512 threads): the row is read once into
// registers (eight 16-byte loads a thread when vec4), its largest magnitude
// reduced over the CTA, and each block's hi and lo halves leave as four
// 16-byte stores each.  kPermute: K positions in the q4_pos order of each
// 32-element block (the Q4_0 kernel's operand order).
template <bool kPermute>
__global__ void __launch_bounds__(512) split_rows_kernel(const float *x, int k, int x_stride, __half *hi, __half *lo,
                                                         float *scale, int vec4) {
    pdl_launch_dependents();  // the GEMM may start streaming its weights
    pdl_wait_prior();         // x may be the previous kernel's output
    __shared__ uint32_t red[16];
    const int blk = threadIdx.x;
    const bool active = blk < (k >> 5);
    const float *src = x + static_cast<long long>(blockIdx.x) * x_stride + 32 * blk;
    float v[32];
    uint32_t m = 0;
    if (active) {
        if (vec4) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 f = __ldg(reinterpret_cast<const float4 *>(src) + q);
                v[4 * q] = f.x;
                v[4 * q + 1] = f.y;
                v[4 * q + 2] = f.z;
                v[4 * q + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __ldg(src + i);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) m = max(m, __float_as_uint(v[i]) & 0x7fffffffu);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = 0;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) m = max(m, red[i]);
    int e = 0;
    if (m != 0 && m < 0x7f800000u) {
        int ex = static_cast<int>(m >> 23) - 127;
        if (m < 0x00800000u) ex = (31 - __clz(static_cast<int>(m))) - 149;
        e = min(max(ex - 14, -126), 113);
    }
    const float s = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    if (active) {
        uint32_t hw[16] = {}, lw[16] = {};  // f16 bits, two per word, in (permuted) K order
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float u = __fmul_rn(v[i], s);
            const __half h = __float2half_rn(u);
            const float hf = __half2float(h);
            const __half l = (__float_as_uint(hf) & 0x7fffffffu) < 0x7f800000u ? __float2half_rn(__fsub_rn(u, hf))
                                                                               : __ushort_as_half(0);
            const int p = kPermute ? q4_pos(i) : i;
            hw[p >> 1] |= static_cast<uint32_t>(__half_as_ushort(h)) << (16 * (p & 1));
            lw[p >> 1] |= static_cast<uint32_t>(__half_as_ushort(l)) << (16 * (p & 1));
        }
        const long long off = static_cast<long long>(blockIdx.x) * k + 32 * blk;
        uint4 *ho = reinterpret_cast<uint4 *>(hi + off), *lo4 = reinterpret_cast<uint4 *>(lo + off);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            ho[q] = make_uint4(hw[4 * q], hw[4 * q + 1], hw[4 * q + 2], hw[4 * q + 3]);
            lo4[q] = make_uint4(lw[4 * q], lw[4 * q + 1], lw[4 * q + 2], lw[4 * q + 3]);
        }
    }
    if (threadIdx.x == 0) scale[blockIdx.x] = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// ---- host side -------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tc_encode_fn() {
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

// [rows][k] bytes, boxes of box_rows x 128 bytes, 128-byte swizzle.
bool encode_kmajor(CUtensorMap &m, const void *ptr, long long row_bytes, int rows, int box_rows) {
    auto fn = tc_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kStepBytes), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// q4_0 weights [rows][row_bytes] as 4-byte elements, boxes of 128 rows x
// kRawRow bytes, no swizzle (a box past the row end reads zeros).
bool encode_raw_boxes(CUtensorMap &m, const void *ptr, long long row_bytes, int rows) {
    auto fn = tc_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 4), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kRawRow / 4), static_cast<cuuint32_t>(kTileM)};
    cuuint32_t estr[2] = {1, 1};
    return fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool gemm_tc_supported(int wt, int k, int n, int batch) {
    (void)n;
    if (k % 16) return false;
    if (wt == 3 || wt == 1) return batch >= kTcMinBatch;
    // q4: 16-byte multiple row strides (36 * k / 64 bytes)
    return wt == 2 && batch >= kTcMinBatchQ4 && k % 256 == 0;
}

namespace {
size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Tile shape and schedule of one batched matmul.
struct TcShape {
    int nb;             // activation columns per tile (MMA N)
    int ksteps, chunks; // K steps of 128 operand bytes, schedule chunks per tile
    int tiles, ncolt;
    long long iters;
};

TcShape tc_shape(int wt, int k, int n, int batch) {
    TcShape t{};
    const bool i8 = wt == 3;
    const int cap = i8 ? 256 : 128;  // the f16/q4 epilogue keeps NB sums per thread in registers
    t.nb = batch >= cap ? cap : (batch + 15) / 16 * 16;
    if (!i8) t.nb = t.nb <= 16 ? 16 : t.nb <= 32 ? 32 : t.nb <= 64 ? 64 : 128;
    const long long row_bytes = i8 ? k : 2ll * k;  // bytes per row of the MMA operands
    t.ksteps = static_cast<int>((row_bytes + kStepBytes - 1) / kStepBytes);
    t.chunks = (t.ksteps + kChunkSteps - 1) / kChunkSteps;
    t.ncolt = (batch + t.nb - 1) / t.nb;
    t.tiles = ((n + kTileM - 1) / kTileM) * t.ncolt;
    t.iters = static_cast<long long>(t.tiles) * t.chunks;
    return t;
}

// Stream-K pays when one CTA per tile would leave SMs idle: fewer tiles
// than SMs, or a last wave that is less than 95% full.  Measured on B200
// (per-step time, stream-K against one CTA per tile): f16 K8192 N8192 B64
// 57 vs 78 us, int8 K8192 N28672 B32 75 vs 82 us, B256 174 vs 175 us,
// q4_0 K4096 N14336 B16 57 vs 59 us; but q4_0 with wide tiles lost (B128
// 83 vs 70 us, B512 254 vs 249 us: its four dequantiser warps restart their
// pipeline at every segment and the 64 KB partials do not pay back), so
// q4_0 takes it only for tiles of at most 32 columns.
bool tc_stream_k(int wt, const TcShape &t, int sms, bool allowed) {
    if (!allowed || sms <= 0 || t.tiles % sms == 0) return false;
    if (wt == 2 && t.nb > 32) return false;
    const long long waves = (t.tiles + sms - 1) / sms;
    return t.tiles < sms || static_cast<double>(t.tiles) / static_cast<double>(waves * sms) < 0.95;
}

size_t tc_partial_slot_bytes(int wt, const TcShape &t) {
    return static_cast<size_t>(kTileM) * t.nb * 4 * (wt == 3 ? 2 : 1);
}
}  // namespace

// Scratch of one batched matmul: the f16 hi/lo activation split (f16 and
// q4_0), then, when the stream-K schedule is used, the per-tile arrival
// counters (zero) and two partial-accumulator slots per CTA.
size_t gemm_tc_scratch_bytes(int wt, int k, int n, int batch, const DeviceInfo &dev) {
    if (wt != 1 && wt != 2 && wt != 3) return 0;
    size_t bytes = wt == 3 ? 0 : 2 * align256(static_cast<size_t>(batch) * k * 2) + align256(static_cast<size_t>(batch) * 4);
    const TcShape t = tc_shape(wt, k, n, batch);
    if (tc_stream_k(wt, t, dev.sm_count, dev.stream_k))
        bytes += align256(static_cast<size_t>(t.tiles) * 4) + 2 * static_cast<size_t>(dev.sm_count) * tc_partial_slot_bytes(wt, t);
    return bytes;
}

cudaError_t launch_gemm_tc(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    if (!gemm_tc_supported(r.wt, r.k, r.n, r.batch)) return cudaErrorNotSupported;
    const bool i8 = r.wt == 3, q4 = r.wt == 2;
    if (reinterpret_cast<uintptr_t>(r.w) & 15) return cudaErrorNotSupported;
    if (q4 && r.k % 256) return cudaErrorNotSupported;  // 16-byte multiple rows
    if (i8 && ((reinterpret_cast<uintptr_t>(r.q) & 15) || (r.q_comp & 15) || r.q_stride != r.k))
        return cudaErrorNotSupported;
    if (!i8 && (!r.split || r.split_bytes < 2 * align256(static_cast<size_t>(r.batch) * r.k * 2) +
                                               align256(static_cast<size_t>(r.batch) * 4)))
        return cudaErrorNotSupported;
    TcArgs a{};
    a.w = static_cast<const uint8_t *>(r.w);
    a.row_bytes = static_cast<long long>(r.k / 32) * 18;
    a.y = r.y;
    a.row_scale = r.row_scale;
    a.act_max = r.act_max;
    a.err = dev.err;
    a.k = r.k;
    a.n = r.n;
    a.batch = r.batch;
    a.y_stride = r.y_stride;
    const TcShape shape = tc_shape(r.wt, r.k, r.n, r.batch);
    a.nb = shape.nb;
    const long long row_bytes = i8 ? r.k : 2ll * r.k;  // bytes per row of the MMA operands
    a.ksteps = shape.ksteps;
    a.chunks = shape.chunks;
    a.ncolt = shape.ncolt;
    a.iters = shape.iters;
    // one CTA per tile, or (with the scratch for partials) one per SM over equal shares of the work
    const size_t act_bytes = i8 ? 0 : 2 * align256(static_cast<size_t>(r.batch) * r.k * 2) + align256(static_cast<size_t>(r.batch) * 4);
    const bool sk = tc_stream_k(r.wt, shape, dev.sm_count, dev.stream_k) && r.split &&
                    r.split_bytes >= gemm_tc_scratch_bytes(r.wt, r.k, r.n, r.batch, dev);
    // (at least one iteration per CTA: then consecutive CTAs start at strictly
    // increasing iterations, and a tile's segments come from consecutive CTAs)
    a.grid = sk ? static_cast<int>(shape.iters < dev.sm_count ? shape.iters : dev.sm_count) : shape.tiles;
    if (sk) {
        char *sk_base = static_cast<char *>(r.split) + act_bytes;
        a.counters = reinterpret_cast<int *>(sk_base);
        a.partials = sk_base + align256(static_cast<size_t>(shape.tiles) * 4);
    }
    uint32_t cols = 32;
    // i8: two accumulators; f16 and q4: two chunk slots of 2 x nb columns
    while (cols < static_cast<uint32_t>((i8 ? 2 : 4) * a.nb)) cols <<= 1;
    a.tmem_cols = cols;
    const size_t stage = static_cast<size_t>(kTileM) * kStepBytes * (q4 ? 2 : 1) + 2 * static_cast<size_t>(a.nb) * kStepBytes;
    // q4: three raw slots while that leaves three operand stages, else two
    int raw_slots = q4 ? 3 : 0, stages = 0;
    for (;;) {
        const size_t fixed = q4 ? kBarBytesQ4 + static_cast<size_t>(raw_slots) * kRawBox : 256;
        stages = static_cast<int>((static_cast<size_t>(dev.smem_optin) - 1024 - fixed) / stage);
        if (!q4 || stages >= 3 || raw_slots == 2) break;
        --raw_slots;
    }
    if (stages > 6) stages = 6;
    if (stages < 2) return cudaErrorNotSupported;
    a.stages = stages;
    a.raw_slots = raw_slots;
    const size_t smem = 1024 + stages * stage + (q4 ? kBarBytesQ4 + static_cast<size_t>(raw_slots) * kRawBox : 256);
    TcMaps maps;
    const void *b0 = r.q, *b1 = r.q ? r.q + r.q_comp : nullptr;
    if (!i8) {
        // split the activation rows into f16 hi/lo (scratch: hi | lo | scales)
        const size_t part = align256(static_cast<size_t>(r.batch) * r.k * 2);
        char *sbase = static_cast<char *>(r.split);
        __half *hi = reinterpret_cast<__half *>(sbase), *lo = reinterpret_cast<__half *>(sbase + part);
        float *sc = reinterpret_cast<float *>(sbase + 2 * part);
        const int vec4 = (reinterpret_cast<uintptr_t>(r.x) & 15) == 0 && r.x_stride % 4 == 0;
        cudaLaunchConfig_t scfg{};
        scfg.gridDim = dim3(r.batch);
        scfg.blockDim = dim3((r.k / 32 + 31) / 32 * 32);
        scfg.stream = stream;
        cudaLaunchAttribute sattr[1];
        sattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        sattr[0].val.programmaticStreamSerializationAllowed = 1;
        scfg.attrs = sattr;
        scfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&scfg, q4 ? split_rows_kernel<true> : split_rows_kernel<false>, r.x, r.k,
                                           r.x_stride, hi, lo, sc, vec4);
        if (e != cudaSuccess) return e;
        b0 = hi;
        b1 = lo;
        a.col_scale = sc;
    }
    if ((q4 ? !encode_raw_boxes(maps.a, r.w, a.row_bytes, r.n) : !encode_kmajor(maps.a, r.w, row_bytes, r.n, kTileM)) ||
        !encode_kmajor(maps.b0, b0, row_bytes, r.batch, a.nb) || !encode_kmajor(maps.b1, b1, row_bytes, r.batch, a.nb))
        return cudaErrorNotSupported;
    void (*kern)(TcMaps, TcArgs) = gemm_i8_kernel;
    int ki = 0;
    if (!i8) {
        const int which = a.nb == 16 ? 0 : a.nb == 32 ? 1 : a.nb == 64 ? 2 : 3;
        static void (*const f16k[4])(TcMaps, TcArgs) = {gemm_f16_kernel<16>, gemm_f16_kernel<32>, gemm_f16_kernel<64>,
                                                          gemm_f16_kernel<128>};
        static void (*const q4k[4])(TcMaps, TcArgs) = {gemm_q4_kernel<16>, gemm_q4_kernel<32>, gemm_q4_kernel<64>,
                                                         gemm_q4_kernel<128>};
        kern = q4 ? q4k[which] : f16k[which];
        ki = 1 + which + (q4 ? 4 : 0);
    }
    static int configured[9][64] = {{0}};
    int devno = 0;
    cudaGetDevice(&devno);
    if (devno < 0 || devno >= 64 || configured[ki][devno] < static_cast<int>(smem)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (devno >= 0 && devno < 64) configured[ki][devno] = static_cast<int>(smem);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3(q4 ? kThreadsQ4 : kThreadsTc);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, maps, a);
}

}  // namespace k200
