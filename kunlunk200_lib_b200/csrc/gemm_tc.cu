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
//  * Q4_0 weights (the same kernel with a second weight operand): the blocks
//    are first expanded into f16 pairs W' = d*(q-8) = hi + lo (exact: hi =
//    f16(d*(q-8)), lo = fma(d, q-8, -hi), the residual has at most 3
//    significant bits), then three products are accumulated per K step:
//    hi*x_hi + hi*x_lo + lo*x_hi (lo*x_lo is below 2^-21 of the term).
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
    CUtensorMap a1;   // second weight operand (the lo half of split weights)
    CUtensorMap b0;   // activation operand 0 [batch][k]
    CUtensorMap b1;   // activation operand 1 [batch][k]
};

struct TcArgs {
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
};

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

// ---- the kernel --------------------------------------------------------------
__global__ void __launch_bounds__(kThreadsTc, 1) gemm_i8_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned stages: [A 128 x 128 B][B0 nb x 128 B][B1 nb x 128 B]
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t a_bytes = kTileM * kStepBytes, b_bytes = a.nb * kStepBytes;
    const uint32_t stage_bytes = a_bytes + 2 * b_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.stages * stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *accum = empty + a.stages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTileM, n0 = blockIdx.y * a.nb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
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
            for (int ks = 0; ks < a.ksteps; ++ks) {
                const int s = ks % a.stages;
                if (ks >= a.stages && !mbar_wait(&empty[s], ((ks / a.stages) - 1) & 1, a.err, kErrBulkTimeout)) break;
                const uint32_t st = base + s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                tma_2d(st, &maps.a, ks * kStepBytes, m0, &full[s]);
                tma_2d(st + a_bytes, &maps.b0, ks * kStepBytes, n0, &full[s]);
                tma_2d(st + a_bytes + b_bytes, &maps.b1, ks * kStepBytes, n0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = instr_desc(2, 1, 1, kTileM, a.nb);  // s32 <- s8 x s8
            for (int ks = 0; ks < a.ksteps; ++ks) {
                const int s = ks % a.stages;
                if (!mbar_wait(&full[s], (ks / a.stages) & 1, a.err, kErrBulkTimeout)) break;
                tc_fence_after();
                const uint32_t st = base + s * stage_bytes;
                const uint64_t da = sw128_desc(st), db0 = sw128_desc(st + a_bytes), db1 = sw128_desc(st + a_bytes + b_bytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K per 128-byte step: +2 in the address field
                    const uint32_t acc = (ks | kk) != 0;
                    mma_i8(taddr, da + 2 * kk, db0 + 2 * kk, idesc, acc);
                    mma_i8(taddr + a.nb, da + 2 * kk, db1 + 2 * kk, idesc, acc);
                }
                mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
            }
            mma_commit(accum);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warps 2..5 -> TMEM lane quarters 2,3,0,1 ----------------
        const int quarter = warp & 3;
        const int row = m0 + quarter * 32 + lane;  // weight row of this thread
        const bool ok = mbar_wait(accum, 0, a.err, kErrMmaTimeout);
        tc_fence_after();
        if (ok) {
            const uint32_t lane_addr = taddr + (static_cast<uint32_t>(quarter * 32) << 16);
            const float s0 = __fdiv_rn(a.act_max[0], 127.0f), s1 = __fdiv_rn(a.act_max[1], 127.0f);
            const float rs = row < a.n ? a.row_scale[row] : 0.f;
            for (int c0 = 0; c0 < a.nb; c0 += 16) {
                uint32_t p0[16], p1[16];
                tmem_ld16(lane_addr + c0, p0);
                tmem_ld16(lane_addr + a.nb + c0, p1);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int col = n0 + c0 + i;
                    if (row < a.n && col < a.batch) {
                        const float t0 = __fmul_rn(static_cast<float>(static_cast<int>(p0[i])), s0);
                        const float t1 = __fmul_rn(static_cast<float>(static_cast<int>(p1[i])), s1);
                        a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(__fadd_rn(t0, t1), rs);
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

// f16 weights, chunked accumulation; NB activation columns per CTA.
constexpr int kChunkSteps = 4;
template <int NB, bool SPLITW>
__global__ void __launch_bounds__(kThreadsTc, 1) gemm_f16_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - smem_u32(smem_raw));
    // stage: [A 128 x 128 B][A1 (split weights)][B0 NB x 128 B][B1 NB x 128 B]
    constexpr uint32_t a_bytes = kTileM * kStepBytes, b_bytes = NB * kStepBytes;
    constexpr uint32_t a_total = SPLITW ? 2 * a_bytes : a_bytes;
    constexpr uint32_t stage_bytes = a_total + 2 * b_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.stages * stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *tfull = empty + a.stages;  // [2] a tensor-memory slot holds a finished chunk
    uint64_t *tfree = tfull + 2;         // [2] the epilogue has read a slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfree + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTileM, n0 = blockIdx.y * NB;
    const int nchunks = (a.ksteps + kChunkSteps - 1) / kChunkSteps;

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
            for (int ks = 0; ks < a.ksteps; ++ks) {
                const int s = ks % a.stages;
                if (ks >= a.stages && !mbar_wait(&empty[s], ((ks / a.stages) - 1) & 1, a.err, kErrBulkTimeout)) break;
                const uint32_t st = base + s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                tma_2d(st, &maps.a, ks * kStepBytes, m0, &full[s]);
                if constexpr (SPLITW) tma_2d(st + a_bytes, &maps.a1, ks * kStepBytes, m0, &full[s]);
                tma_2d(st + a_total, &maps.b0, ks * kStepBytes, n0, &full[s]);
                tma_2d(st + a_total + b_bytes, &maps.b1, ks * kStepBytes, n0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc(1, 0, 0, kTileM, NB);  // f32 <- f16 x f16
            bool ok = true;
            for (int c = 0; c < nchunks && ok; ++c) {
                const int slot = c & 1;
                if (c >= 2 && !mbar_wait(&tfree[slot], ((c >> 1) - 1) & 1, a.err, kErrMmaTimeout)) break;
                tc_fence_after();
                const uint32_t d = taddr + slot * NB;
                const int ks_end = min(a.ksteps, (c + 1) * kChunkSteps);
                for (int ks = c * kChunkSteps; ks < ks_end; ++ks) {
                    const int s = ks % a.stages;
                    if (!mbar_wait(&full[s], (ks / a.stages) & 1, a.err, kErrBulkTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t st = base + s * stage_bytes;
                    const uint64_t da = sw128_desc(st), da1 = sw128_desc(st + a_bytes);
                    const uint64_t db0 = sw128_desc(st + a_total), db1 = sw128_desc(st + a_total + b_bytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        mma_f16(d, da + 2 * kk, db0 + 2 * kk, idesc, (ks != c * kChunkSteps) || kk != 0);
                        mma_f16(d, da + 2 * kk, db1 + 2 * kk, idesc, 1);
                        if constexpr (SPLITW) mma_f16(d, da1 + 2 * kk, db0 + 2 * kk, idesc, 1);
                    }
                    mma_commit(&empty[s]);
                }
                mma_commit(&tfull[slot]);
            }
        }
        __syncwarp();
    } else {
        const int quarter = warp & 3;
        const int row = m0 + quarter * 32 + lane;
        const uint32_t lane_addr = taddr + (static_cast<uint32_t>(quarter * 32) << 16);
        float sum[NB];
#pragma unroll
        for (int i = 0; i < NB; ++i) sum[i] = 0.f;
        bool ok = true;
        for (int c = 0; c < nchunks; ++c) {
            const int slot = c & 1;
            if (!mbar_wait(&tfull[slot], (c >> 1) & 1, a.err, kErrMmaTimeout)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int c0 = 0; c0 < NB; c0 += 16) {
                uint32_t p[16];
                tmem_ld16(lane_addr + slot * NB + c0, p);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) sum[c0 + i] = __fadd_rn(sum[c0 + i], __uint_as_float(p[i]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfree[slot]);
        }
        if (ok && row < a.n) {
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int col = n0 + i;
                if (col < a.batch) a.y[static_cast<long long>(col) * a.y_stride + row] = __fmul_rn(sum[i], a.col_scale[col]);
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

// Q4_0 rows -> f16 hi/lo halves of W' = d*(q-8), row-major [rows][k]; one
// thread per 32-element block (element j < 16: low nibble of byte j, j >= 16:
// high nibble of byte j-16, as kernels/kunlun-matvec.xpu:51-59 decodes).
__global__ void __launch_bounds__(256) dequant_q4_split_kernel(const uint8_t *q4, long long row_bytes, int k, int rows,
                                                               __half *hi, __half *lo) {
    const int blocks = k >> 5;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(rows) * blocks) return;
    const int r = static_cast<int>(idx / blocks), b = static_cast<int>(idx - static_cast<long long>(r) * blocks);
    const uint8_t *blk = q4 + r * row_bytes + 18ll * b;
    const uint16_t dbits = static_cast<uint16_t>(blk[0] | (blk[1] << 8));
    const __half2 d2 = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
    uint32_t qs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        qs[i] = static_cast<uint32_t>(blk[2 + 4 * i]) | (static_cast<uint32_t>(blk[3 + 4 * i]) << 8) |
                (static_cast<uint32_t>(blk[4 + 4 * i]) << 16) | (static_cast<uint32_t>(blk[5 + 4 * i]) << 24);
    uint32_t h[16], l[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        // elements e, e+1 of the block
        const int b0 = e & 15;                     // byte index
        const int sh = e < 16 ? 0 : 4;             // nibble
        const int v0 = ((qs[b0 >> 2] >> (8 * (b0 & 3) + sh)) & 15) - 8;
        const int v1 = ((qs[(b0 + 1) >> 2] >> (8 * ((b0 + 1) & 3) + sh)) & 15) - 8;
        const __half2 q2 = __halves2half2(__int2half_rn(v0), __int2half_rn(v1));
        const __half2 hv = __hmul2(d2, q2);
        const __half2 lv = __hfma2(d2, q2, __hneg2(hv));
        h[e >> 1] = *reinterpret_cast<const uint32_t *>(&hv);
        l[e >> 1] = *reinterpret_cast<const uint32_t *>(&lv);
    }
    uint4 *ho = reinterpret_cast<uint4 *>(hi + static_cast<long long>(r) * k + 32ll * b);
    uint4 *lo4 = reinterpret_cast<uint4 *>(lo + static_cast<long long>(r) * k + 32ll * b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        ho[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
        lo4[i] = make_uint4(l[4 * i], l[4 * i + 1], l[4 * i + 2], l[4 * i + 3]);
    }
}

// Activation rows for the f16 kernel: x[b, :] = 2^e[b] * (hi + lo), e chosen so that the
// row's largest magnitude lies in [2^14, 2^15) (f16 hi/lo keep ~22 bits for
// values down to ~2^-28 of it).  One CTA per row.
__global__ void __launch_bounds__(256) split_rows_kernel(const float *x, int k, int x_stride, __half *hi, __half *lo,
                                                         float *scale) {
    __shared__ uint32_t red[8];
    const float *src = x + static_cast<long long>(blockIdx.x) * x_stride;
    uint32_t m = 0;
    for (int j = threadIdx.x; j < k; j += blockDim.x) m = max(m, __float_as_uint(src[j]) & 0x7fffffffu);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = 0;
    for (int i = 0; i < (blockDim.x >> 5); ++i) m = max(m, red[i]);
    int e = 0;
    if (m != 0 && m < 0x7f800000u) {
        int ex = static_cast<int>(m >> 23) - 127;
        if (m < 0x00800000u) ex = (31 - __clz(static_cast<int>(m))) - 149;
        e = min(max(ex - 14, -126), 113);
    }
    const float s = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    __half *h = hi + static_cast<long long>(blockIdx.x) * k, *l = lo + static_cast<long long>(blockIdx.x) * k;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const float v = __fmul_rn(src[j], s);
        const __half hv = __float2half_rn(v);
        const float hf = __half2float(hv);
        h[j] = hv;
        l[j] = (__float_as_uint(hf) & 0x7fffffffu) < 0x7f800000u ? __float2half_rn(__fsub_rn(v, hf)) : __ushort_as_half(0);
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

}  // namespace

bool gemm_tc_supported(int wt, int k, int n, int batch) {
    (void)n;
    if (k % 16) return false;
    if (wt == 3 || wt == 1) return batch >= kTcMinBatch;
    return wt == 2 && batch >= kTcMinBatchQ4;
}

namespace {
size_t align256(size_t b) { return (b + 255) & ~size_t(255); }
}  // namespace

size_t gemm_tc_scratch_bytes(int wt, int k, int n, int batch) {
    if (wt != 1 && wt != 2) return 0;
    size_t bytes = 2 * align256(static_cast<size_t>(batch) * k * 2) + align256(static_cast<size_t>(batch) * 4);
    if (wt == 2) bytes += 2 * align256(static_cast<size_t>(n) * k * 2);  // expanded weights, hi and lo
    return bytes;
}

cudaError_t launch_gemm_tc(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    if (!gemm_tc_supported(r.wt, r.k, r.n, r.batch)) return cudaErrorNotSupported;
    const bool i8 = r.wt == 3, q4 = r.wt == 2;
    if (reinterpret_cast<uintptr_t>(r.w) & 15) return cudaErrorNotSupported;
    if (i8 && ((reinterpret_cast<uintptr_t>(r.q) & 15) || (r.q_comp & 15) || r.q_stride != r.k))
        return cudaErrorNotSupported;
    if (!i8 && (!r.split || r.split_bytes < gemm_tc_scratch_bytes(r.wt, r.k, r.n, r.batch))) return cudaErrorNotSupported;
    TcArgs a{};
    a.y = r.y;
    a.row_scale = r.row_scale;
    a.act_max = r.act_max;
    a.err = dev.err;
    a.k = r.k;
    a.n = r.n;
    a.batch = r.batch;
    a.y_stride = r.y_stride;
    const int cap = i8 ? 256 : 128;  // the f16 epilogue keeps NB sums per thread in registers
    a.nb = r.batch >= cap ? cap : (r.batch + 15) / 16 * 16;
    if (!i8) a.nb = a.nb <= 16 ? 16 : a.nb <= 32 ? 32 : a.nb <= 64 ? 64 : 128;
    const long long row_bytes = i8 ? r.k : 2ll * r.k;
    a.ksteps = static_cast<int>((row_bytes + kStepBytes - 1) / kStepBytes);
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(2 * a.nb)) cols <<= 1;  // two accumulators or two slots
    a.tmem_cols = cols;
    const size_t stage = static_cast<size_t>(kTileM) * kStepBytes * (q4 ? 2 : 1) + 2 * static_cast<size_t>(a.nb) * kStepBytes;
    const size_t budget = static_cast<size_t>(dev.smem_optin) - 1024 - 256;
    int stages = static_cast<int>(budget / stage);
    if (stages > 6) stages = 6;
    if (stages < 2) return cudaErrorNotSupported;
    a.stages = stages;
    const size_t smem = 1024 + stages * stage + 256;
    TcMaps maps;
    const void *w0 = r.w, *w1 = r.w, *b0 = r.q, *b1 = r.q ? r.q + r.q_comp : nullptr;
    if (!i8) {
        // split the activation rows into f16 hi/lo (scratch: hi | lo | scales | expanded weights)
        const size_t part = align256(static_cast<size_t>(r.batch) * r.k * 2);
        char *base = static_cast<char *>(r.split);
        __half *hi = reinterpret_cast<__half *>(base), *lo = reinterpret_cast<__half *>(base + part);
        float *sc = reinterpret_cast<float *>(base + 2 * part);
        split_rows_kernel<<<r.batch, 256, 0, stream>>>(r.x, r.k, r.x_stride, hi, lo, sc);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        b0 = hi;
        b1 = lo;
        a.col_scale = sc;
        if (q4) {
            char *wbase = base + 2 * part + align256(static_cast<size_t>(r.batch) * 4);
            const size_t wpart = align256(static_cast<size_t>(r.n) * r.k * 2);
            __half *whi = reinterpret_cast<__half *>(wbase), *wlo = reinterpret_cast<__half *>(wbase + wpart);
            const long long blocks = static_cast<long long>(r.n) * (r.k / 32);
            dequant_q4_split_kernel<<<static_cast<unsigned>((blocks + 255) / 256), 256, 0, stream>>>(
                static_cast<const uint8_t *>(r.w), static_cast<long long>(r.k / 32) * 18, r.k, r.n, whi, wlo);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
            w0 = whi;
            w1 = wlo;
        }
    }
    if (!encode_kmajor(maps.a, w0, row_bytes, r.n, kTileM) || !encode_kmajor(maps.a1, w1, row_bytes, r.n, kTileM) ||
        !encode_kmajor(maps.b0, b0, row_bytes, r.batch, a.nb) || !encode_kmajor(maps.b1, b1, row_bytes, r.batch, a.nb))
        return cudaErrorNotSupported;
    void (*kern)(TcMaps, TcArgs) = gemm_i8_kernel;
    int ki = 0;
    if (!i8) {
        const int which = a.nb == 16 ? 0 : a.nb == 32 ? 1 : a.nb == 64 ? 2 : 3;
        static void (*const f16k[4])(TcMaps, TcArgs) = {gemm_f16_kernel<16, false>, gemm_f16_kernel<32, false>,
                                                          gemm_f16_kernel<64, false>, gemm_f16_kernel<128, false>};
        static void (*const q4k[4])(TcMaps, TcArgs) = {gemm_f16_kernel<16, true>, gemm_f16_kernel<32, true>,
                                                         gemm_f16_kernel<64, true>, gemm_f16_kernel<128, true>};
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
    cfg.gridDim = dim3((r.n + kTileM - 1) / kTileM, (r.batch + a.nb - 1) / a.nb);
    cfg.blockDim = dim3(kThreadsTc);
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
