// Batched F32 matmul, Y[b, r] = sum_j W[r, j] * X[b, j], in FP32 on the SIMT
// pipes (sm_100a): the reference computes F32 weights with FP32 products and
// sums (kernels/kunlun-matvec.xpu:37-77), and no tensor-core format holds an
// f32 weight exactly, so this kernel keeps the reference's arithmetic class
// and reads every weight once per tile of activation columns instead of once
// per pair of columns (the streaming GEMV's cost at batch > 2).
//
// One CTA (256 threads) computes 64 weight rows x BN columns (BN = 16, 32 or
// 64 by the batch).  K advances in steps of 64 through a ring of 4-8
// stages filled with 16-byte cp.async copies (L2 256-byte prefetch; several
// steps of weights in flight per SM): the weight tile (64 rows x 256 bytes)
// and the activation tile (BN columns x 256 bytes) are stored row-major with
// the 16-byte chunk index XOR-ed with (row mod 8), so that the 16-byte reads
// below fall in different banks.  Thread (tm, tn) of a 16 x 16 grid owns rows tm + 16 i
// (i < 4) and columns tn + 16 j (j < BN/16); per group of four k it reads its
// rows and columns as 16-byte vectors and issues 16 * BN/16 FMAs.
//
// Each output is a blocked sum in increasing k order: every 8 products are
// chained with FP32 FMAs into a fresh partial (the reference's FP32
// arithmetic), four such partials are added in FP32, and those sums of 32
// products are added in double precision (one conversion and one add per 32
// FMAs).  The error is then about a third of that of 32-term FP32 chains
// (which reach 1.1e-5 at K = 8192 with U[-1, 1] data, above the 1e-5 F32
// bar), far below a K-term running FP32 sum, for one extra FP32 add per 8
// FMAs.
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

constexpr int kRows = 64;      // weight rows per CTA
constexpr int kStep = 64;      // K per pipeline step (K must be a multiple)
constexpr int kRowBytes = kStep * 4;     // bytes of one row of a step's tile
constexpr int kChunks = kRowBytes / 16;  // 16-byte copies per row
constexpr int kThreadsF32 = 256;
// ring stages: deeper for narrow column tiles, whose steps compute little
// and must keep more weight bytes in flight per SM
template <int BN>
__host__ __device__ constexpr int stages_for() { return BN <= 16 ? 8 : BN <= 32 ? 6 : 4; }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool ok) {
    // src-size 0 zero-fills the 16 bytes (rows or columns past the matrix)
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// byte offset of 16-byte chunk q of row r in a row-major tile of kRowBytes rows
__device__ __forceinline__ uint32_t swz(int r, int q) { return static_cast<uint32_t>(r * kRowBytes + ((q ^ (r & 7)) << 4)); }

template <int BN>
__global__ void __launch_bounds__(kThreadsF32, 1) gemm_f32_kernel(const float *__restrict__ w, const float *__restrict__ x,
                                                             float *__restrict__ y, int k, int n, int batch,
                                                             int x_stride, int y_stride) {
    constexpr int TN = BN / 16;  // columns per thread
    constexpr int kStagesF32 = stages_for<BN>();
    constexpr int kWBytes = kRows * kRowBytes, kXBytes = BN * kRowBytes;
    constexpr int kStageBytesF32 = kWBytes + kXBytes;
    extern __shared__ __align__(128) uint8_t smf[];
    const uint32_t base = smem_u32(smf);
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * kRows, c0 = blockIdx.y * BN;

    // copies of one stage: weight chunks (64 rows x 8) and activation chunks
    // (BN columns x 8), 16 bytes each, spread over the 256 threads
    auto issue = [&](int st, int k0) {
        const uint32_t sw = base + st * kStageBytesF32, sx = sw + kWBytes;
#pragma unroll
        for (int i = 0; i < kRows * kChunks / kThreadsF32; ++i) {
            const int v = tid + i * kThreadsF32, r = v / kChunks, q = v % kChunks;
            const bool ok = r0 + r < n;
            cp_async16(sw + swz(r, q), w + static_cast<size_t>(ok ? r0 + r : 0) * k + k0 + 4 * q, ok);
        }
#pragma unroll
        for (int i = 0; i < (BN * kChunks + kThreadsF32 - 1) / kThreadsF32; ++i) {
            const int v = tid + i * kThreadsF32;
            if (v < BN * kChunks) {
                const int cc = v / kChunks, q = v % kChunks;
                const bool ok = c0 + cc < batch;
                cp_async16(sx + swz(cc, q), x + static_cast<size_t>(ok ? c0 + cc : 0) * x_stride + k0 + 4 * q, ok);
            }
        }
    };

    const int tm = tid & 15, tn = tid >> 4;
    double acc[4][TN];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0;

    pdl_launch_dependents();
    pdl_wait_prior();  // X (and Y) may belong to the previous kernel
    const int steps = k / kStep;
#pragma unroll
    for (int st = 0; st < kStagesF32 - 1; ++st) {
        if (st < steps) issue(st, st * kStep);
        cp_async_commit();
    }
    for (int s = 0; s < steps; ++s) {
        cp_async_wait<kStagesF32 - 2>();  // this thread's copies of step s have landed ...
        __syncthreads();                   // ... and every thread's; the stage of step s-1 is free
        if (s + kStagesF32 - 1 < steps) issue((s + kStagesF32 - 1) % kStagesF32, (s + kStagesF32 - 1) * kStep);
        cp_async_commit();
        const uint32_t sw = base + (s % kStagesF32) * kStageBytesF32, sx = sw + kWBytes;
        float part[4][TN];  // the current 8 products
        float mid[4][TN];   // the current 32 products, four partials of 8
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) part[i][j] = mid[i][j] = 0.f;
#pragma unroll
        for (int q = 0; q < kChunks; ++q) {
            float4 a[4], b[TN];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t ad = sw + swz(tm + 16 * i, q);
                asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(a[i].x), "=f"(a[i].y), "=f"(a[i].z), "=f"(a[i].w)
                             : "r"(ad));
            }
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const uint32_t ad = sx + swz(tn + 16 * j, q);
                asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(b[j].x), "=f"(b[j].y), "=f"(b[j].z), "=f"(b[j].w)
                             : "r"(ad));
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) {
                    part[i][j] = fmaf(a[i].x, b[j].x, part[i][j]);
                    part[i][j] = fmaf(a[i].y, b[j].y, part[i][j]);
                    part[i][j] = fmaf(a[i].z, b[j].z, part[i][j]);
                    part[i][j] = fmaf(a[i].w, b[j].w, part[i][j]);
                }
            if (q % 2 == 1) {  // every 8 products
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) {
                        mid[i][j] = __fadd_rn(mid[i][j], part[i][j]);
                        part[i][j] = 0.f;
                    }
            }
            if (q % 8 == 7) {  // every 32 products
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) {
                        acc[i][j] += static_cast<double>(mid[i][j]);
                        mid[i][j] = 0.f;
                    }
            }
        }
    }
    cp_async_wait<0>();  // no copy may still target shared memory at exit
#pragma unroll
    for (int j = 0; j < TN; ++j) {
        const int col = c0 + tn + 16 * j;
        if (col >= batch) continue;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = r0 + tm + 16 * i;
            if (row < n) y[static_cast<size_t>(col) * y_stride + row] = static_cast<float>(acc[i][j]);
        }
    }
}

template <int BN>
cudaError_t launch_bn(const GemvRequest &r, cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(stages_for<BN>()) * (kRows + BN) * kRowBytes;
    static bool configured[64] = {false};
    int devno = 0;
    cudaGetDevice(&devno);
    if (devno < 0 || devno >= 64 || !configured[devno]) {
        const cudaError_t e = cudaFuncSetAttribute(gemm_f32_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (devno >= 0 && devno < 64) configured[devno] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((r.n + kRows - 1) / kRows, (r.batch + BN - 1) / BN);
    cfg.blockDim = dim3(kThreadsF32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_f32_kernel<BN>, static_cast<const float *>(r.w), r.x, r.y, r.k, r.n,
                              r.batch, r.x_stride, r.y_stride);
}

}  // namespace

bool gemm_f32_supported(const GemvRequest &r) {
    if (r.wt != 0 || r.batch < kF32GemmMinBatch || r.k % kStep) return false;
    const uintptr_t wp = reinterpret_cast<uintptr_t>(r.w), xp = reinterpret_cast<uintptr_t>(r.x);
    return (wp & 15) == 0 && (xp & 15) == 0 && r.x_stride % 4 == 0;
}

cudaError_t launch_gemm_f32(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream) {
    (void)dev;
    if (!gemm_f32_supported(r)) return cudaErrorNotSupported;
    if (r.batch <= 16) return launch_bn<16>(r, stream);
    if (r.batch <= 32) return launch_bn<32>(r, stream);
    return launch_bn<64>(r, stream);
}

}  // namespace k200
