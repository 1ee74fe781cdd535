// Internal interfaces between the host runtime (runtime.cpp, matmul.cpp) and
// the CUDA kernels of libkunlunk200.  Not installed; not part of the ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace k200 {

struct DeviceInfo {
    int id = -1;
    int sm_count = 0;
    int smem_optin = 0;     // max dynamic shared memory per block (opt-in)
    int *err = nullptr;     // device view of the mapped error word
    bool stream_k = true;   // batched GEMMs may use the persistent stream-K schedule (KUNLUN_STREAM_K=0: never)
};

// Fused all-gather of a row-sharded matmul over peer memory (k200_gather,
// exchange.cuh): the values this rank computes are stored as tagged words
// {f32, epoch} into every rank's tag array of the exchange, and the launch's
// last block raises this rank's epoch of it.  A batch-1 Q4_0 GEMV can read
// its X from another exchange's tags, waiting for each word's epoch.
constexpr int kGatherMaxRanks = 8;
constexpr int kGatherUnsupported = -4;  // K200_GATHER_UNSUPPORTED
struct GatherLaunch {
    int ranks = 0, rank = 0;                          // ranks 0: no gather
    unsigned long long *tags[kGatherMaxRanks] = {};   // every rank's tag array (offset to this shard)
    unsigned *counter = nullptr;                      // this rank's {arrivals, epoch} words
    const unsigned long long *wait_tags = nullptr;    // this rank's tags of the exchange that made X, at X[0]
    const unsigned *wait_counter = nullptr;           // this rank's counter of that exchange
    int wait_tagged = 0;                              // X[0, wait_tagged) is tagged; the rest is read plain
};

// One legacy matmul launch: Y[c, r] = W[r, :] . X[c, :].
struct GemvRequest {
    int wt;                        // 0 f32, 1 f16, 2 q4_0, 3 rowwise int8
    const void *w;                 // weight rows
    const float *x;                // f32 activations (wt 0..2)
    const int8_t *q;               // int8 activation components (wt 3): [2][q_batch][q_stride]
    const float *act_max;          // {max0, max1} (wt 3)
    const float *row_scale;        // per-row scales (wt 3)
    float *y;
    int k, n, batch;
    int x_stride, q_stride, y_stride;
    long long q_comp;              // elements between component 0 and 1 of q (wt 3)
    bool prefetch_weights;         // weights are not written by the preceding kernel: stream
                                   // them before that kernel completes (programmatic launch)
    void *fixup = nullptr;         // Kernel-owned scratch of the tensor-core Q4_0 GEMV (counters
    size_t fixup_bytes = 0;        // zeroed at allocation, partial sums), see q4_mma_scratch_bytes
    bool tensor_cores = true;      // batched shapes may take the tcgen05 GEMM (KUNLUN_TC=0: never)
    void *split = nullptr;         // Kernel-owned scratch for the GEMM's split activations
    size_t split_bytes = 0;        // (gemm_tc_scratch_bytes)
    const GatherLaunch *gather = nullptr;  // batch-1 Q4_0 only (launch_q4_mma_gemv)
};

// Streaming GEMV launcher (handles any batch by column groups).
cudaError_t launch_gemv(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream);

// Tensor-core Q4_0 GEMV for one activation column (gemv_q4_mma.cu).  Scratch
// it needs for this shape (0: shape not handled; the caller then leaves
// GemvRequest::fixup empty and launch_gemv takes the streaming kernel): the
// partial sums of row tiles shared between CTAs, which must be zero before
// the first launch; every launch leaves them zero.
size_t q4_mma_scratch_bytes(int k, int n, int batch, const DeviceInfo &dev);

// tcgen05 GEMM for batches of columns (gemm_tc.cu): rowwise-int8 with the
// activation components already quantised (GemvRequest::q), and f16 and
// q4_0 weights with f32 activations.  GemvRequest::split holds its scratch
// (gemm_tc_scratch_bytes): the f16 activation split (f16, q4_0; required)
// and, for shapes whose tiles would leave SMs idle, the stream-K counters
// (which must be zero before the first launch; every launch leaves them
// zero) and partial slots.  Without that part (e.g. the allocation-free
// int8 entry point) every CTA computes whole tiles.
constexpr int kTcMinBatch = 4;
constexpr int kTcMinBatchQ4 = 4;
bool gemm_tc_supported(int wt, int k, int n, int batch);  // (q4_0 also needs k % 64 == 0)
size_t gemm_tc_scratch_bytes(int wt, int k, int n, int batch, const DeviceInfo &dev);
cudaError_t launch_gemm_tc(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream);
cudaError_t launch_q4_mma_gemv(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream);
// Waits for the first `count` tagged words of this rank's tag array of an
// exchange to carry this rank's current epoch and stores their values into
// y (kErrPeerTimeout after the budget).
cudaError_t launch_gather_wait(const unsigned long long *tags, float *y, long long count, const unsigned *counter,
                               const DeviceInfo &dev, cudaStream_t stream);
// Row gather (gather.cu): [batch][n] slice -> tagged words in columns of
// every rank's [batch][rows] tag array (xg.tags[r] point at the slice's
// first column) and plain values in this rank's own [batch][rows] output y
// (at the slice's first column), then the exchange's next epoch.
cudaError_t launch_gather_rows(const GatherLaunch &xg, float *y, const float *shard, int n, int batch, int rows,
                               const DeviceInfo &dev, cudaStream_t stream);
// Row gathers (get_rows.cu); an index outside [0, n) writes no output and
// sets *status to 1 (else 0).
cudaError_t launch_get_rows_f32(float *out, const float *in, const int32_t *idx, int *status, int k, int n, int rows,
                                cudaStream_t stream);
cudaError_t launch_common_get_rows(float *out, const uint8_t *w, size_t scale_offset, int kp, int np,
                                   const int32_t *idx, int *status, int k, int n, int rows, cudaStream_t stream);
// Q6_K typed GEMV (q6_k.cu), n % 32 == 0, k % 256 == 0: raw GGML blocks
// [n][k/256][210 B] -> packed int8 values and f32 group scales (a non-finite
// block scale sets *status); chunk-256 A8 of m activation rows ([m][k] int8,
// [m][k/256] scales); then the int8 x int8 GEMV of those m rows.
cudaError_t launch_q6_unpack(const uint8_t *raw, int k, int n, int8_t *w, float *wscale, int *status,
                             cudaStream_t stream);
cudaError_t launch_q6_quant(const void *x, int dtype, int k, int m, int8_t *q, float *scales, cudaStream_t stream);
cudaError_t launch_q6_gemv(float *y, const int8_t *w, const float *wscale, const int8_t *q, const float *ascale, int k,
                           int n, int m, const DeviceInfo &dev, cudaStream_t stream);
// kunlun::swiglu (swiglu.cu): y = SiLU(gate) * up, strides in bytes, f16 != 0: F16 rows.
cudaError_t launch_swiglu(void *y, const void *gate, const void *up, int width, int rows, int gs, int us, int ys,
                          int f16, const DeviceInfo &dev, cudaStream_t stream);
// FP32 SIMT GEMM for f32 weights at batch >= kF32GemmMinBatch and K % 64 == 0
// (gemm_f32.cu): reads W once per tile of up to 64 columns instead of once
// per column pair.  Measured on B200 at K = N = 8192 it streams the weights
// at ~1.5 TB/s, so below 9 columns the column-pair streaming kernel (one
// ~6 TB/s pass per two columns) is faster.
constexpr int kF32GemmMinBatch = 9;
bool gemm_f32_supported(const GemvRequest &r);
cudaError_t launch_gemm_f32(const GemvRequest &r, const DeviceInfo &dev, cudaStream_t stream);
bool gemv_fast_path_ok(int wt, const void *w, const void *x, const void *y, int k, long long row_bytes);

// Per-tensor two-component A8 quantiser of the rowwise-int8 path
// (src/k200.cpp:209-229).  q receives [2][count] int8, maxima {max0, max1}.
// `scratch` holds count floats (residual) plus 64 bytes of reduction words.
cudaError_t launch_a8_tensor(const float *x, size_t count, int8_t *q, float *maxima, void *scratch,
                             const DeviceInfo &dev, cudaStream_t stream);
size_t a8_tensor_scratch_bytes(size_t count);

// upload_i8_rows on the device (src/k200.cpp:107-116): f32 rows -> int8 rows
// and per-row scales.
cudaError_t launch_i8_rows(const float *w, int k, int rows, int8_t *q, float *scales, const DeviceInfo &dev,
                           cudaStream_t stream);

// kunlun::elementwise (op 0 add, 1 multiply, 2 silu, 3 rms_norm, 4 scale).
cudaError_t launch_elementwise(float *y, const float *a, const float *b, int n, int width, int bn, int op, float p,
                               const DeviceInfo &dev, cudaStream_t stream);

// GGML Q4_0 block quantiser (f32 [n][k] -> 18-byte blocks).
cudaError_t launch_q4_0_quantize(const float *w, int n, int k, uint8_t *q4, cudaStream_t stream);

// Native and common Q4 layouts (q4_layouts.cu).  dtype: 0 f32, 1 f16 input.
// Two-component A8 of one activation vector, params {s0, s1, max0, max1}.
// kq == 0: q0, q1 [k] int8; kq > 0 (the common layout's activation view):
// element j at (j/32)*64 + j%32 of each [2*kq] component, the rest zero.
cudaError_t launch_a8x2(const void *x, int k, int dtype, int kq, int8_t *q0, int8_t *q1, float *params,
                        cudaStream_t stream);
// Row A8 of m activation rows into [m][kq] int8 (zero past k), row scales
// every scale_stride floats.
cudaError_t launch_row_a8(const void *x, int m, int k, int dtype, int kq, int8_t *q, float *row_scale,
                          int scale_stride, cudaStream_t stream);
cudaError_t launch_native_gemv_a8x2(const uint8_t *w, const uint16_t *scales, const int8_t *q0, const int8_t *q1,
                                    const float *params, int k, int n, float *y, const DeviceInfo &dev,
                                    cudaStream_t stream);
cudaError_t launch_native_fallback(const uint8_t *w, const uint16_t *scales, const void *x, int dtype, int k, int n,
                                   int batch, float *y, const DeviceInfo &dev, cudaStream_t stream);
cudaError_t launch_common_gemv_a8x2(const uint8_t *w, size_t scale_offset, int kp, int np, const int8_t *q0,
                                    const int8_t *q1, const float *params, int k, int n, float *y,
                                    const DeviceInfo &dev, cudaStream_t stream);
// row_scale: one scale every 16 floats (the activation view's layout).
cudaError_t launch_common_gemv_pair(const uint8_t *w0, const uint8_t *w1, size_t scale_offset, int kp, int np,
                                    const int8_t *q0, const int8_t *q1, const float *params, int k, int n, float *y0,
                                    float *y1, const DeviceInfo &dev, cudaStream_t stream);
cudaError_t launch_common_gemm_a8(const uint8_t *w, size_t scale_offset, int kp, int np, const int8_t *q,
                                  const float *row_scale, int k, int n, int m, float *y, cudaStream_t stream);

// Copy by a kernel (copy.cu); either side may be pinned host memory.
cudaError_t launch_copy_kernel(void *dst, const void *src, size_t bytes, const DeviceInfo &dev, cudaStream_t stream);

// Runtime hooks (runtime.cpp).
cudaStream_t library_stream(int device);
const DeviceInfo &device_info(int device);
void count_matmul(int device);

// Static scratch of the allocation-free rowwise-int8 matmul (static_scratch.cu):
// room for batch*k <= kNoAllocMaxElements activations, two int8 components
// each, plus a 256-byte parameter block.
constexpr size_t kNoAllocMaxElements = size_t(1) << 21;
constexpr size_t kNoAllocParamsOffset = 2 * kNoAllocMaxElements;
constexpr size_t kNoAllocScratchBytes = kNoAllocParamsOffset + 256;
// Device address of that scratch on the CURRENT device (cudaGetSymbolAddress).
cudaError_t noalloc_scratch_address(void **ptr);
// Statuses of matmul_i8_noalloc besides CUDA errors (K200_NOALLOC_* in k200_c.h).
constexpr int kNoAllocTooLarge = -2;
constexpr int kNoAllocNotReady = -3;
int matmul_i8_noalloc(int device, void *y, const void *w, const void *x, int k, int n, int batch,
                      const float *scales, const float *maximum);

}  // namespace k200
