// kunlun/k200.h -- B200 (sm_100a) implementation of the KunlunK200 library's
// matmul hot path, Y[batch,n] = X[batch,k] . W^T[n,k].
//
// This header declares the subset of the reference API (UnagiDojyou/
// kunlunK200_lib v0.7.12, include/kunlun/k200.h) that libkunlunk200.so.0
// implements.  Names, signatures, enum values and class layouts are kept
// identical so that code compiled against the reference header links against
// this library unchanged (same Itanium-mangled symbols):
//
//   runtime            k200.h:10-23    runtime_mutex check diagnostic_tensor
//                                      require device_count select wait copy
//                                      peer allocate release allocated_bytes
//   Buffer             k200.h:25-37    layout {int device_; size_t bytes_; void *ptr_;}
//   Kernel             k200.h:62-88    pimpl (one Impl pointer)
//   rowwise int8       k200.h:90-96    aligned packed_i8_size/_scales/_maxima upload_i8_rows
//   matmul             k200.h:98-105
//   elementwise        k200.h:106-107
//   native Q4 layout   k200.h:127-131,203-224  native_q4_* NativeQ4Workspace
//   common Q4 ABI v1   k200.h:226-335  CommonQ4Weight CommonQ4Workspace
//                                      common_q4_matmul (not the activation
//                                      lease / shared / pair calls)
//   statistics/version k200.h:345-350
//
// Device model: a "PD" index is a CUDA device ordinal (0..7 on an 8-GPU box).
// All work is issued on one library stream per device; wait() synchronises
// that stream.  Every entry point serialises on runtime_mutex(), like the
// reference.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

namespace kunlun {

// Process-global lock.  Every API takes it; callers composing raw
// select/copy/wait sequences hold it across the sequence.
std::recursive_mutex &runtime_mutex();
// Abort with a diagnostic when status != 0 (fail-fast, like the reference).
void check(int status);
// Borrowed tensor name printed by check()/require() diagnostics.
void diagnostic_tensor(const char *name, const int64_t *dimensions = nullptr);
// Abort with a diagnostic when the condition is false.
void require(bool condition);
// Number of usable devices (CUDA ordinals); returns a CUDA status.
int device_count(int *count);
// Make `device` current for this thread (0 <= device < device_count).
void select(int device);
// Complete all work submitted to the current device; returns 0 or a nonzero
// status (a CUDA error, or a kernel-posted error such as non-finite input).
int wait();
enum CopyKind { host_to_device, device_to_host, device_to_device };
// Copy on the current device's library stream; completes before returning.
int copy(void *dst, const void *src, size_t bytes, CopyKind kind);
// Device-to-device copy between GPUs over NVLink; completes before returning.
void peer(int dst_device, void *dst, int src_device, const void *src, size_t bytes);
// Device allocation (at least 256 bytes, 256-byte aligned); null on failure.
void *allocate(int device, size_t bytes);
void release(int device, void *ptr, size_t bytes);
size_t allocated_bytes(int device);

class Buffer {
public:
    Buffer(int device, size_t bytes);
    ~Buffer();
    Buffer(const Buffer &) = delete;
    Buffer &operator=(const Buffer &) = delete;
    void *data() const { return ptr_; }
    size_t size() const { return bytes_; }
private:
    int device_;
    size_t bytes_;
    void *ptr_;
};

enum class WeightType { f32 = 0, f16 = 1, q4_0 = 2, rowwise_i8 = 3, q6_k = 4 };
enum class ElementwiseOp { add = 0, multiply = 1, silu = 2, rms_norm = 3, scale = 4 };
enum class InputType { f32, f16 };

// Per-call state: device binding and lazily grown scratch (quantised
// activations of the rowwise int8 path).  Bound to the first device used.
class CommonQ4Weight;
struct SwiGLULayout;

class Kernel {
public:
    Kernel();
    ~Kernel();
    Kernel(const Kernel &) = delete;
    Kernel &operator=(const Kernel &) = delete;
    struct Impl;
private:
    Impl *impl_;
    friend void matmul(Kernel &, int, void *, const void *, const void *, int, int, int, WeightType, const float *,
                       const float *, int);
    friend void elementwise(Kernel &, int, void *, const void *, const void *, int, int, int, ElementwiseOp,
                            float);
    friend bool get_rows_f32(Kernel &, int, void *, size_t, const void *, size_t, const int32_t *, size_t, int, int,
                             int);
    friend bool common_q4_get_rows(Kernel &, int, void *, size_t, const CommonQ4Weight &, const int32_t *, size_t,
                                   int);
    friend bool swiglu(Kernel &, int, void *, size_t, const void *, size_t, const void *, size_t,
                       const SwiGLULayout &);
};

// Rowwise int8 weights: aligned(k*rows) int8 values, then aligned(rows*4)
// f32 row scales, then 256 bytes holding maxima[6] = {127, ...}.
size_t aligned(size_t bytes);
size_t packed_i8_size(int k, int rows);
float *packed_i8_scales(void *weights, int k, int rows);
float *packed_i8_maxima(void *weights, int k, int rows);
// Quantise host F32 rows [first_row, first_row+count) into a caller-owned
// packed_i8_size(k, rows) device allocation.  Completes before returning.
void upload_i8_rows(int device, void *weights, int k, int rows, int first_row, int count, const float *input);

// W: [n,k], X: [batch,k] f32, Y: [batch,n] f32.  All pointers are device
// memory.  Q4_0: 18-byte blocks (little-endian F16 scale + 16 paired 4-bit
// values).  rowwise_i8 requires scales[n] and maxima[6] in device memory.
// matmul submits work; select(device) + check(wait()) completes it.
// K must be divisible by 32, K <= 16384.  `tile` (1 or 16) is accepted for
// compatibility; it does not change results.
void matmul(Kernel &, int device, void *y, const void *w, const void *x, int k, int n, int batch, WeightType type,
            const float *scales = nullptr, const float *maxima = nullptr, int tile = 16);
// Y = op(A, B) over `count` F32 values (B broadcast with period b_count);
// rms_norm normalises rows of `width`.  Completes before returning.
void elementwise(Kernel &, int device, void *y, const void *a, const void *b, int count, int width, int b_count,
                 ElementwiseOp op, float parameter = 0);

// ---- native Q4 layout (reference k200.h:127-131, 203-224) ------------------
// The original Q4_0 values and FP16 block scales, N padded to 32:
// [N32 tile][K32 block][16 byte pairs][32 rows] of signed 4-bit pairs, then the
// scales.  Packing runs on the host.
bool native_q4_layout_supported(int k, int n);
size_t native_q4_size(int k, int n);
bool pack_native_q4(void *destination, size_t bytes, const void *q4, int k, int n);
void upload_native_q4(int device, void *weights, const void *q4, int k, int n);
// Empty string: the W4A8x2 path applies (batch 1, N % 128 == 0, ...).
const char *native_q4_reason(int k, int n, int batch, InputType type);
struct NativeQ4Statistics {
    size_t accelerated, fallback;
    size_t hbm_workspace_bytes, l3_workspace_bytes;
};
class NativeQ4Workspace {
public:
    NativeQ4Workspace();
    ~NativeQ4Workspace();
    NativeQ4Workspace(const NativeQ4Workspace &) = delete;
    NativeQ4Workspace &operator=(const NativeQ4Workspace &) = delete;
    NativeQ4Statistics statistics() const;
    struct Impl;
private:
    Impl *impl_;
    friend bool native_q4_matmul(NativeQ4Workspace &, int, void *, const void *, const void *, int, int, int,
                                 InputType);
};
// Completes before returning.  True: W4A8x2 (two-component per-tensor int8
// activations); false: the exact FP32 fallback.  Y [batch,n] f32, X [batch,k].
bool native_q4_matmul(NativeQ4Workspace &, int device, void *y, const void *weights, const void *input, int k, int n,
                      int batch = 1, InputType type = InputType::f32);

// ---- common Q4 ABI v1 (reference k200.h:226-335) --------------------------
struct CommonQ4Info {
    uint32_t abi_version, quant_type, layout, scale_order;
    int k, n, kp, np, device;
    size_t scale_offset, payload_bytes;
};
bool common_q4_supported(int k, int n);
size_t common_q4_size(int k, int n);
struct CommonQ4ActivationStatistics {
    size_t prepare_calls, quantized_chunks, quant_kernel_launches;
    size_t prepared_matmuls, prepared_chunks, invalidations, rejected_calls;
    size_t hbm_activation_bytes;
    uint64_t quantization_ns, preparation_ns;
};
struct CommonQ4ActivationChunk {
    const void *values;
    const void *scales;
    int first, rows, padded_rows, kp, components;
    size_t values_bytes, scales_bytes;
};
class CommonQ4ActivationLease;
class CommonQ4Workspace;
struct CommonQ4WeightStatistics {
    size_t uploads, upload_bytes;
    double pack_ms, upload_ms;
};
class CommonQ4Weight {
public:
    // Borrowed storage must be 256-byte aligned; null storage allocates a Buffer.
    CommonQ4Weight(int device, int k, int n, void *storage = nullptr, size_t bytes = 0);
    ~CommonQ4Weight();
    CommonQ4Weight(const CommonQ4Weight &) = delete;
    CommonQ4Weight &operator=(const CommonQ4Weight &) = delete;
    CommonQ4Info info() const;
    CommonQ4WeightStatistics statistics() const;
    void *data() const;
    // Packs N rows of K/32 Q4_0 blocks on the host and uploads them.
    void upload(const void *q4, size_t bytes);
    struct Impl;
private:
    Impl *impl_;
    friend void common_q4_matmul(class CommonQ4Workspace &, int, void *, const CommonQ4Weight &, const void *, int,
                                 InputType);
    friend bool common_q4_matmul_pair(CommonQ4Workspace &, int, void *, void *, const CommonQ4Weight &,
                                      const CommonQ4Weight &, const CommonQ4ActivationLease &, uint64_t);
    friend bool common_q4_matmul_shared(class CommonQ4Workspace &, int, void *, const CommonQ4Weight &,
                                        const CommonQ4ActivationLease &, uint64_t);
};
struct CommonQ4Statistics {
    // GEMV, Combined, Wide, Rows64, Rows128, Combo2, Combo4, exact CL.
    size_t paths[8], calls, chunks;
    size_t hbm_workspace_bytes, l3_workspace_bytes, slice_bytes;
};
struct CommonQ4MacStatistics {
    size_t baseline_sd_calls, stream_sd_calls, shape_fallbacks, resident_l1d_bytes;
};
struct CommonQ4Quantization {
    const void *values;
    const void *scales;
    int rows, kp, components;
};
struct CommonQ4PairStatistics {
    size_t calls, declined, l3_partial_bytes;
};
enum class CommonQ4PairStatus {
    NotAttempted, Success, Disabled, InvalidInput, Configuration, WeightAbi, Lease, Alias, Workspace
};
class CommonQ4Workspace {
public:
    CommonQ4Workspace();
    ~CommonQ4Workspace();
    CommonQ4Workspace(const CommonQ4Workspace &) = delete;
    CommonQ4Workspace &operator=(const CommonQ4Workspace &) = delete;
    CommonQ4Statistics statistics() const;
    CommonQ4ActivationStatistics activation_statistics() const;
    CommonQ4MacStatistics mac_statistics() const;
    // The last call's quantised activations (device buffers, valid until the next call).
    CommonQ4Quantization quantization() const;
    struct Impl;
private:
    Impl *impl_;
    friend CommonQ4PairStatistics common_q4_pair_statistics(const CommonQ4Workspace &);
    friend CommonQ4PairStatus common_q4_pair_last_status(const CommonQ4Workspace &);
    friend bool common_q4_matmul_pair(CommonQ4Workspace &, int, void *, void *, const CommonQ4Weight &,
                                      const CommonQ4Weight &, const CommonQ4ActivationLease &, uint64_t);
    friend void common_q4_matmul(CommonQ4Workspace &, int, void *, const CommonQ4Weight &, const void *, int,
                                 InputType);
    friend bool common_q4_prepare(CommonQ4Workspace &, int, const void *, int, int, InputType, uint64_t,
                                  CommonQ4ActivationLease &);
    friend bool common_q4_matmul_shared(class CommonQ4Workspace &, int, void *, const CommonQ4Weight &,
                                        const CommonQ4ActivationLease &, uint64_t);
};
// X [m,k], Y [m,n].  Completes before returning.  M = 1: two-component A8;
// M > 1: one int8 scale per activation row (Row A8).
void common_q4_matmul(CommonQ4Workspace &, int device, void *y, const CommonQ4Weight &, const void *input, int m,
                      InputType type = InputType::f32);

// A snapshot of quantised activations in a workspace, valid until that
// workspace quantises again (another prepare, a plain common_q4_matmul, a
// reset or the workspace's destruction).  The owner passes a nonzero
// generation it changes after writing the input.
class CommonQ4ActivationLease {
public:
    CommonQ4ActivationLease();
    ~CommonQ4ActivationLease();
    CommonQ4ActivationLease(const CommonQ4ActivationLease &) = delete;
    CommonQ4ActivationLease &operator=(const CommonQ4ActivationLease &) = delete;
    void reset();
    bool matches(int device, int k, int rows, InputType, uint64_t generation) const;
    size_t chunks() const;
    CommonQ4ActivationChunk chunk(size_t index) const;
    struct Impl;
private:
    Impl *impl_;
    friend bool common_q4_matmul_pair(CommonQ4Workspace &, int, void *, void *, const CommonQ4Weight &,
                                      const CommonQ4Weight &, const CommonQ4ActivationLease &, uint64_t);
    friend bool common_q4_prepare(CommonQ4Workspace &, int, const void *, int, int, InputType, uint64_t,
                                  CommonQ4ActivationLease &);
    friend bool common_q4_matmul_shared(CommonQ4Workspace &, int, void *, const CommonQ4Weight &,
                                        const CommonQ4ActivationLease &, uint64_t);
};
// Quantises X [rows, k] once into the workspace and points the lease at it
// (chunks of up to 128 rows).  False: unsupported descriptor, nothing done.
bool common_q4_prepare(CommonQ4Workspace &, int device, const void *input, int k, int rows, InputType,
                       uint64_t generation, CommonQ4ActivationLease &);
// common_q4_matmul on the lease's activations; false: stale or mismatched
// lease or a pointer contract violation, no output written.
bool common_q4_matmul_shared(CommonQ4Workspace &, int device, void *y, const CommonQ4Weight &,
                             const CommonQ4ActivationLease &, uint64_t generation);
// y0 = X W0^T and y1 = X W1^T for one prepared F32 activation row and two
// weights of the same shape (the 7B/1B gate and up projections), in one pass
// over the activations.  False (with the reason in common_q4_pair_last_status)
// when declined; outputs untouched.
bool common_q4_matmul_pair(CommonQ4Workspace &, int device, void *y0, void *y1, const CommonQ4Weight &w0,
                           const CommonQ4Weight &w1, const CommonQ4ActivationLease &, uint64_t generation);
CommonQ4PairStatistics common_q4_pair_statistics(const CommonQ4Workspace &);
CommonQ4PairStatus common_q4_pair_last_status(const CommonQ4Workspace &);

// ---- Q6_K typed GEMV (reference k200.h:135-165) ----------------------------
struct Q6KInfo {
    uint32_t abi_version;
    int device, k, n;
    size_t scale_offset, payload_bytes;
};
struct Q6KStatistics {
    size_t calls, uploads, upload_bytes, workspace_bytes;
    double pack_ms, upload_ms;
};
bool q6_k_supported(int k, int n);
size_t q6_k_size(int k, int n);
class Q6KWeight {
public:
    // Borrowed storage must be 256-byte aligned; null storage allocates a Buffer.
    Q6KWeight(int device, int k, int n, void *storage = nullptr, size_t bytes = 0);
    ~Q6KWeight();
    Q6KWeight(const Q6KWeight &) = delete;
    Q6KWeight &operator=(const Q6KWeight &) = delete;
    // Packs N rows of K/256 GGML Q6_K blocks on the host and uploads them.
    void upload(const void *q6, size_t bytes);
    Q6KInfo info() const;
    Q6KStatistics statistics() const;
    void *data() const;
    struct Impl;
private:
    Impl *impl_;
    friend void q6_k_matmul(class Q6KWorkspace &, int, void *, const Q6KWeight &, const void *, int, InputType);
};
class Q6KWorkspace {
public:
    Q6KWorkspace();
    ~Q6KWorkspace();
    Q6KWorkspace(const Q6KWorkspace &) = delete;
    Q6KWorkspace &operator=(const Q6KWorkspace &) = delete;
    Q6KStatistics statistics() const;
    size_t legacy_calls() const;
    struct Impl;
private:
    Impl *impl_;
    friend void q6_k_matmul(Q6KWorkspace &, int, void *, const Q6KWeight &, const void *, int, InputType);
};
// X [m,k] (m = 1..512), Y [m,n]; activations quantised per 256-value chunk.
// Completes before returning.
void q6_k_matmul(Q6KWorkspace &, int device, void *y, const Q6KWeight &, const void *x, int m = 1,
                 InputType type = InputType::f32);

// Row gathers: output[r] = input row indices[r] (F32 rows; K % 16 == 0,
// 16 <= K <= 1048576) or the decoded common-Q4 weight column indices[r]
// (K % 64 == 0), rows = 1..512, output 64-byte aligned.  Complete before
// returning; false (and no output written) on a contract violation or an
// index outside [0, n).
bool get_rows_f32(Kernel &, int device, void *output, size_t output_bytes, const void *input, size_t input_bytes,
                  const int32_t *indices, size_t index_bytes, int k, int n, int rows);
bool common_q4_get_rows(Kernel &, int device, void *output, size_t output_bytes, const CommonQ4Weight &,
                        const int32_t *indices, size_t index_bytes, int rows);

// Fused gate/up activation: y = SiLU(gate) * up with F32 intermediates and
// one final rounding, rows of `width` contiguous F32 or F16 values at byte
// strides.  An empty reason means supported.  Completes before returning;
// false means an unsupported layout or pointer contract (nothing submitted).
// An exact alias of y with gate or up (same start and row stride) is allowed.
struct SwiGLULayout {
    int width, rows;
    int gate_stride, up_stride, output_stride;  // bytes between rows
    InputType type;
};
const char *swiglu_reason(const SwiGLULayout &);
bool swiglu(Kernel &, int device, void *y, size_t y_bytes, const void *gate, size_t gate_bytes, const void *up,
            size_t up_bytes, const SwiGLULayout &);

struct Statistics {
    size_t matmuls[2];            // devices 0 and 1 (ABI of the reference struct)
    size_t peer_copies, peer_bytes;
};
Statistics statistics();
const char *version();

}  // namespace kunlun
