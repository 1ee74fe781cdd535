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

struct Statistics {
    size_t matmuls[2];            // devices 0 and 1 (ABI of the reference struct)
    size_t peer_copies, peer_bytes;
};
Statistics statistics();
const char *version();

}  // namespace kunlun
