// Host runtime of libkunlunk200 on CUDA: the kunlun:: API of the reference's
// src/k200.cpp (UnagiDojyou/kunlunK200_lib v0.7.12) re-implemented over the
// CUDA runtime.  Semantics kept from the reference:
//   * one process-global recursive mutex taken by every entry point
//     (src/k200.cpp:25,48);
//   * fail-fast: check()/require() print the device, tensor and shape context
//     and abort (src/k200.cpp:32-36,53-62); allocate() returns null on failure
//     (src/k200.cpp:76-83);
//   * matmul() validates the reference contract (src/k200.cpp:268-279) and
//     only submits work; select(device) + check(wait()) completes it;
//   * copy()/peer()/upload_i8_rows()/elementwise() complete before returning.
// Device model: a PD index is a CUDA ordinal.  Each device gets one library
// stream (a blocking stream, so it is ordered after work on the legacy default
// stream, e.g. cudaMemcpy or a framework's default stream) and one error word
// in mapped host memory that kernels post to instead of trapping.
#include <kunlun/k200.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "k200_internal.h"

namespace kunlun {

namespace {

constexpr int kMaxDevices = 64;

std::recursive_mutex mutex;
std::atomic<size_t> peer_copies{0}, peer_bytes{0};

struct DeviceState {
    bool ready = false;
    cudaStream_t own = nullptr;      // the library stream created at first use
    cudaStream_t stream = nullptr;   // the stream work is issued on (own, or a caller's)
    int *err_host = nullptr;
    k200::DeviceInfo info;
    std::atomic<size_t> allocated{0};
    std::atomic<size_t> matmuls{0};
    bool static_weights = false;     // see k200_set_static_weights
    bool q4_mma = true;              // tensor-core Q4_0 GEMV (KUNLUN_Q4_MMA=0 selects the FP32 kernel)
    bool tensor_cores = true;        // tcgen05 GEMM for batched shapes (KUNLUN_TC=0: streaming kernels only)
    void *noalloc_scratch = nullptr; // static scratch address (k200_matmul_i8_noalloc)
};
DeviceState devices[kMaxDevices];

thread_local int current_device = -1;
thread_local int diagnostic_device = -1;
thread_local const char *diagnostic_name = nullptr;
thread_local int64_t diagnostic_shape[4] = {};

void diagnostic_print() {
    std::fprintf(stderr, "Kunlun context: pd=%d tensor=%s shape=[%lld,%lld,%lld,%lld]\n", diagnostic_device,
                 diagnostic_name ? diagnostic_name : "<outside graph>", (long long)diagnostic_shape[0],
                 (long long)diagnostic_shape[1], (long long)diagnostic_shape[2], (long long)diagnostic_shape[3]);
    std::fflush(stderr);
}

int cuda_device_count() {
    static int count = -1;
    if (count < 0) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        count = std::min(n, kMaxDevices);
    }
    return count;
}

void fail_cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        diagnostic_print();
        std::fprintf(stderr, "Kunlun CUDA failure: %s: %s (%d)\n", what, cudaGetErrorString(e), (int)e);
        std::fflush(stderr);
        std::abort();
    }
}

DeviceState &state(int id) {
    DeviceState &d = devices[id];
    if (!d.ready) {
        fail_cuda(cudaSetDevice(id), "cudaSetDevice");
        fail_cuda(cudaStreamCreate(&d.own), "cudaStreamCreate");
        d.stream = d.own;
        fail_cuda(cudaHostAlloc(reinterpret_cast<void **>(&d.err_host), 64, cudaHostAllocMapped),
                  "cudaHostAlloc(error word)");
        *d.err_host = 0;
        int *dev_err = nullptr;
        fail_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&dev_err), d.err_host, 0),
                  "cudaHostGetDevicePointer");
        d.info.id = id;
        d.info.err = dev_err;
        const char *sw = std::getenv("KUNLUN_STATIC_WEIGHTS");
        d.static_weights = sw && std::strcmp(sw, "1") == 0;
        const char *qm = std::getenv("KUNLUN_Q4_MMA");
        d.q4_mma = !(qm && std::strcmp(qm, "0") == 0);
        const char *tc = std::getenv("KUNLUN_TC");
        d.tensor_cores = !(tc && std::strcmp(tc, "0") == 0);
        const char *sk = std::getenv("KUNLUN_STREAM_K");
        d.info.stream_k = !(sk && std::strcmp(sk, "0") == 0);
        fail_cuda(cudaDeviceGetAttribute(&d.info.sm_count, cudaDevAttrMultiProcessorCount, id), "sm count");
        fail_cuda(cudaDeviceGetAttribute(&d.info.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, id),
                  "smem opt-in");
        // The static scratch of k200_matmul_i8_noalloc lives in a module that
        // CUDA loads lazily, on first use.  Looking its address up here makes
        // the module (and its fixed array) load during device set-up, so the
        // allocation-free entry point itself never causes a device
        // allocation.
        fail_cuda(k200::noalloc_scratch_address(&d.noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)");
        d.ready = true;
    }
    return d;
}

DeviceState &current() {
    require(current_device >= 0);
    return state(current_device);
}

}  // namespace

// ---------------------------------------------------------------------------
// runtime
// ---------------------------------------------------------------------------
std::recursive_mutex &runtime_mutex() { return mutex; }

void diagnostic_tensor(const char *name, const int64_t *dimensions) {
    diagnostic_name = name;
    for (int i = 0; i < 4; ++i) diagnostic_shape[i] = dimensions ? dimensions[i] : 0;
}

void check(int rc) {
    if (rc) {
        diagnostic_print();
        std::fprintf(stderr, "Kunlun runtime error %d\n", rc);
        std::fflush(stderr);
        std::abort();
    }
}

void require(bool ok) {
    if (!ok) {
        diagnostic_print();
        std::fprintf(stderr, "Kunlun invalid argument or unavailable resource\n");
        std::fflush(stderr);
        std::abort();
    }
}

int device_count(int *n) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    if (!n) return (int)cudaErrorInvalidValue;
    *n = cuda_device_count();
    return 0;
}

void select(int id) {
    diagnostic_device = id;
    require(id >= 0 && id < cuda_device_count());
    std::lock_guard<std::recursive_mutex> lock(mutex);
    state(id);
    fail_cuda(cudaSetDevice(id), "cudaSetDevice");
    current_device = id;
}

int wait() {
    if (current_device < 0) return (int)cudaErrorInvalidDevice;
    DeviceState &d = state(current_device);
    cudaError_t e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess) return (int)e;
    int posted = __atomic_exchange_n(d.err_host, 0, __ATOMIC_SEQ_CST);
    return posted;
}

int copy(void *dst, const void *src, size_t bytes, CopyKind kind) {
    require(kind == host_to_device || kind == device_to_host || kind == device_to_device);
    std::lock_guard<std::recursive_mutex> lock(mutex);
    DeviceState &d = current();
    if (bytes == 0) return 0;
    cudaMemcpyKind k = kind == host_to_device   ? cudaMemcpyHostToDevice
                       : kind == device_to_host ? cudaMemcpyDeviceToHost
                                                : cudaMemcpyDeviceToDevice;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, k, d.stream);
    if (e != cudaSuccess) return (int)e;
    return (int)cudaStreamSynchronize(d.stream);
}

void *allocate(int id, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    select(id);
    void *ptr = nullptr;
    size_t size = std::max<size_t>(bytes, 256);
    if (cudaMalloc(&ptr, size) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    devices[id].allocated += size;
    return ptr;
}

void release(int id, void *ptr, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    if (!ptr) return;
    select(id);
    check((int)cudaFree(ptr));
    devices[id].allocated -= std::max<size_t>(bytes, 256);
}

size_t allocated_bytes(int id) {
    require(id >= 0 && id < kMaxDevices);
    return devices[id].allocated.load();
}

void peer(int dst, void *dp, int src, const void *sp, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    select(src);
    check(wait());
    select(dst);
    if (dst != src) {
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, dst, src) == cudaSuccess && can) {
            cudaError_t e = cudaDeviceEnablePeerAccess(src, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else fail_cuda(e, "cudaDeviceEnablePeerAccess");
        }
    }
    fail_cuda(cudaMemcpyPeerAsync(dp, dst, sp, src, bytes, state(dst).stream), "cudaMemcpyPeerAsync");
    check(wait());
    ++peer_copies;
    peer_bytes += bytes;
}

Buffer::Buffer(int id, size_t bytes) : device_(id), bytes_(bytes), ptr_(allocate(id, bytes)) { require(ptr_); }
Buffer::~Buffer() { release(device_, ptr_, bytes_); }

size_t aligned(size_t n) {
    require(n <= SIZE_MAX - 255);
    return (n + 255) & ~size_t(255);
}
size_t packed_i8_size(int k, int n) {
    require(k > 0 && n >= 0);
    return aligned((size_t)k * n) + aligned((size_t)n * 4) + 256;
}
float *packed_i8_scales(void *p, int k, int n) { return (float *)((char *)p + aligned((size_t)k * n)); }
float *packed_i8_maxima(void *p, int k, int n) {
    return (float *)((char *)packed_i8_scales(p, k, n) + aligned((size_t)n * 4));
}

// ---------------------------------------------------------------------------
// Kernel handle
// ---------------------------------------------------------------------------
struct Kernel::Impl {
    int id = -1;
    void *quant = nullptr;   // rowwise int8: [2][batch*k] quantised activations
    size_t quant_size = 0;
    void *params = nullptr;  // {max0, max1} + reduction words (256 bytes)
    void *alias = nullptr;   // elementwise broadcast operand copy when y aliases b
    size_t alias_size = 0;
    void *fixup = nullptr;   // tensor-core Q4_0 GEMV: tile counters (zeroed) + partial sums
    size_t fixup_size = 0;
    void *split = nullptr;   // tensor-core GEMM: activations split into f16 hi/lo
    size_t split_size = 0;
    void *rows_status = nullptr;  // row gathers: index verdict written by the kernel (256 bytes)
};

Kernel::Kernel() : impl_(new Impl{}) {}
Kernel::~Kernel() {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    Impl &s = *impl_;
    if (s.id >= 0) {
        select(s.id);
        check(wait());
        release(s.id, s.quant, s.quant_size);
        release(s.id, s.params, 256);
        release(s.id, s.alias, s.alias_size);
        release(s.id, s.fixup, s.fixup_size);
        release(s.id, s.split, s.split_size);
        release(s.id, s.rows_status, 256);
    }
    delete impl_;
}

namespace {
void grow(Kernel::Impl &s, void *&ptr, size_t &size, size_t need) {
    if (size >= need) return;
    if (ptr) {
        check(wait());  // in-flight work may still read the old buffer
        release(s.id, ptr, size);
    }
    ptr = allocate(s.id, need);
    require(ptr);
    size = need;
}
}  // namespace

namespace {
// Scratch of the tcgen05 GEMM (activation split, stream-K counters and
// partials) in the Kernel's split buffer; zeroed when it grows, since the
// counters must start at zero (every launch leaves them zero).
void tc_scratch(Kernel::Impl &s, DeviceState &d, k200::GemvRequest &r, int type, int k, int n, int batch) {
    if (!d.tensor_cores || !k200::gemm_tc_supported(type, k, n, batch)) return;
    const size_t need = k200::gemm_tc_scratch_bytes(type, k, n, batch, d.info);
    if (!need) return;
    if (s.split_size < need) {
        grow(s, s.split, s.split_size, need);
        fail_cuda(cudaMemsetAsync(s.split, 0, s.split_size, d.stream), "cudaMemsetAsync(split)");
    }
    r.split = s.split;
    r.split_bytes = s.split_size;
}
}  // namespace

// ---------------------------------------------------------------------------
// matmul (src/k200.cpp:187-279)
// ---------------------------------------------------------------------------
void matmul(Kernel &kernel, int id, void *y, const void *w, const void *x, int k, int n, int batch, WeightType type,
            const float *scales, const float *maximum, int tile) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(type == WeightType::f32 || type == WeightType::f16 || type == WeightType::q4_0 ||
            type == WeightType::rowwise_i8);
    require(k > 0 && k <= 16384 && k % 32 == 0 && n > 0 && batch > 0 && n <= INT_MAX / batch &&
            k <= INT_MAX / batch);
    require((size_t)n * batch <= INT_MAX / 4 && (size_t)k * batch <= INT_MAX / 4);
    size_t row_bytes = type == WeightType::f32   ? (size_t)k * 4
                       : type == WeightType::f16 ? (size_t)k * 2
                       : type == WeightType::q4_0 ? (size_t)k / 32 * 18
                                                  : (size_t)k;
    require(y && w && x && (size_t)n <= INT_MAX / row_bytes && (tile == 1 || tile == 16));
    require(kernel.impl_->id == -1 || kernel.impl_->id == id);
    require(type != WeightType::rowwise_i8 || (scales && maximum));
    select(id);
    Kernel::Impl &s = *kernel.impl_;
    s.id = id;
    DeviceState &d = state(id);

    k200::GemvRequest r{};
    r.wt = (int)type;
    r.w = w;
    r.y = static_cast<float *>(y);
    r.k = k;
    r.n = n;
    r.batch = batch;
    r.x_stride = k;
    r.y_stride = n;
    r.prefetch_weights = d.static_weights;
    r.tensor_cores = d.tensor_cores;
    if (type == WeightType::rowwise_i8) {
        const size_t count = (size_t)k * batch;
        grow(s, s.quant, s.quant_size, aligned(2 * count));
        if (!s.params) {
            size_t dummy = 0;
            grow(s, s.params, dummy, 256);
        }
        float *maxima = static_cast<float *>(s.params);
        void *words = static_cast<char *>(s.params) + 64;
        check((int)k200::launch_a8_tensor(static_cast<const float *>(x), count, static_cast<int8_t *>(s.quant),
                                          maxima, words, d.info, d.stream));
        r.q = static_cast<const int8_t *>(s.quant);
        r.q_stride = k;
        r.q_comp = (long long)count;
        r.act_max = maxima;
        r.row_scale = scales;
        tc_scratch(s, d, r, (int)type, k, n, batch);
    } else {
        r.x = static_cast<const float *>(x);
        const size_t need = type == WeightType::q4_0 && d.q4_mma ? k200::q4_mma_scratch_bytes(k, n, batch, d.info) : 0;
        if (need) {
            if (s.fixup_size < need) {
                grow(s, s.fixup, s.fixup_size, need);
                // arrival counters start at zero; every launch leaves them zero
                fail_cuda(cudaMemsetAsync(s.fixup, 0, need, d.stream), "cudaMemsetAsync(fixup)");
            }
            r.fixup = s.fixup;
            r.fixup_bytes = s.fixup_size;
        }
        tc_scratch(s, d, r, (int)type, k, n, batch);
    }
    check((int)k200::launch_gemv(r, d.info, d.stream));
    ++d.matmuls;
}

// ---------------------------------------------------------------------------
// upload_i8_rows (src/k200.cpp:102-123)
// ---------------------------------------------------------------------------
void upload_i8_rows(int id, void *weights, int k, int n, int first, int count, const float *input) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(weights && input && k > 0 && n > 0 && first >= 0 && count >= 0 && first <= n && count <= n - first);
    select(id);
    DeviceState &d = state(id);
    if (count > 0) {
        const size_t bytes = (size_t)count * k * 4;
        void *staging = nullptr;
        fail_cuda(cudaMalloc(&staging, bytes), "cudaMalloc(upload staging)");
        fail_cuda(cudaMemcpyAsync(staging, input, bytes, cudaMemcpyHostToDevice, d.stream), "upload copy");
        check((int)k200::launch_i8_rows(static_cast<const float *>(staging), k, count,
                                        static_cast<int8_t *>(weights) + (size_t)first * k,
                                        packed_i8_scales(weights, k, n) + first, d.info, d.stream));
        int rc = wait();
        cudaFree(staging);
        require(rc == 0);  // non-finite input aborts, as in the reference
    }
    const float maximum[6] = {127, 127, 127, 127, 127, 127};
    check(copy(packed_i8_maxima(weights, k, n), maximum, sizeof(maximum), host_to_device));
}

// ---------------------------------------------------------------------------
// elementwise (src/k200.cpp:280-323)
// ---------------------------------------------------------------------------
void elementwise(Kernel &kernel, int id, void *y, const void *a, const void *b, int n, int width, int bn,
                 ElementwiseOp operation, float parameter) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    int op = (int)operation;
    require(y && a && b && n > 0 && n <= INT_MAX / 4 && width > 0 && width <= 16384 && n % width == 0);
    require(op >= 0 && op <= 4 && (bn == n || bn == width));
    if (op == 3) require(std::isfinite(parameter) && parameter > 0);
    require(kernel.impl_->id == -1 || kernel.impl_->id == id);
    Kernel::Impl &s = *kernel.impl_;
    s.id = id;
    select(id);
    DeviceState &d = state(id);
    if (y == b && bn != n && (op == 0 || op == 1)) {
        // the broadcast operand would be overwritten while still being read
        grow(s, s.alias, s.alias_size, (size_t)bn * 4);
        fail_cuda(cudaMemcpyAsync(s.alias, b, (size_t)bn * 4, cudaMemcpyDeviceToDevice, d.stream), "alias copy");
        b = s.alias;
    }
    check((int)k200::launch_elementwise(static_cast<float *>(y), static_cast<const float *>(a),
                                        static_cast<const float *>(b), n, width, bn, op, parameter, d.info,
                                        d.stream));
    check(wait());
}

// ---------------------------------------------------------------------------
// row gathers (src/get-rows-f32.inc, src/get-rows.inc)
// ---------------------------------------------------------------------------
namespace {
bool spans_overlap(const void *a, size_t an, const void *b, size_t bn) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return x < y + bn && y < x + an;
}
bool fits(const void *p, size_t bytes) { return (uintptr_t)p <= UINTPTR_MAX - bytes; }

// Binds the Kernel to `id` and returns its status word (allocated on first use).
int *rows_status(Kernel::Impl &s, int id) {
    require(s.id < 0 || s.id == id);
    s.id = id;
    select(id);
    if (!s.rows_status) {
        s.rows_status = allocate(id, 256);
        require(s.rows_status != nullptr);
    }
    return static_cast<int *>(s.rows_status);
}

// Completes the gather and reads the kernel's verdict (0: every index valid).
bool rows_verdict(const int *status) {
    int verdict = 1;
    check(copy(&verdict, status, sizeof(verdict), device_to_host));
    return verdict == 0;
}
}  // namespace

bool get_rows_f32(Kernel &kernel, int id, void *output, size_t output_bytes, const void *input, size_t input_bytes,
                  const int32_t *indices, size_t index_bytes, int k, int n, int rows) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    if (id < 0 || id >= cuda_device_count() || k < 16 || k > 1048576 || k % 16 || n < 1 || rows < 1 || rows > 512)
        return false;
    const size_t row_bytes = (size_t)k * 4;
    if ((size_t)n > SIZE_MAX / row_bytes) return false;
    const size_t xbytes = (size_t)n * row_bytes, ybytes = (size_t)rows * row_bytes, ibytes = (size_t)rows * 4;
    if (!output || !input || !indices || (uintptr_t)output % 64 || (uintptr_t)input % 64 || (uintptr_t)indices % 4 ||
        output_bytes < ybytes || input_bytes < xbytes || index_bytes < ibytes)
        return false;
    if (!fits(output, ybytes) || !fits(input, xbytes) || !fits(indices, ibytes)) return false;
    if (spans_overlap(output, ybytes, input, xbytes) || spans_overlap(output, ybytes, indices, ibytes) ||
        spans_overlap(input, xbytes, indices, ibytes))
        return false;
    int *status = rows_status(*kernel.impl_, id);
    DeviceState &d = state(id);
    check((int)k200::launch_get_rows_f32(static_cast<float *>(output), static_cast<const float *>(input), indices,
                                         status, k, n, rows, d.stream));
    return rows_verdict(status);
}

bool common_q4_get_rows(Kernel &kernel, int id, void *output, size_t output_bytes, const CommonQ4Weight &weight,
                        const int32_t *indices, size_t index_bytes, int rows) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    const CommonQ4Info a = weight.info();
    if (a.abi_version != 1 || a.quant_type != 2 || a.layout != 1 || a.scale_order != 1 ||
        weight.statistics().uploads == 0 || a.device != id || id < 0 || id >= cuda_device_count() || a.k % 64 ||
        rows < 1 || rows > 512)
        return false;
    const size_t ybytes = (size_t)rows * a.k * 4, ibytes = (size_t)rows * 4;
    if (!output || !indices || (uintptr_t)output % 64 || (uintptr_t)indices % 4 || output_bytes < ybytes ||
        index_bytes < ibytes)
        return false;
    require(fits(output, ybytes) && fits(indices, ibytes) && fits(weight.data(), a.payload_bytes));
    if (spans_overlap(output, ybytes, indices, ibytes) || spans_overlap(output, ybytes, weight.data(), a.payload_bytes) ||
        spans_overlap(indices, ibytes, weight.data(), a.payload_bytes))
        return false;
    int *status = rows_status(*kernel.impl_, id);
    DeviceState &d = state(id);
    check((int)k200::launch_common_get_rows(static_cast<float *>(output), static_cast<const uint8_t *>(weight.data()),
                                            a.scale_offset, a.kp, a.np, indices, status, a.k, a.n, rows, d.stream));
    return rows_verdict(status);
}

// ---------------------------------------------------------------------------
// swiglu (src/k200.cpp:324-368)
// ---------------------------------------------------------------------------
const char *swiglu_reason(const SwiGLULayout &p) {
    if (p.type != InputType::f32 && p.type != InputType::f16) return "type";
    const int bytes = p.type == InputType::f32 ? 4 : 2;
    if (p.width <= 0 || p.width > 65536 || p.rows <= 0 || p.rows > INT_MAX / p.width / bytes) return "shape";
    for (int stride : {p.gate_stride, p.up_stride, p.output_stride}) {
        if (stride < p.width * bytes || stride % bytes) return "stride";
        if ((size_t)(p.rows - 1) * stride + (size_t)p.width * bytes > INT_MAX) return "byte extent";
    }
    return "";
}

bool swiglu(Kernel &kernel, int id, void *y, size_t y_bytes, const void *gate, size_t gate_bytes, const void *up,
            size_t up_bytes, const SwiGLULayout &p) {
    std::lock_guard<std::recursive_mutex> lock(mutex);
    if (*swiglu_reason(p) || id < 0 || id >= cuda_device_count() || !y || !gate || !up) return false;
    const int bytes = p.type == InputType::f32 ? 4 : 2;
    const uintptr_t yp = (uintptr_t)y, gp = (uintptr_t)gate, upp = (uintptr_t)up;
    const size_t ys = (size_t)(p.rows - 1) * p.output_stride + (size_t)p.width * bytes;
    const size_t gs = (size_t)(p.rows - 1) * p.gate_stride + (size_t)p.width * bytes;
    const size_t us = (size_t)(p.rows - 1) * p.up_stride + (size_t)p.width * bytes;
    if (ys > y_bytes || gs > gate_bytes || us > up_bytes || yp % bytes || gp % bytes || upp % bytes) return false;
    if (yp + ys < yp || gp + gs < gp || upp + us < upp) return false;
    // an exact alias (same start, same row stride) is element-wise safe
    const bool ga = yp == gp && p.output_stride == p.gate_stride;
    const bool ua = yp == upp && p.output_stride == p.up_stride;
    // gate and up packed in one row: overlapping spans, disjoint elements
    auto row_disjoint = [&](uintptr_t input, int stride) {
        const size_t delta = yp > input ? yp - input : input - yp;
        return (ga || ua) && stride == p.output_stride && delta >= (size_t)p.width * bytes &&
               delta <= (size_t)stride - (size_t)p.width * bytes;
    };
    if ((!ga && yp < gp + gs && gp < yp + ys && !row_disjoint(gp, p.gate_stride)) ||
        (!ua && yp < upp + us && upp < yp + ys && !row_disjoint(upp, p.up_stride)))
        return false;
    Kernel::Impl &s = *kernel.impl_;
    if (s.id != -1 && s.id != id) return false;
    s.id = id;
    select(id);
    DeviceState &d = state(id);
    check((int)k200::launch_swiglu(y, gate, up, p.width, p.rows, p.gate_stride, p.up_stride, p.output_stride,
                                   bytes == 2, d.info, d.stream));
    check(wait());
    return true;
}

Statistics statistics() {
    return {{devices[0].matmuls.load(), devices[1].matmuls.load()}, peer_copies.load(), peer_bytes.load()};
}

const char *version() { return "0.7.12"; }

}  // namespace kunlun

// ---------------------------------------------------------------------------
// hooks used by the C ABI (capi.cpp)
// ---------------------------------------------------------------------------
namespace k200 {
cudaStream_t library_stream(int device) {
    kunlun::require(device >= 0 && device < kunlun::cuda_device_count());
    std::lock_guard<std::recursive_mutex> lock(kunlun::mutex);
    return kunlun::state(device).stream;
}
void set_static_weights(int device, bool on) {
    kunlun::require(device >= 0 && device < kunlun::cuda_device_count());
    std::lock_guard<std::recursive_mutex> lock(kunlun::mutex);
    kunlun::state(device).static_weights = on;
}
void set_stream(int device, cudaStream_t s) {
    kunlun::require(device >= 0 && device < kunlun::cuda_device_count());
    std::lock_guard<std::recursive_mutex> lock(kunlun::mutex);
    kunlun::DeviceState &d = kunlun::state(device);
    d.stream = s ? s : d.own;
}
const DeviceInfo &device_info(int device) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::mutex);
    return kunlun::state(device).info;
}
int current_device() { return kunlun::current_device; }
size_t matmul_count(int device) {
    kunlun::require(device >= 0 && device < kunlun::kMaxDevices);
    return kunlun::devices[device].matmuls.load();
}
void count_matmul(int device) {
    kunlun::require(device >= 0 && device < kunlun::kMaxDevices);
    ++kunlun::devices[device].matmuls;
}
size_t peer_copy_count() { return kunlun::peer_copies.load(); }
size_t peer_byte_count() { return kunlun::peer_bytes.load(); }

size_t q4_gather_scratch(int id, int k, int n) {
    using namespace kunlun;
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(id >= 0 && id < cuda_device_count());
    if (k <= 0 || k > 16384 || k % 32 != 0 || n <= 0) return 0;
    return q4_mma_scratch_bytes(k, n, 1, state(id).info);
}

// Batch-1 Q4_0 GEMV of this rank's rows with the fused all-gather
// (k200_matmul_q4_gather).  Only the tensor-core GEMV stores rows to peers,
// so a shape it does not take is declined, never run another way.
int matmul_q4_gather(int id, const GatherLaunch &g, float *y, const void *w, const void *x, int k, int n,
                     void *scratch, size_t scratch_bytes) {
    using namespace kunlun;
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(id >= 0 && id < cuda_device_count());
    require(k > 0 && k <= 16384 && k % 32 == 0 && n > 0 && w && x && y && scratch);
    require(g.ranks >= 1 && g.ranks <= kGatherMaxRanks && g.rank >= 0 && g.rank < g.ranks && g.counter);
    require(!g.wait_tags || (g.wait_counter && g.wait_tagged >= 0));
    select(id);
    DeviceState &d = state(id);
    const size_t need = q4_mma_scratch_bytes(k, n, 1, d.info);
    if (!need || !d.q4_mma) return kGatherUnsupported;
    require(scratch_bytes >= need);
    GemvRequest r{};
    r.wt = (int)WeightType::q4_0;
    r.w = w;
    r.x = static_cast<const float *>(x);
    r.y = y;
    r.k = k;
    r.n = n;
    r.batch = 1;
    r.x_stride = k;
    r.y_stride = n;
    r.prefetch_weights = d.static_weights;
    r.fixup = scratch;
    r.fixup_bytes = scratch_bytes;
    r.gather = &g;
    const cudaError_t e = launch_q4_mma_gemv(r, d.info, d.stream);
    if (e == cudaErrorNotSupported) return kGatherUnsupported;
    if (e != cudaSuccess) return (int)e;
    ++d.matmuls;
    return 0;
}

int gather_rows(int id, const GatherLaunch &g, float *y, const float *shard, int n, int batch, int rows) {
    using namespace kunlun;
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(id >= 0 && id < cuda_device_count() && y && shard && n > 0 && batch > 0 && rows >= n);
    require(g.ranks >= 1 && g.ranks <= kGatherMaxRanks && g.rank >= 0 && g.rank < g.ranks && g.counter);
    require((size_t)batch * (size_t)rows <= (size_t)INT_MAX);
    select(id);
    DeviceState &d = state(id);
    return (int)launch_gather_rows(g, y, shard, n, batch, rows, d.info, d.stream);
}

int gather_wait(int id, const unsigned long long *tags, float *y, long long count, const unsigned *counter) {
    using namespace kunlun;
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(id >= 0 && id < cuda_device_count() && tags && y && counter && count >= 1);
    select(id);
    DeviceState &d = state(id);
    return (int)launch_gather_wait(tags, y, count, counter, d.info, d.stream);
}

// Rowwise-int8 matmul whose activation scratch is the module's static array
// instead of the Kernel's grown buffer.  Same contract, kernels and results as
// kunlun::matmul(..., rowwise_i8, ...), including the KUNLUN_TC switch.
// Nothing here allocates: the size check comes before any CUDA call, and the
// device must already be set up, since its first select creates its stream
// and error word and loads the module that holds the scratch (whose address
// it records).
int matmul_i8_noalloc(int id, void *y, const void *w, const void *x, int k, int n, int batch, const float *scales,
                      const float *maximum) {
    using namespace kunlun;
    if (k > 0 && batch > 0 && (size_t)k * (size_t)batch > kNoAllocMaxElements) {
        std::fprintf(stderr,
                     "k200_matmul_i8_noalloc: batch*k = %zu exceeds the static scratch limit of %zu elements "
                     "(use k200_matmul)\n",
                     (size_t)k * (size_t)batch, kNoAllocMaxElements);
        std::fflush(stderr);
        return kNoAllocTooLarge;
    }
    std::lock_guard<std::recursive_mutex> lock(mutex);
    require(id >= 0 && id < cuda_device_count());
    require(k > 0 && k <= 16384 && k % 32 == 0 && n > 0 && batch > 0 && n <= INT_MAX / batch);
    require((size_t)n * batch <= INT_MAX / 4 && (size_t)n <= INT_MAX / (size_t)k);
    require(y && w && x && scales && maximum);
    DeviceState &d = devices[id];
    if (!d.ready) {
        std::fprintf(stderr, "k200_matmul_i8_noalloc: device %d is not set up; call k200_select(%d) once first\n",
                     id, id);
        std::fflush(stderr);
        return kNoAllocNotReady;
    }
    kunlun::select(id);  // the state exists, so this only makes the device current
    if (!d.noalloc_scratch) return (int)cudaErrorInvalidSymbol;  // set-up records it or aborts
    const size_t count = (size_t)k * batch;
    int8_t *q = static_cast<int8_t *>(d.noalloc_scratch);
    float *maxima = reinterpret_cast<float *>(static_cast<char *>(d.noalloc_scratch) + kNoAllocParamsOffset);
    void *words = static_cast<char *>(d.noalloc_scratch) + kNoAllocParamsOffset + 64;
    // launch_a8_tensor zeroes the reduction words itself before the
    // multi-CTA passes (cudaMemsetAsync, no allocation); the single-CTA form
    // writes every word it reads.
    cudaError_t e = launch_a8_tensor(static_cast<const float *>(x), count, q, maxima, words, d.info, d.stream);
    if (e != cudaSuccess) return (int)e;
    GemvRequest r{};
    r.wt = (int)WeightType::rowwise_i8;
    r.w = w;
    r.y = static_cast<float *>(y);
    r.k = k;
    r.n = n;
    r.batch = batch;
    r.x_stride = k;
    r.y_stride = n;
    r.q = q;
    r.q_stride = k;
    r.q_comp = (long long)count;
    r.act_max = maxima;
    r.row_scale = scales;
    r.prefetch_weights = d.static_weights;
    r.tensor_cores = d.tensor_cores;
    e = launch_gemv(r, d.info, d.stream);
    if (e != cudaSuccess) return (int)e;
    ++d.matmuls;
    return 0;
}
}  // namespace k200
