// extern "C" entry points of libkunlunk200 (declared in include/k200_c.h):
// thin forwards to the kunlun:: C++ API so that FFIs bind unmangled names.
#include <k200_c.h>
#include <kunlun/k200.h>

#include <cuda_runtime.h>

#include <climits>
#include <cstring>

#include "k200_internal.h"

namespace k200 {
void set_stream(int device, cudaStream_t s);
void set_static_weights(int device, bool on);
int current_device();
size_t matmul_count(int device);
bool common_q4_pack(const void *raw, size_t bytes, int k, int n, void *out, size_t out_bytes);
size_t peer_copy_count();
size_t peer_byte_count();
int matmul_q4_gather(int device, const GatherLaunch &g, float *y, const void *w, const void *x, int k, int n,
                     void *scratch, size_t scratch_bytes);
int gather_wait(int device, const unsigned long long *tags, float *y, long long count, const unsigned *counter);
int gather_rows(int device, const GatherLaunch &g, float *y, const float *shard, int n, int batch, int rows);
size_t q4_gather_scratch(int device, int k, int n);
}  // namespace k200

namespace {
bool gather_ok(const k200_gather *g) {
    if (!g || g->ranks < 1 || g->ranks > K200_GATHER_MAX_RANKS || g->rank < 0 || g->rank >= g->ranks || !g->counter ||
        !g->y || g->rows < 1 || g->batch < 1 || (long long)g->rows * g->batch > INT_MAX)
        return false;
    for (int r = 0; r < g->ranks; ++r)
        if (!g->tags[r]) return false;
    return true;
}
}  // namespace

extern "C" {

const char *k200_version(void) { return kunlun::version(); }
int k200_device_count(int *count) { return kunlun::device_count(count); }
void k200_select(int device) { kunlun::select(device); }
int k200_wait(void) { return kunlun::wait(); }
void k200_check(int status) { kunlun::check(status); }
void k200_require(int condition) { kunlun::require(condition != 0); }

int k200_copy(void *dst, const void *src, size_t bytes, int kind) {
    kunlun::require(kind >= 0 && kind <= 2);
    return kunlun::copy(dst, src, bytes, static_cast<kunlun::CopyKind>(kind));
}

void k200_peer(int dst_device, void *dst, int src_device, const void *src, size_t bytes) {
    kunlun::peer(dst_device, dst, src_device, src, bytes);
}

void *k200_allocate(int device, size_t bytes) { return kunlun::allocate(device, bytes); }
void k200_release(int device, void *ptr, size_t bytes) { kunlun::release(device, ptr, bytes); }
size_t k200_allocated_bytes(int device) { return kunlun::allocated_bytes(device); }
void k200_lock(void) { kunlun::runtime_mutex().lock(); }
void k200_unlock(void) { kunlun::runtime_mutex().unlock(); }

void *k200_kernel_create(void) { return new kunlun::Kernel(); }
void k200_kernel_destroy(void *kernel) { delete static_cast<kunlun::Kernel *>(kernel); }

size_t k200_aligned(size_t bytes) { return kunlun::aligned(bytes); }
size_t k200_packed_i8_size(int k, int rows) { return kunlun::packed_i8_size(k, rows); }
float *k200_packed_i8_scales(void *weights, int k, int rows) { return kunlun::packed_i8_scales(weights, k, rows); }
float *k200_packed_i8_maxima(void *weights, int k, int rows) { return kunlun::packed_i8_maxima(weights, k, rows); }
void k200_upload_i8_rows(int device, void *weights, int k, int rows, int first_row, int count,
                         const float *host_input) {
    kunlun::upload_i8_rows(device, weights, k, rows, first_row, count, host_input);
}

void k200_matmul(void *kernel, int device, void *y, const void *w, const void *x, int k, int n, int batch, int type,
                 const float *scales, const float *maxima, int tile) {
    kunlun::require(kernel != nullptr && type >= 0 && type <= 3);
    kunlun::matmul(*static_cast<kunlun::Kernel *>(kernel), device, y, w, x, k, n, batch,
                   static_cast<kunlun::WeightType>(type), scales, maxima, tile);
}

void k200_elementwise(void *kernel, int device, void *y, const void *a, const void *b, int count, int width,
                      int b_count, int op, float parameter) {
    kunlun::require(kernel != nullptr && op >= 0 && op <= 4);
    kunlun::elementwise(*static_cast<kunlun::Kernel *>(kernel), device, y, a, b, count, width, b_count,
                        static_cast<kunlun::ElementwiseOp>(op), parameter);
}

size_t k200_matmul_count(int device) { return k200::matmul_count(device); }
size_t k200_peer_copies(void) { return k200::peer_copy_count(); }
size_t k200_peer_bytes(void) { return k200::peer_byte_count(); }

void *k200_stream(int device) { return static_cast<void *>(k200::library_stream(device)); }

void k200_set_stream(int device, void *stream) { k200::set_stream(device, static_cast<cudaStream_t>(stream)); }

void k200_set_static_weights(int device, int enabled) { k200::set_static_weights(device, enabled != 0); }

// ---- CUDA graphs of library work ----------------------------------------------
int k200_graph_begin(int device) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::select(device);
    const cudaError_t e = cudaStreamBeginCapture(k200::library_stream(device), cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) cudaGetLastError();
    return (int)e;
}

int k200_graph_end(int device, void **graph) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(graph != nullptr);
    kunlun::select(device);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(k200::library_stream(device), &g);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (g) cudaGraphDestroy(g);
        return (int)e;
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return (int)e;
    }
    *graph = static_cast<void *>(exec);
    return 0;
}

int k200_graph_launch(int device, void *graph) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(graph != nullptr);
    kunlun::select(device);
    return (int)cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), k200::library_stream(device));
}

int k200_graph_destroy(void *graph) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    if (!graph) return 0;
    return (int)cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph));
}

int k200_copy_async(void *dst, const void *src, size_t bytes, int kind) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(kind >= 0 && kind <= 2 && k200::current_device() >= 0);
    const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost
                                                                            : cudaMemcpyDeviceToDevice;
    return (int)cudaMemcpyAsync(dst, src, bytes, k, k200::library_stream(k200::current_device()));
}

int k200_copy_kernel(void *dst, const void *src, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(k200::current_device() >= 0 && (bytes == 0 || (dst && src)));
    const int dev = k200::current_device();
    return (int)k200::launch_copy_kernel(dst, src, bytes, k200::device_info(dev), k200::library_stream(dev));
}

void k200_quantize_q4_0(int device, void *q4, const float *w, int k, int n) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(q4 && w && k > 0 && k % 32 == 0 && n > 0);
    kunlun::require((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    kunlun::select(device);
    kunlun::check((int)k200::launch_q4_0_quantize(w, n, k, static_cast<uint8_t *>(q4), k200::library_stream(device)));
}

void k200_pack_i8_rows_device(int device, void *weights, int k, int rows, int first_row, int count,
                              const float *device_input) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(weights && device_input && k > 0 && rows > 0 && first_row >= 0 && count >= 0 &&
                    first_row <= rows && count <= rows - first_row);
    kunlun::select(device);
    const k200::DeviceInfo &info = k200::device_info(device);
    cudaStream_t s = k200::library_stream(device);
    kunlun::check((int)k200::launch_i8_rows(device_input, k, count,
                                            static_cast<int8_t *>(weights) + (size_t)first_row * k,
                                            kunlun::packed_i8_scales(weights, k, rows) + first_row, info, s));
    static const float maximum[6] = {127, 127, 127, 127, 127, 127};
    kunlun::check((int)cudaMemcpyAsync(kunlun::packed_i8_maxima(weights, k, rows), maximum, sizeof(maximum),
                                       cudaMemcpyHostToDevice, s));
}

int k200_matmul_i8_noalloc(int device, void *y, const void *w, const void *x, int k, int n, int batch,
                           const float *scales, const float *maxima) {
    static_assert(K200_NOALLOC_MAX_ELEMENTS == k200::kNoAllocMaxElements, "k200_c.h limit out of date");
    static_assert(K200_NOALLOC_TOO_LARGE == k200::kNoAllocTooLarge, "k200_c.h status out of date");
    static_assert(K200_NOALLOC_NOT_READY == k200::kNoAllocNotReady, "k200_c.h status out of date");
    return k200::matmul_i8_noalloc(device, y, w, x, k, n, batch, scales, maxima);
}

// ---- row-sharded Q4_0 GEMV with a fused all-gather ---------------------------
int k200_ipc_handle(const void *device_ptr, void *handle) {
    kunlun::require(device_ptr && handle);
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(device_ptr));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return (int)e;
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

int k200_ipc_open(int device, const void *handle, void **device_ptr) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(handle && device_ptr);
    kunlun::select(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) cudaGetLastError();
    return (int)e;
}

int k200_ipc_close(int device, void *device_ptr) {
    std::lock_guard<std::recursive_mutex> lock(kunlun::runtime_mutex());
    kunlun::require(device_ptr != nullptr);
    kunlun::select(device);
    const cudaError_t e = cudaIpcCloseMemHandle(device_ptr);
    if (e != cudaSuccess) cudaGetLastError();
    return (int)e;
}

size_t k200_matmul_q4_gather_scratch(int device, int k, int n) { return k200::q4_gather_scratch(device, k, n); }

int k200_matmul_q4_gather(int device, const k200_gather *out, int row_begin, const void *w, const void *x, int k,
                          int n, void *scratch, size_t scratch_bytes, const k200_gather *wait_for) {
    static_assert(K200_GATHER_MAX_RANKS == k200::kGatherMaxRanks, "k200_c.h rank limit out of date");
    kunlun::require(gather_ok(out) && (!wait_for || gather_ok(wait_for)) && row_begin >= 0 && n > 0 && x);
    // one column: the rows are stored as tagged words into every rank's tag array
    kunlun::require(out->batch == 1 && n <= out->rows && row_begin <= out->rows - n);
    k200::GatherLaunch g;
    g.ranks = out->ranks;
    g.rank = out->rank;
    for (int r = 0; r < out->ranks; ++r) g.tags[r] = out->tags[r] + row_begin;
    g.counter = out->counter;
    if (wait_for) {
        // X lies in wait_for's own output buffer; its tagged words sit at the same offset
        const float *base = wait_for->y;
        const float *xf = static_cast<const float *>(x);
        const long long extent = (long long)wait_for->rows * wait_for->batch;
        kunlun::require(xf >= base && xf - base <= extent);
        const long long offset = xf - base;
        g.wait_tags = wait_for->tags[wait_for->rank] + offset;
        g.wait_counter = wait_for->counter;
        g.wait_tagged = (int)(extent - offset);
    }
    return k200::matmul_q4_gather(device, g, out->y + row_begin, w, x, k, n, scratch, scratch_bytes);
}

int k200_gather_rows(int device, const k200_gather *out, int row_begin, const float *shard, int n, int batch) {
    kunlun::require(gather_ok(out) && shard && row_begin >= 0 && n > 0 && batch > 0);
    kunlun::require(batch == out->batch && n <= out->rows && row_begin <= out->rows - n);
    k200::GatherLaunch g;
    g.ranks = out->ranks;
    g.rank = out->rank;
    for (int r = 0; r < out->ranks; ++r) g.tags[r] = out->tags[r] + row_begin;
    g.counter = out->counter;
    return k200::gather_rows(device, g, out->y + row_begin, shard, n, batch, out->rows);
}

int k200_gather_wait(int device, const k200_gather *exchange) {
    kunlun::require(gather_ok(exchange));
    return k200::gather_wait(device, exchange->tags[exchange->rank], exchange->y,
                             (long long)exchange->rows * exchange->batch, exchange->counter);
}

// ---- native Q4 layout ---------------------------------------------------------
int k200_native_q4_layout_supported(int k, int n) { return kunlun::native_q4_layout_supported(k, n) ? 1 : 0; }
size_t k200_native_q4_size(int k, int n) { return kunlun::native_q4_size(k, n); }
int k200_pack_native_q4(void *destination, size_t bytes, const void *q4, int k, int n) {
    return kunlun::pack_native_q4(destination, bytes, q4, k, n) ? 1 : 0;
}
void k200_upload_native_q4(int device, void *weights, const void *q4, int k, int n) {
    kunlun::upload_native_q4(device, weights, q4, k, n);
}
const char *k200_native_q4_reason(int k, int n, int batch, int type) {
    kunlun::require(type == 0 || type == 1);
    return kunlun::native_q4_reason(k, n, batch, static_cast<kunlun::InputType>(type));
}
void *k200_native_q4_workspace_create(void) { return new kunlun::NativeQ4Workspace(); }
void k200_native_q4_workspace_destroy(void *workspace) { delete static_cast<kunlun::NativeQ4Workspace *>(workspace); }
void k200_native_q4_statistics(void *workspace, size_t out[4]) {
    kunlun::require(workspace && out);
    const kunlun::NativeQ4Statistics s = static_cast<kunlun::NativeQ4Workspace *>(workspace)->statistics();
    out[0] = s.accelerated;
    out[1] = s.fallback;
    out[2] = s.hbm_workspace_bytes;
    out[3] = s.l3_workspace_bytes;
}
int k200_native_q4_matmul(void *workspace, int device, void *y, const void *weights, const void *input, int k, int n,
                          int batch, int type) {
    kunlun::require(workspace && (type == 0 || type == 1));
    return kunlun::native_q4_matmul(*static_cast<kunlun::NativeQ4Workspace *>(workspace), device, y, weights, input, k,
                                    n, batch, static_cast<kunlun::InputType>(type))
               ? 1
               : 0;
}

// ---- common Q4 ABI v1 ---------------------------------------------------------
static_assert(sizeof(k200_common_q4_info) == sizeof(kunlun::CommonQ4Info), "k200_common_q4_info layout");
int k200_common_q4_supported(int k, int n) { return kunlun::common_q4_supported(k, n) ? 1 : 0; }
size_t k200_common_q4_size(int k, int n) { return kunlun::common_q4_size(k, n); }
int k200_common_q4_pack(const void *q4, size_t bytes, int k, int n, void *out, size_t out_bytes) {
    return k200::common_q4_pack(q4, bytes, k, n, out, out_bytes) ? 1 : 0;
}
void *k200_common_q4_weight_create(int device, int k, int n, void *storage, size_t bytes) {
    return new kunlun::CommonQ4Weight(device, k, n, storage, bytes);
}
void k200_common_q4_weight_destroy(void *weight) { delete static_cast<kunlun::CommonQ4Weight *>(weight); }
void k200_common_q4_weight_upload(void *weight, const void *q4, size_t bytes) {
    kunlun::require(weight != nullptr);
    static_cast<kunlun::CommonQ4Weight *>(weight)->upload(q4, bytes);
}
void *k200_common_q4_weight_data(void *weight) {
    kunlun::require(weight != nullptr);
    return static_cast<kunlun::CommonQ4Weight *>(weight)->data();
}
void k200_common_q4_weight_info(void *weight, k200_common_q4_info *out) {
    kunlun::require(weight && out);
    const kunlun::CommonQ4Info a = static_cast<kunlun::CommonQ4Weight *>(weight)->info();
    out->abi_version = a.abi_version;
    out->quant_type = a.quant_type;
    out->layout = a.layout;
    out->scale_order = a.scale_order;
    out->k = a.k;
    out->n = a.n;
    out->kp = a.kp;
    out->np = a.np;
    out->device = a.device;
    out->scale_offset = a.scale_offset;
    out->payload_bytes = a.payload_bytes;
}
void *k200_common_q4_workspace_create(void) { return new kunlun::CommonQ4Workspace(); }
void k200_common_q4_workspace_destroy(void *workspace) { delete static_cast<kunlun::CommonQ4Workspace *>(workspace); }
void k200_common_q4_matmul(void *workspace, int device, void *y, const void *weight, const void *input, int m,
                           int type) {
    kunlun::require(workspace && weight && (type == 0 || type == 1));
    kunlun::common_q4_matmul(*static_cast<kunlun::CommonQ4Workspace *>(workspace), device, y,
                             *static_cast<const kunlun::CommonQ4Weight *>(weight), input, m,
                             static_cast<kunlun::InputType>(type));
}
void k200_common_q4_quantization(void *workspace, const void **values, const void **scales, int out[3]) {
    kunlun::require(workspace && values && scales && out);
    const kunlun::CommonQ4Quantization q = static_cast<kunlun::CommonQ4Workspace *>(workspace)->quantization();
    *values = q.values;
    *scales = q.scales;
    out[0] = q.rows;
    out[1] = q.kp;
    out[2] = q.components;
}
void k200_common_q4_statistics(void *workspace, size_t out[10]) {
    kunlun::require(workspace && out);
    const kunlun::CommonQ4Statistics s = static_cast<kunlun::CommonQ4Workspace *>(workspace)->statistics();
    for (int i = 0; i < 8; ++i) out[i] = s.paths[i];
    out[8] = s.calls;
    out[9] = s.chunks;
}

int k200_get_rows_f32(void *kernel, int device, void *output, size_t output_bytes, const void *input,
                      size_t input_bytes, const int32_t *indices, size_t index_bytes, int k, int n, int rows) {
    return kunlun::get_rows_f32(*static_cast<kunlun::Kernel *>(kernel), device, output, output_bytes, input,
                                input_bytes, indices, index_bytes, k, n, rows)
               ? 1
               : 0;
}

void *k200_common_q4_lease_create(void) { return new kunlun::CommonQ4ActivationLease(); }
void k200_common_q4_lease_destroy(void *lease) { delete static_cast<kunlun::CommonQ4ActivationLease *>(lease); }
void k200_common_q4_lease_reset(void *lease) { static_cast<kunlun::CommonQ4ActivationLease *>(lease)->reset(); }
int k200_common_q4_lease_matches(void *lease, int device, int k, int rows, int type, uint64_t generation) {
    return static_cast<kunlun::CommonQ4ActivationLease *>(lease)->matches(device, k, rows,
                                                                         static_cast<kunlun::InputType>(type),
                                                                         generation)
               ? 1
               : 0;
}
size_t k200_common_q4_lease_chunks(void *lease) { return static_cast<kunlun::CommonQ4ActivationLease *>(lease)->chunks(); }
void k200_common_q4_lease_chunk(void *lease, size_t index, const void **values, const void **scales, int out[5],
                                size_t bytes[2]) {
    kunlun::require(lease && values && scales && out && bytes);
    const kunlun::CommonQ4ActivationChunk c = static_cast<kunlun::CommonQ4ActivationLease *>(lease)->chunk(index);
    *values = c.values;
    *scales = c.scales;
    out[0] = c.first;
    out[1] = c.rows;
    out[2] = c.padded_rows;
    out[3] = c.kp;
    out[4] = c.components;
    bytes[0] = c.values_bytes;
    bytes[1] = c.scales_bytes;
}
int k200_common_q4_prepare(void *workspace, int device, const void *input, int k, int rows, int type,
                           uint64_t generation, void *lease) {
    return kunlun::common_q4_prepare(*static_cast<kunlun::CommonQ4Workspace *>(workspace), device, input, k, rows,
                                     static_cast<kunlun::InputType>(type), generation,
                                     *static_cast<kunlun::CommonQ4ActivationLease *>(lease))
               ? 1
               : 0;
}
int k200_common_q4_matmul_shared(void *workspace, int device, void *y, void *weight, void *lease, uint64_t generation) {
    return kunlun::common_q4_matmul_shared(*static_cast<kunlun::CommonQ4Workspace *>(workspace), device, y,
                                           *static_cast<kunlun::CommonQ4Weight *>(weight),
                                           *static_cast<kunlun::CommonQ4ActivationLease *>(lease), generation)
               ? 1
               : 0;
}
int k200_common_q4_matmul_pair(void *workspace, int device, void *y0, void *y1, void *weight0, void *weight1,
                               void *lease, uint64_t generation) {
    return kunlun::common_q4_matmul_pair(*static_cast<kunlun::CommonQ4Workspace *>(workspace), device, y0, y1,
                                         *static_cast<kunlun::CommonQ4Weight *>(weight0),
                                         *static_cast<kunlun::CommonQ4Weight *>(weight1),
                                         *static_cast<kunlun::CommonQ4ActivationLease *>(lease), generation)
               ? 1
               : 0;
}
void k200_common_q4_pair_statistics(void *workspace, size_t out[3]) {
    kunlun::require(workspace && out);
    const kunlun::CommonQ4PairStatistics s =
        kunlun::common_q4_pair_statistics(*static_cast<kunlun::CommonQ4Workspace *>(workspace));
    out[0] = s.calls;
    out[1] = s.declined;
    out[2] = s.l3_partial_bytes;
}
int k200_common_q4_pair_last_status(void *workspace) {
    return static_cast<int>(kunlun::common_q4_pair_last_status(*static_cast<kunlun::CommonQ4Workspace *>(workspace)));
}
void k200_common_q4_activation_statistics(void *workspace, size_t out[8]) {
    kunlun::require(workspace && out);
    const kunlun::CommonQ4ActivationStatistics s =
        static_cast<kunlun::CommonQ4Workspace *>(workspace)->activation_statistics();
    const size_t v[8] = {s.prepare_calls,   s.quantized_chunks, s.quant_kernel_launches, s.prepared_matmuls,
                         s.prepared_chunks, s.invalidations,    s.rejected_calls,        s.hbm_activation_bytes};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
}

int k200_q6_k_supported(int k, int n) { return kunlun::q6_k_supported(k, n) ? 1 : 0; }
size_t k200_q6_k_size(int k, int n) { return kunlun::q6_k_size(k, n); }
void *k200_q6_k_weight_create(int device, int k, int n, void *storage, size_t bytes) {
    return new kunlun::Q6KWeight(device, k, n, storage, bytes);
}
void k200_q6_k_weight_destroy(void *weight) { delete static_cast<kunlun::Q6KWeight *>(weight); }
void k200_q6_k_weight_upload(void *weight, const void *q6, size_t bytes) {
    static_cast<kunlun::Q6KWeight *>(weight)->upload(q6, bytes);
}
void *k200_q6_k_weight_data(void *weight) { return static_cast<kunlun::Q6KWeight *>(weight)->data(); }
void *k200_q6_k_workspace_create(void) { return new kunlun::Q6KWorkspace(); }
void k200_q6_k_workspace_destroy(void *workspace) { delete static_cast<kunlun::Q6KWorkspace *>(workspace); }
void k200_q6_k_workspace_statistics(void *workspace, size_t out[4]) {
    kunlun::require(workspace && out);
    const kunlun::Q6KStatistics s = static_cast<kunlun::Q6KWorkspace *>(workspace)->statistics();
    out[0] = s.calls;
    out[1] = s.uploads;
    out[2] = s.upload_bytes;
    out[3] = s.workspace_bytes;
}
void k200_q6_k_matmul(void *workspace, int device, void *y, void *weight, const void *x, int m, int type) {
    kunlun::q6_k_matmul(*static_cast<kunlun::Q6KWorkspace *>(workspace), device, y,
                        *static_cast<kunlun::Q6KWeight *>(weight), x, m, static_cast<kunlun::InputType>(type));
}

const char *k200_swiglu_reason(int width, int rows, int gate_stride, int up_stride, int output_stride, int type) {
    const kunlun::SwiGLULayout p{width, rows, gate_stride, up_stride, output_stride,
                                 static_cast<kunlun::InputType>(type)};
    return kunlun::swiglu_reason(p);
}

int k200_swiglu(void *kernel, int device, void *y, size_t y_bytes, const void *gate, size_t gate_bytes,
                const void *up, size_t up_bytes, int width, int rows, int gate_stride, int up_stride,
                int output_stride, int type) {
    const kunlun::SwiGLULayout p{width, rows, gate_stride, up_stride, output_stride,
                                 static_cast<kunlun::InputType>(type)};
    return kunlun::swiglu(*static_cast<kunlun::Kernel *>(kernel), device, y, y_bytes, gate, gate_bytes, up,
                          up_bytes, p)
               ? 1
               : 0;
}

int k200_common_q4_get_rows(void *kernel, int device, void *output, size_t output_bytes, void *weight,
                            const int32_t *indices, size_t index_bytes, int rows) {
    return kunlun::common_q4_get_rows(*static_cast<kunlun::Kernel *>(kernel), device, output, output_bytes,
                                      *static_cast<kunlun::CommonQ4Weight *>(weight), indices, index_bytes, rows)
               ? 1
               : 0;
}

}  // extern "C"
