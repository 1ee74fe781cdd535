// Q6_K typed GEMV behind the reference's API (k200.h:135-165, src/q6-k.inc):
// Q6KWeight, Q6KWorkspace and q6_k_matmul.
//
// Design on B200:
//  * upload() moves the caller's raw GGML Q6_K blocks to the device as they
//    are and unpacks them there (q6_unpack_kernel): int8 values q - 32 in the
//    [N32 tile][K16 group][16][32 rows] layout the GEMV streams, and one f32
//    scale d * sub-scale per row and group.  A block whose fp16 d is Inf or
//    NaN makes the upload abort, as the reference's host pack does.
//    statistics(): pack_ms is the device unpack, upload_ms the raw copy, and
//    upload_bytes the packed payload written into the weight's storage;
//  * q6_k_matmul() quantises all m activation rows in one launch and runs the
//    GEMV of all m rows in one more (the reference launches both per row);
//    `calls` still counts rows.  The workspace holds the [m][k] int8
//    activations and their [m][k/256] chunk scales, grown on demand.
#include <kunlun/k200.h>

#include <chrono>
#include <climits>
#include <cstdint>
#include <memory>

#include <cuda_runtime.h>

#include "k200_internal.h"

namespace kunlun {

namespace {

using Clock = std::chrono::steady_clock;

double elapsed_ms(Clock::time_point since) {
    return std::chrono::duration<double, std::milli>(Clock::now() - since).count();
}

// True when [a, a + an) and [b, b + bn) share a byte; both spans must be
// representable.
bool intersects(const void *a, size_t an, const void *b, size_t bn) {
    const uintptr_t lo_a = reinterpret_cast<uintptr_t>(a), lo_b = reinterpret_cast<uintptr_t>(b);
    require(lo_a <= UINTPTR_MAX - an && lo_b <= UINTPTR_MAX - bn);
    return lo_a < lo_b + bn && lo_b < lo_a + an;
}

bool valid_device(int id) {
    int count = 0;
    return device_count(&count) == 0 && id >= 0 && id < count;
}

constexpr size_t kRawBlockBytes = 210;

size_t raw_bytes(int k, int n) { return static_cast<size_t>(n) * (k / 256) * kRawBlockBytes; }

}  // namespace

bool q6_k_supported(int k, int n) {
    const bool k_ok = k >= 256 && k <= 4096 && k % 256 == 0;
    const bool n_ok = n >= 32 && n <= 32000 && n % 32 == 0;
    return k_ok && n_ok;
}

size_t q6_k_size(int k, int n) {
    if (!q6_k_supported(k, n)) return 0;
    const size_t values = aligned(static_cast<size_t>(k) * n);   // int8 weights
    const size_t scales = static_cast<size_t>(k / 16) * n * 4;   // f32 group scales
    return values + scales;
}

struct Q6KWeight::Impl {
    Q6KInfo info{};
    Q6KStatistics stats{};
    std::unique_ptr<Buffer> own;   // set when the weight allocated its storage
    void *payload = nullptr;
    bool uploaded = false;
};

Q6KWeight::Q6KWeight(int id, int k, int n, void *storage, size_t bytes) : impl_(new Impl{}) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    require(valid_device(id) && q6_k_supported(k, n));
    Impl &w = *impl_;
    w.info.abi_version = 1;
    w.info.device = id;
    w.info.k = k;
    w.info.n = n;
    w.info.scale_offset = aligned(static_cast<size_t>(k) * n);
    w.info.payload_bytes = q6_k_size(k, n);
    if (storage == nullptr) {
        w.own = std::make_unique<Buffer>(id, w.info.payload_bytes);
        w.payload = w.own->data();
    } else {
        require(reinterpret_cast<uintptr_t>(storage) % 256 == 0 && bytes >= w.info.payload_bytes);
        w.payload = storage;
    }
}

Q6KWeight::~Q6KWeight() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    select(impl_->info.device);
    check(wait());  // a GEMV still in flight may read the storage
    delete impl_;
}

Q6KInfo Q6KWeight::info() const { return impl_->info; }
void *Q6KWeight::data() const { return impl_->payload; }

Q6KStatistics Q6KWeight::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return impl_->stats;
}

void Q6KWeight::upload(const void *q6, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Impl &w = *impl_;
    const Q6KInfo &a = w.info;
    require(q6 != nullptr && bytes == raw_bytes(a.k, a.n));
    w.uploaded = false;
    select(a.device);
    check(wait());
    // raw blocks and the unpack status word share one staging allocation
    const size_t status_at = aligned(bytes);
    Buffer staging(a.device, status_at + 256);
    auto *status = reinterpret_cast<int *>(static_cast<char *>(staging.data()) + status_at);
    const int zero = 0;
    Clock::time_point t = Clock::now();
    check(copy(staging.data(), q6, bytes, host_to_device));
    check(copy(status, &zero, sizeof(zero), host_to_device));
    w.stats.upload_ms += elapsed_ms(t);
    t = Clock::now();
    char *dst = static_cast<char *>(w.payload);
    check(static_cast<int>(k200::launch_q6_unpack(static_cast<const uint8_t *>(staging.data()), a.k, a.n,
                                                  reinterpret_cast<int8_t *>(dst),
                                                  reinterpret_cast<float *>(dst + a.scale_offset), status,
                                                  k200::library_stream(a.device))));
    int verdict = 1;
    check(copy(&verdict, status, sizeof(verdict), device_to_host));  // completes the unpack
    w.stats.pack_ms += elapsed_ms(t);
    require(verdict == 0);  // an Inf/NaN block scale
    w.stats.uploads += 1;
    w.stats.upload_bytes += a.payload_bytes;
    w.uploaded = true;
}

struct Q6KWorkspace::Impl {
    int device = -1;
    std::unique_ptr<Buffer> act;   // [rows][k] int8, then [rows][k/256] f32 at scales_at
    size_t scales_at = 0;
    Q6KStatistics stats{};
};

Q6KWorkspace::Q6KWorkspace() : impl_(new Impl{}) {}

Q6KWorkspace::~Q6KWorkspace() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    if (impl_->device >= 0) {
        select(impl_->device);
        check(wait());
    }
    delete impl_;
}

Q6KStatistics Q6KWorkspace::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Q6KStatistics s = impl_->stats;
    s.workspace_bytes = impl_->act ? impl_->act->size() : 0;
    return s;
}

// The reference's KUNLUN_Q6_K_LEGACY diagnostic (partials through HBM)
// computes the same values; this library has one path, so no call is legacy.
size_t Q6KWorkspace::legacy_calls() const { return 0; }

void q6_k_matmul(Q6KWorkspace &workspace, int id, void *y, const Q6KWeight &weight, const void *x, int m,
                 InputType type) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Q6KWorkspace::Impl &ws = *workspace.impl_;
    const Q6KInfo a = weight.info();
    const bool f16 = type == InputType::f16;
    const size_t elem = f16 ? 2 : 4;
    // the reference's acceptance rules (src/q6-k.inc q6_k_matmul)
    require(a.abi_version == 1 && weight.impl_->uploaded && a.device == id && q6_k_supported(a.k, a.n));
    require(m >= 1 && m <= 512 && (type == InputType::f32 || f16));
    require(valid_device(id) && x != nullptr && y != nullptr);
    require(reinterpret_cast<uintptr_t>(y) % 64 == 0 && reinterpret_cast<uintptr_t>(x) % elem == 0);
    const size_t x_span = static_cast<size_t>(a.k) * m * elem, y_span = static_cast<size_t>(a.n) * m * 4;
    require(!intersects(x, x_span, y, y_span));
    require(!intersects(x, x_span, weight.data(), a.payload_bytes));
    require(!intersects(y, y_span, weight.data(), a.payload_bytes));
    if (ws.device < 0) ws.device = id;
    require(ws.device == id);
    select(id);

    const size_t values = aligned(static_cast<size_t>(a.k) * m);
    const size_t need = values + aligned(static_cast<size_t>(a.k / 256) * m * 4);
    if (!ws.act || ws.act->size() < need) {
        check(wait());  // the old buffer may still be read
        ws.act = std::make_unique<Buffer>(id, need);
        ws.scales_at = values;
    }
    auto *q = static_cast<int8_t *>(ws.act->data());
    auto *qscale = reinterpret_cast<float *>(static_cast<char *>(ws.act->data()) + ws.scales_at);
    const char *packed = static_cast<const char *>(weight.data());
    cudaStream_t stream = k200::library_stream(id);
    check(static_cast<int>(k200::launch_q6_quant(x, f16 ? 1 : 0, a.k, m, q, qscale, stream)));
    check(static_cast<int>(k200::launch_q6_gemv(static_cast<float *>(y), reinterpret_cast<const int8_t *>(packed),
                                                reinterpret_cast<const float *>(packed + a.scale_offset), q,
                                                qscale, a.k, a.n, m, k200::device_info(id), stream)));
    check(wait());
    ws.stats.calls += static_cast<size_t>(m);
    k200::count_matmul(id);
}

}  // namespace kunlun
