// Host side of the native and common Q4 layouts: the kunlun:: API of the
// reference's src/q4-layout.cpp, src/k200.cpp:477-632 (native_q4_*) and
// src/q4-common.inc:1-334 (common_q4_*), over the kernels of q4_layouts.cu.
//
// Semantics kept from the reference:
//  * every entry point takes runtime_mutex and validates the same contract
//    with require() (device, shape, type, alignment, non-overlap);
//  * native_q4_matmul and common_q4_matmul complete before returning;
//  * native_q4_matmul returns true when it took the W4A8x2 path
//    (native_q4_reason() empty and X, Y 64-byte aligned) and false after the
//    exact FP32 fallback;
//  * a workspace binds to the first device it is used on; CommonQ4Weight
//    owns a Buffer unless given 256-byte-aligned storage;
//  * every call counts in statistics().matmuls.
// Packing runs on the host, as in the reference (the upload is not timed in
// a forward call).
#include <kunlun/k200.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include <cuda_runtime.h>

#include "k200_internal.h"

namespace kunlun {

namespace {

bool overlap(uintptr_t a, size_t as, uintptr_t b, size_t bs) { return !(a + as <= b || b + bs <= a); }

int device_ordinals() {
    int n = 0;
    check(device_count(&n));
    return n;
}

// Q4_0 element j (0..31) of an 18-byte block as a signed value (nibble - 8):
// elements 0-15 in the low nibbles of bytes 2..17, 16-31 in the high nibbles.
int q4_element(const unsigned char *block, int j) { return ((block[2 + (j & 15)] >> (j < 16 ? 0 : 4)) & 15) - 8; }

// A growable device buffer of one workspace.
struct Scratch {
    std::unique_ptr<Buffer> buffer;
    void reserve(int id, size_t bytes) {
        if (buffer && buffer->size() >= bytes) return;
        if (buffer) check(wait());  // in-flight work may still read the old buffer
        buffer.reset(new Buffer(id, bytes));
    }
    void *data() const { return buffer ? buffer->data() : nullptr; }
    size_t size() const { return buffer ? buffer->size() : 0; }
};

// ---- common Q4 ABI v1 geometry (src/q4-common-pack.h:16-31) -----------------
struct CommonGeometry {
    int k, n, kp, np;
    size_t scale_offset, payload_bytes;
};
CommonGeometry common_geometry(int k, int n) {
    CommonGeometry g;
    g.k = k;
    g.n = n;
    const int ka = k < 512 ? 512 : 256;
    g.kp = (k + ka - 1) / ka * ka;
    g.np = (n + 255) / 256 * 256;
    g.scale_offset = (size_t)g.kp * g.np / 2;
    g.payload_bytes = g.scale_offset + (size_t)g.kp * g.np / 16;
    return g;
}
// Byte of pair `pair` (elements 2*pair, 2*pair+1 along K) of column `col` in
// the Micro32Bank payload: 512-byte blocks per (32-column tile, K32 block);
// inside, bank = col % 16 and row = (col % 32 / 16) * 8 + (pair % 16) / 2.
size_t common_weight_byte(const CommonGeometry &g, int col, int pair) {
    const int kb = pair / 16, p = pair % 16;
    const int row = (col % 32 / 16) * 8 + p / 2, bank = col % 16;
    const size_t tile = (size_t)(col / 32) * (g.kp / 32);
    return (tile + kb) * 512 + (size_t)(bank * 16 + row) * 2 + p % 2;
}
// K-major FP16 scales after the payload of nibbles.
size_t common_scale_byte(const CommonGeometry &g, int col, int kb) {
    return g.scale_offset + ((size_t)kb * g.np + col) * 2;
}
void common_pack_host(const unsigned char *raw, const CommonGeometry &g, unsigned char *out) {
    std::memset(out, 0, g.payload_bytes);
    const int blocks = (g.k + 31) / 32;
    for (int c = 0; c < g.n; ++c)
        for (int b = 0; b < blocks; ++b) {
            const unsigned char *block = raw + ((size_t)c * blocks + b) * 18;
            const size_t s = common_scale_byte(g, c, b);
            out[s] = block[0];
            out[s + 1] = block[1];
            for (int p = 0; p < 16; ++p) {
                const int lo = q4_element(block, 2 * p), hi = q4_element(block, 2 * p + 1);
                out[common_weight_byte(g, c, b * 16 + p)] = (unsigned char)((lo & 15) | ((hi & 15) << 4));
            }
        }
}

}  // namespace

// ---------------------------------------------------------------------------
// native layout (src/q4-layout.cpp)
// ---------------------------------------------------------------------------
bool native_q4_layout_supported(int k, int n) { return k > 0 && k <= 16384 && k % 32 == 0 && n > 0 && n <= 90000000 / k; }

size_t native_q4_size(int k, int n) {
    if (!native_q4_layout_supported(k, n)) return 0;
    const size_t rows = ((size_t)n + 31) & ~size_t(31);
    return aligned(rows * k / 2) + aligned(rows * (k / 32) * 2);
}

bool pack_native_q4(void *destination, size_t bytes, const void *source, int k, int n) {
    const size_t need = native_q4_size(k, n);
    if (!need || bytes < need || !destination || !source) return false;
    const uintptr_t dst = (uintptr_t)destination, src = (uintptr_t)source;
    const size_t source_bytes = (size_t)n * (k / 32) * 18;
    if (dst + need < dst || src + source_bytes < src || overlap(dst, need, src, source_bytes)) return false;
    unsigned char *out = static_cast<unsigned char *>(destination);
    const unsigned char *in = static_cast<const unsigned char *>(source);
    const int blocks = k / 32;
    const size_t payload = aligned((((size_t)n + 31) & ~size_t(31)) * k / 2);
    std::memset(out, 0, need);
    // byte [(row/32)*blocks + b][j][row%32] = element 2j (low nibble) | element 2j+1 (high), signed 4-bit
    for (int row = 0; row < n; ++row)
        for (int b = 0; b < blocks; ++b) {
            const unsigned char *block = in + ((size_t)row * blocks + b) * 18;
            const size_t tb = (size_t)(row / 32) * blocks + b;
            out[payload + (tb * 32 + row % 32) * 2] = block[0];
            out[payload + (tb * 32 + row % 32) * 2 + 1] = block[1];
            for (int j = 0; j < 16; ++j) {
                const int lo = q4_element(block, 2 * j), hi = q4_element(block, 2 * j + 1);
                out[tb * 512 + j * 32 + row % 32] = (unsigned char)((lo & 15) | ((hi & 15) << 4));
            }
        }
    return true;
}

void upload_native_q4(int device, void *weights, const void *q4, int k, int n) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    std::vector<unsigned char> packed(native_q4_size(k, n));
    require(pack_native_q4(packed.data(), packed.size(), q4, k, n));
    select(device);
    check(copy(weights, packed.data(), packed.size(), host_to_device));
    check(wait());
}

const char *native_q4_reason(int k, int n, int batch, InputType type) {
    if (!native_q4_layout_supported(k, n)) return "K/N/layout capacity";
    if (type != InputType::f32 && type != InputType::f16) return "input type";
    if (batch != 1) return "batch != 1";
    if (n % 128) return "rows not divisible by 128 (N64 requires 256)";
    if ((size_t)n * (k / 32) * 4 > 16 * 1024 * 1024) return "partial capacity";
    return "";
}

struct NativeQ4Workspace::Impl {
    int id = -1;
    Scratch quant;  // [2][k] int8 components + 16 floats of parameters
    size_t accelerated = 0, fallbacks = 0;
};

NativeQ4Workspace::NativeQ4Workspace() : impl_(new Impl{}) {}
NativeQ4Workspace::~NativeQ4Workspace() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    if (impl_->id >= 0) {
        select(impl_->id);
        check(wait());
    }
    delete impl_;
}
NativeQ4Statistics NativeQ4Workspace::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return {impl_->accelerated, impl_->fallbacks, impl_->quant.size(), 0};
}

bool native_q4_matmul(NativeQ4Workspace &workspace, int id, void *y, const void *weights, const void *input, int k,
                      int n, int batch, InputType type) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    require(id >= 0 && id < device_ordinals() && native_q4_layout_supported(k, n));
    require(type == InputType::f32 || type == InputType::f16);
    require(batch > 0 && (size_t)n * batch <= INT_MAX / 4 && (size_t)k * batch <= INT_MAX / 4);
    require(y && weights && input);
    const uintptr_t yp = (uintptr_t)y, wp = (uintptr_t)weights, xp = (uintptr_t)input;
    const int xbytes = type == InputType::f16 ? 2 : 4;
    const size_t ys = (size_t)n * batch * 4, ws = native_q4_size(k, n), xs = (size_t)k * batch * xbytes;
    require(yp % 4 == 0 && wp % 256 == 0 && xp % xbytes == 0);
    require(yp + ys >= yp && wp + ws >= wp && xp + xs >= xp);
    require(!overlap(yp, ys, wp, ws) && !overlap(yp, ys, xp, xs) && !overlap(wp, ws, xp, xs));
    NativeQ4Workspace::Impl &s = *workspace.impl_;
    require(s.id == -1 || s.id == id);
    s.id = id;
    select(id);
    const k200::DeviceInfo &dev = k200::device_info(id);
    cudaStream_t stream = k200::library_stream(id);
    const size_t payload = aligned((((size_t)n + 31) & ~size_t(31)) * k / 2);
    const uint8_t *w = static_cast<const uint8_t *>(weights);
    const uint16_t *scales = reinterpret_cast<const uint16_t *>(w + payload);
    const int dtype = type == InputType::f16 ? 1 : 0;
    bool accelerated = !*native_q4_reason(k, n, batch, type) && !((yp | xp) & 63);
    if (!accelerated) {
        check((int)k200::launch_native_fallback(w, scales, input, dtype, k, n, batch, static_cast<float *>(y), dev,
                                                stream));
        check(wait());
        ++s.fallbacks;
    } else {
        s.quant.reserve(id, 2 * (size_t)k + 256);
        int8_t *q0 = static_cast<int8_t *>(s.quant.data()), *q1 = q0 + k;
        float *params = reinterpret_cast<float *>(static_cast<char *>(s.quant.data()) + aligned(2 * (size_t)k));
        check((int)k200::launch_a8x2(input, k, dtype, 0, q0, q1, params, stream));
        check((int)k200::launch_native_gemv_a8x2(w, scales, q0, q1, params, k, n, static_cast<float *>(y), dev,
                                                 stream));
        check(wait());
        ++s.accelerated;
    }
    k200::count_matmul(id);
    return accelerated;
}

// ---------------------------------------------------------------------------
// common Q4 ABI v1 (src/q4-common.inc)
// ---------------------------------------------------------------------------
bool common_q4_supported(int k, int n) { return k > 0 && k <= 16384 && n > 0 && n <= 32000; }
size_t common_q4_size(int k, int n) {
    if (!common_q4_supported(k, n)) return 0;
    return common_geometry(k, n).payload_bytes;
}

struct CommonQ4Weight::Impl {
    CommonQ4Info info;
    std::unique_ptr<Buffer> owned;
    void *storage = nullptr;
    bool ready = false;
    CommonQ4WeightStatistics stats{};
};

CommonQ4Weight::CommonQ4Weight(int id, int k, int n, void *storage, size_t bytes) : impl_(new Impl{}) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    require(id >= 0 && id < device_ordinals() && common_q4_supported(k, n));
    const CommonGeometry g = common_geometry(k, n);
    // abi_version 1, quant_type 2 (Q4_0), layout 1 (Micro32Bank), scale_order 1 (K-major)
    impl_->info = {1, 2, 1, 1, k, n, g.kp, g.np, id, g.scale_offset, g.payload_bytes};
    if (!storage) {
        impl_->owned.reset(new Buffer(id, g.payload_bytes));
        storage = impl_->owned->data();
        bytes = g.payload_bytes;
    }
    require((uintptr_t)storage % 256 == 0 && bytes >= g.payload_bytes);
    impl_->storage = storage;
}
CommonQ4Weight::~CommonQ4Weight() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    select(impl_->info.device);
    check(wait());
    delete impl_;
}
CommonQ4Info CommonQ4Weight::info() const { return impl_->info; }
void *CommonQ4Weight::data() const { return impl_->storage; }
CommonQ4WeightStatistics CommonQ4Weight::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return impl_->stats;
}
void CommonQ4Weight::upload(const void *raw, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Impl &s = *impl_;
    const CommonQ4Info &a = s.info;
    require(raw && bytes == (size_t)a.n * ((a.k + 31) / 32) * 18);
    auto t0 = std::chrono::steady_clock::now();
    std::vector<unsigned char> packed(a.payload_bytes);
    common_pack_host(static_cast<const unsigned char *>(raw), common_geometry(a.k, a.n), packed.data());
    s.stats.pack_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    select(a.device);
    check(wait());
    t0 = std::chrono::steady_clock::now();
    check(copy(s.storage, packed.data(), a.payload_bytes, host_to_device));
    check(wait());
    s.stats.upload_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    ++s.stats.uploads;
    s.stats.upload_bytes += a.payload_bytes;
    s.ready = true;
}

// Quantised activations of a workspace, shared with the leases that point at
// them: every new quantisation (prepare, plain matmul) or a reset of the
// current lease moves the epoch on, which retires older leases.
struct ActivationStorage {
    // M = 1: [4*kp + 1024] int8 (component 0 of element j at (j/32)*64 + j%32,
    // component 1 at 2*kp + the same index), then {s0, s1, max0, max1};
    // M > 1: [rows][kp] int8 up to the end of the last 128-row chunk, then one
    // row scale every 16 floats.
    Scratch quant;
    uint64_t epoch = 0;
    bool valid = false;
    CommonQ4ActivationStatistics stats{};
};

namespace {
void invalidate(ActivationStorage &st) {
    if (st.valid) ++st.stats.invalidations;
    st.valid = false;
    require(++st.epoch != 0);
}

// Device pointers of one quantisation in an ActivationStorage.
struct Quantized {
    int8_t *q0 = nullptr, *q1 = nullptr;  // M = 1 components (view layout)
    float *params = nullptr;              // M = 1 {s0, s1, max0, max1}
    int8_t *q = nullptr;                  // M > 1 rows
    float *row_scale = nullptr;           // M > 1, every 16 floats
};

size_t quant_bytes(int kp, int m, size_t &split) {
    if (m == 1) {
        split = aligned(4 * (size_t)kp + 1024);
        return split + 256;
    }
    const size_t rows = (size_t)(m - 1) / 128 * 128 + 128;
    split = aligned(rows * kp);
    return split + rows * 64;
}

// Quantises X [m, k] (two-component A8 for m = 1, Row A8 otherwise) into st.
Quantized quantize(ActivationStorage &st, int id, const void *x, int k, int kp, int m, int dtype,
                   cudaStream_t stream) {
    size_t split = 0;
    st.quant.reserve(id, quant_bytes(kp, m, split));
    Quantized z;
    char *base = static_cast<char *>(st.quant.data());
    if (m == 1) {
        // kernels/native-q4/quant.h:4-10 (src/q4-common.inc:171-238)
        z.q0 = reinterpret_cast<int8_t *>(base);
        z.q1 = z.q0 + 2 * (size_t)kp;
        z.params = reinterpret_cast<float *>(base + split);
        check((int)k200::launch_a8x2(x, k, dtype, kp, z.q0, z.q1, z.params, stream));
    } else {
        // .../quant-row-serial-fused.xpu:8-23
        z.q = reinterpret_cast<int8_t *>(base);
        z.row_scale = reinterpret_cast<float *>(base + split);
        check((int)k200::launch_row_a8(x, m, k, dtype, kp, z.q, z.row_scale, 16, stream));
    }
    ++st.stats.quant_kernel_launches;
    st.stats.quantized_chunks += (size_t)(m + 127) / 128;
    return z;
}

Quantized quantized_of(ActivationStorage &st, int kp, int m) {
    size_t split = 0;
    (void)quant_bytes(kp, m, split);
    Quantized z;
    char *base = static_cast<char *>(st.quant.data());
    if (m == 1) {
        z.q0 = reinterpret_cast<int8_t *>(base);
        z.q1 = z.q0 + 2 * (size_t)kp;
        z.params = reinterpret_cast<float *>(base + split);
    } else {
        z.q = reinterpret_cast<int8_t *>(base);
        z.row_scale = reinterpret_cast<float *>(base + split);
    }
    return z;
}

bool common_abi_ok(const CommonQ4Info &a) {
    const CommonGeometry g = common_geometry(a.k, a.n);
    return a.abi_version == 1 && a.quant_type == 2 && a.layout == 1 && a.scale_order == 1 && a.kp == g.kp &&
           a.np == g.np && a.scale_offset == g.scale_offset && a.payload_bytes == g.payload_bytes;
}
}  // namespace

struct CommonQ4Workspace::Impl {
    int id = -1;
    std::shared_ptr<ActivationStorage> act = std::make_shared<ActivationStorage>();
    CommonQ4Statistics stats{};
    CommonQ4Quantization last{nullptr, nullptr, 0, 0, 0};
    CommonQ4PairStatistics pair_stats{};
    CommonQ4PairStatus pair_status = CommonQ4PairStatus::NotAttempted;

    // Y = W X from the quantised activations z (m rows); the common GEMV or GEMM.
    void run(int id_, const CommonQ4Info &a, const void *wstorage, const Quantized &z, int m, void *y) {
        const k200::DeviceInfo &dev = k200::device_info(id_);
        cudaStream_t stream = k200::library_stream(id_);
        const uint8_t *wb = static_cast<const uint8_t *>(wstorage);
        if (m == 1) {
            check((int)k200::launch_common_gemv_a8x2(wb, a.scale_offset, a.kp, a.np, z.q0, z.q1, z.params, a.k, a.n,
                                                     static_cast<float *>(y), dev, stream));
            ++stats.paths[0];
        } else {
            check((int)k200::launch_common_gemm_a8(wb, a.scale_offset, a.kp, a.np, z.q, z.row_scale, a.k, a.n, m,
                                                   static_cast<float *>(y), stream));
            ++stats.paths[m <= 64 ? 3 : 4];
        }
        stats.chunks += (size_t)(m + 127) / 128;
    }
    void remember(const Quantized &z, int kp, int m) {
        if (m == 1) {
            last = {z.q0, z.params, 1, kp, 2};
        } else {
            // the view holds the last chunk of up to 128 rows, as the reference's does
            const int first = (m - 1) / 128 * 128;
            last = {z.q + (size_t)first * kp, z.row_scale + (size_t)first * 16, m - first, kp, 1};
        }
    }
};

struct CommonQ4ActivationLease::Impl {
    std::shared_ptr<ActivationStorage> storage;
    uint64_t epoch = 0, generation = 0;
    int id = -1, k = 0, m = 0;
    InputType type = InputType::f32;
    const void *input = nullptr;
    size_t input_bytes = 0;
    std::vector<CommonQ4ActivationChunk> chunks;
    bool current() const { return storage && storage->valid && epoch == storage->epoch; }
};

CommonQ4Workspace::CommonQ4Workspace() : impl_(new Impl{}) {}
CommonQ4Workspace::~CommonQ4Workspace() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    invalidate(*impl_->act);
    if (impl_->id >= 0) {
        select(impl_->id);
        check(wait());
    }
    delete impl_;
}
CommonQ4Statistics CommonQ4Workspace::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    CommonQ4Statistics s = impl_->stats;
    s.hbm_workspace_bytes = impl_->act->quant.size();
    return s;
}
CommonQ4ActivationStatistics CommonQ4Workspace::activation_statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    CommonQ4ActivationStatistics st = impl_->act->stats;
    st.hbm_activation_bytes = impl_->act->quant.size();
    return st;
}
CommonQ4MacStatistics CommonQ4Workspace::mac_statistics() const { return {0, 0, 0, 0}; }
CommonQ4Quantization CommonQ4Workspace::quantization() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return impl_->last;
}

void common_q4_matmul(CommonQ4Workspace &workspace, int id, void *y, const CommonQ4Weight &weight, const void *input,
                      int m, InputType type) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    const CommonQ4Weight::Impl &w = *weight.impl_;
    const CommonQ4Info &a = w.info;
    CommonQ4Workspace::Impl &s = *workspace.impl_;
    require(w.ready && id == a.device && common_q4_supported(a.k, a.n));
    require(common_abi_ok(a));
    require(m > 0 && (size_t)m * a.k <= INT_MAX / 4 && (size_t)m * a.n <= INT_MAX / 4 && input && y &&
            (type == InputType::f32 || type == InputType::f16));
    const int xbytes = type == InputType::f16 ? 2 : 4;
    const uintptr_t yp = (uintptr_t)y, xp = (uintptr_t)input, wp = (uintptr_t)w.storage;
    const size_t ys = (size_t)m * a.n * 4, xs = (size_t)m * a.k * xbytes, ws = a.payload_bytes;
    require(yp % 4 == 0 && xp % xbytes == 0 && wp % 256 == 0 && yp + ys >= yp && xp + xs >= xp && wp + ws >= wp);
    require(!overlap(yp, ys, xp, xs) && !overlap(yp, ys, wp, ws) && !overlap(xp, xs, wp, ws));
    require(s.id == -1 || s.id == id);
    s.id = id;
    select(id);
    invalidate(*s.act);  // this call's quantisation retires any lease
    const Quantized z = quantize(*s.act, id, input, a.k, a.kp, m, type == InputType::f16 ? 1 : 0,
                                 k200::library_stream(id));
    s.run(id, a, w.storage, z, m, y);
    s.remember(z, a.kp, m);
    check(wait());
    ++s.stats.calls;
    k200::count_matmul(id);
}

// ---------------------------------------------------------------------------
// activation lease (src/q4-activation.inc)
// ---------------------------------------------------------------------------
CommonQ4ActivationLease::CommonQ4ActivationLease() : impl_(new Impl{}) {}
CommonQ4ActivationLease::~CommonQ4ActivationLease() {
    reset();
    delete impl_;
}
void CommonQ4ActivationLease::reset() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Impl &l = *impl_;
    if (l.current()) invalidate(*l.storage);
    l.storage.reset();
    l.chunks.clear();
    l.epoch = l.generation = 0;
}
bool CommonQ4ActivationLease::matches(int id, int k, int m, InputType type, uint64_t generation) const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    const Impl &l = *impl_;
    return generation && l.current() && l.generation == generation && l.id == id && l.k == k && l.m == m &&
           l.type == type;
}
size_t CommonQ4ActivationLease::chunks() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return impl_->current() ? impl_->chunks.size() : 0;
}
CommonQ4ActivationChunk CommonQ4ActivationLease::chunk(size_t index) const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return index < chunks() ? impl_->chunks[index] : CommonQ4ActivationChunk{};
}

bool common_q4_prepare(CommonQ4Workspace &work, int id, const void *input, int k, int m, InputType type,
                       uint64_t generation, CommonQ4ActivationLease &lease) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    CommonQ4Workspace::Impl &s = *work.impl_;
    ActivationStorage &st = *s.act;
    auto reject = [&]() {
        ++st.stats.rejected_calls;
        return false;
    };
    if (id < 0 || id >= device_ordinals() || !input || !generation || !common_q4_supported(k, 1) || m <= 0 ||
        (size_t)m * k > INT_MAX / 4 || (type != InputType::f32 && type != InputType::f16) || (s.id != -1 && s.id != id))
        return reject();
    const int bytes = type == InputType::f16 ? 2 : 4;
    const uintptr_t xp = (uintptr_t)input;
    const size_t input_bytes = (size_t)m * k * bytes;
    if (xp % bytes || xp + input_bytes < xp) return reject();
    // the workspace's own quantised buffer is not a valid source for overwriting itself
    if (st.quant.data() && overlap(xp, input_bytes, (uintptr_t)st.quant.data(), st.quant.size())) return reject();
    const int kp = common_geometry(k, 1).kp;
    const size_t count = ((size_t)m + 127) / 128;
    const size_t qstride = m == 1 ? (size_t)4 * kp + 1024 : (size_t)128 * kp + 1024;
    if (count * qstride > 16 * 1024 * 1024) return reject();
    lease.reset();
    invalidate(st);
    s.id = id;
    select(id);
    const Quantized z = quantize(st, id, input, k, kp, m, bytes == 2, k200::library_stream(id));
    CommonQ4ActivationLease::Impl &l = *lease.impl_;
    l.storage = s.act;
    l.epoch = st.epoch;
    l.generation = generation;
    l.id = id;
    l.k = k;
    l.m = m;
    l.type = type;
    l.input = input;
    l.input_bytes = input_bytes;
    for (int first = 0; first < m; first += 128) {
        const int rows = std::min(128, m - first);
        const int padded = m == 1 ? 1 : rows <= 8 ? 8 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
        const int defined = m == 1 ? 1 : (padded + 31) / 32 * 32;
        if (m == 1)
            l.chunks.push_back({z.q0, z.params, 0, 1, 1, kp, 2, qstride, 64});
        else
            l.chunks.push_back({z.q + (size_t)first * kp, z.row_scale + (size_t)first * 16, first, rows, padded, kp, 1,
                                (size_t)defined * kp, (size_t)defined * 64});
    }
    s.remember(z, kp, m);
    check(wait());
    st.valid = true;
    ++st.stats.prepare_calls;
    return true;
}

bool common_q4_matmul_shared(CommonQ4Workspace &work, int id, void *y, const CommonQ4Weight &weight,
                             const CommonQ4ActivationLease &lease, uint64_t generation) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    CommonQ4Workspace::Impl &s = *work.impl_;
    const CommonQ4ActivationLease::Impl &l = *lease.impl_;
    const CommonQ4Weight::Impl &w = *weight.impl_;
    const CommonQ4Info &a = w.info;
    auto reject = [&]() {
        ++s.act->stats.rejected_calls;
        return false;
    };
    if (l.storage != s.act || !lease.matches(id, a.k, l.m, l.type, generation) || !w.ready || id != a.device ||
        s.id != id || !y)
        return reject();
    if (!common_abi_ok(a) || (size_t)l.m * a.n > INT_MAX / 4) return reject();
    const uintptr_t yp = (uintptr_t)y, wp = (uintptr_t)w.storage;
    const size_t ys = (size_t)l.m * a.n * 4;
    if (yp % 4 || yp + ys < yp || wp % 256 || wp + a.payload_bytes < wp || overlap(yp, ys, (uintptr_t)l.input, l.input_bytes) ||
        overlap(yp, ys, wp, a.payload_bytes) || overlap((uintptr_t)l.input, l.input_bytes, wp, a.payload_bytes) ||
        overlap(yp, ys, (uintptr_t)s.act->quant.data(), s.act->quant.size()))
        return reject();
    select(id);
    s.run(id, a, w.storage, quantized_of(*s.act, a.kp, l.m), l.m, y);
    check(wait());
    ++s.stats.calls;
    k200::count_matmul(id);
    ++s.act->stats.prepared_matmuls;
    s.act->stats.prepared_chunks += l.chunks.size();
    return true;
}

// ---------------------------------------------------------------------------
// gate/up pair (src/q4-pair.inc)
// ---------------------------------------------------------------------------
CommonQ4PairStatistics common_q4_pair_statistics(const CommonQ4Workspace &work) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return work.impl_->pair_stats;
}
CommonQ4PairStatus common_q4_pair_last_status(const CommonQ4Workspace &work) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return work.impl_->pair_status;
}

bool common_q4_matmul_pair(CommonQ4Workspace &work, int id, void *y0, void *y1, const CommonQ4Weight &weight0,
                           const CommonQ4Weight &weight1, const CommonQ4ActivationLease &lease, uint64_t generation) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    CommonQ4Workspace::Impl &s = *work.impl_;
    const CommonQ4ActivationLease::Impl &l = *lease.impl_;
    const CommonQ4Weight::Impl &w0 = *weight0.impl_, &w1 = *weight1.impl_;
    const CommonQ4Info &a = w0.info, &b = w1.info;
    auto reject = [&](CommonQ4PairStatus reason) {
        ++s.pair_stats.declined;
        s.pair_status = reason;
        return false;
    };
    const char *flag = std::getenv("GGML_KUNLUN_Q4_GATE_UP_PAIR");
    if (flag && std::strcmp(flag, "auto") && std::strcmp(flag, "1")) return reject(CommonQ4PairStatus::Disabled);
    if (id < 0 || id >= device_ordinals() || s.id != id || !y0 || !y1 || !w0.ready || !w1.ready || a.device != id ||
        b.device != id || a.k != b.k || a.n != b.n || !((a.k == 4096 && a.n == 11008) || (a.k == 2048 && a.n == 5632)))
        return reject(CommonQ4PairStatus::InvalidInput);
    if (l.storage != s.act || l.m != 1 || l.type != InputType::f32 ||
        !lease.matches(id, a.k, 1, InputType::f32, generation) || l.chunks.size() != 1)
        return reject(CommonQ4PairStatus::Lease);
    for (const CommonQ4Info *v : {&a, &b})
        if (!common_abi_ok(*v) || v->k != v->kp || v->n != v->np) return reject(CommonQ4PairStatus::WeightAbi);
    struct Range {
        uintptr_t p;
        size_t bytes;
    };
    const Range outputs[] = {{(uintptr_t)y0, (size_t)a.n * 4}, {(uintptr_t)y1, (size_t)a.n * 4}};
    const Range inputs[] = {{(uintptr_t)w0.storage, a.payload_bytes},
                            {(uintptr_t)w1.storage, b.payload_bytes},
                            {(uintptr_t)l.input, l.input_bytes},
                            {(uintptr_t)s.act->quant.data(), s.act->quant.size()}};
    auto ov = [](const Range &x, const Range &yv) { return overlap(x.p, x.bytes, yv.p, yv.bytes); };
    for (const Range &x : outputs)
        if (x.p % 64 || x.bytes > UINTPTR_MAX - x.p) return reject(CommonQ4PairStatus::Alias);
    for (const Range &x : inputs)
        if (!x.p || x.bytes > UINTPTR_MAX - x.p) return reject(CommonQ4PairStatus::Alias);
    if (ov(outputs[0], outputs[1]) || w0.storage == w1.storage || (uintptr_t)w0.storage % 256 ||
        (uintptr_t)w1.storage % 256 || ov(inputs[0], inputs[2]) || ov(inputs[1], inputs[2]))
        return reject(CommonQ4PairStatus::Alias);
    for (const Range &x : outputs)
        for (const Range &in : inputs)
            if (ov(x, in)) return reject(CommonQ4PairStatus::Alias);
    const CommonQ4ActivationChunk &chunk = l.chunks[0];
    if (chunk.kp != a.k || chunk.rows != 1 || chunk.padded_rows != 1 || chunk.components != 2)
        return reject(CommonQ4PairStatus::Lease);
    select(id);
    const Quantized z = quantized_of(*s.act, a.kp, 1);
    check((int)k200::launch_common_gemv_pair(static_cast<const uint8_t *>(w0.storage),
                                             static_cast<const uint8_t *>(w1.storage), a.scale_offset, a.kp, a.np,
                                             z.q0, z.q1, z.params, a.k, a.n, static_cast<float *>(y0),
                                             static_cast<float *>(y1), k200::device_info(id),
                                             k200::library_stream(id)));
    check(wait());
    s.last = {z.q0, z.params, 1, a.kp, 2};
    s.stats.paths[0] += 2;
    s.stats.calls += 2;
    s.stats.chunks += 2;
    k200::count_matmul(id);
    k200::count_matmul(id);
    s.act->stats.prepared_matmuls += 2;
    s.act->stats.prepared_chunks += 2;
    s.pair_status = CommonQ4PairStatus::Success;
    ++s.pair_stats.calls;
    return true;
}

}  // namespace kunlun

namespace k200 {
// Host pack of N rows of Q4_0 blocks into the common ABI v1 payload (the
// packing CommonQ4Weight::upload performs before its copy).
bool common_q4_pack(const void *raw, size_t bytes, int k, int n, void *out, size_t out_bytes) {
    if (!kunlun::common_q4_supported(k, n) || !raw || !out) return false;
    const kunlun::CommonGeometry g = kunlun::common_geometry(k, n);
    if (bytes != (size_t)n * ((k + 31) / 32) * 18 || out_bytes < g.payload_bytes) return false;
    kunlun::common_pack_host(static_cast<const unsigned char *>(raw), g, static_cast<unsigned char *>(out));
    return true;
}
}  // namespace k200
