// Q6_K weights and GEMV behind the reference's typed API (k200.h:135-165,
// src/q6-k.inc): Q6KWeight (host pack of GGML Q6_K blocks into int8 values
// and f32 group scales, then one upload), Q6KWorkspace and q6_k_matmul.
#include <kunlun/k200.h>

#include <chrono>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include <cuda_runtime.h>

#include "k200_internal.h"

namespace k200 {
cudaStream_t library_stream(int device);
const DeviceInfo &device_info(int device);
void count_matmul(int device);
}  // namespace k200

namespace kunlun {

namespace {

bool spans_overlap(const void *a, size_t as, const void *b, size_t bs) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    require(x <= UINTPTR_MAX - as && y <= UINTPTR_MAX - bs);
    return x < y + bs && y < x + as;
}

int device_total() {
    int n = 0;
    check(device_count(&n));
    return n;
}

// fp16 bits -> float (finite values only; the pack rejects Inf/NaN scales)
float half_value(unsigned h) {
    const int exponent = (h >> 10) & 31;
    require(exponent != 31);
    float d = std::ldexp(float((h & 1023) + (exponent ? 1024 : 0)), exponent ? exponent - 25 : -24);
    return (h & 32768) ? -d : d;
}

// GGML Q6_K block (210 bytes: ql[128], qh[64], int8 scales[16], fp16 d):
// value p (0..255) is ((ql nibble) | (qh pair) << 4) - 32 with
// half = p / 128, l = p % 32, lane = p % 128 / 32, ql byte half*64 + l +
// (lane % 2)*32 (low nibble for lanes 0-1), qh byte 128 + half*32 + l, bits
// 2*lane; its scale is d * scales[p / 16].
std::vector<unsigned char> q6_pack(const unsigned char *raw, size_t bytes, const Q6KInfo &a) {
    require(raw && bytes == (size_t)a.n * (a.k / 256) * 210);
    std::vector<unsigned char> pack(a.payload_bytes, 0);
    const int groups = a.k / 16;
    for (int row = 0; row < a.n; ++row)
        for (int block = 0; block < a.k / 256; ++block) {
            const unsigned char *b = raw + ((size_t)row * (a.k / 256) + block) * 210;
            const float d = half_value(b[208] | (unsigned)b[209] << 8);
            for (int sub = 0; sub < 16; ++sub) {
                const int g = block * 16 + sub;
                const size_t tg = (size_t)(row / 32) * groups + g;
                const float scale = d * (float)(int8_t)b[192 + sub];  // exact in f32
                std::memcpy(pack.data() + a.scale_offset + (tg * 32 + row % 32) * 4, &scale, 4);
                for (int j = 0; j < 16; ++j) {
                    const int p = sub * 16 + j, half = p / 128, l = p % 32, lane = p % 128 / 32;
                    const int lo = half * 64 + l + (lane % 2) * 32;
                    const int nib = lane < 2 ? (b[lo] & 15) : (b[lo] >> 4);
                    const int q = (nib | (((b[128 + half * 32 + l] >> (lane * 2)) & 3) << 4)) - 32;
                    pack[tg * 512 + j * 32 + row % 32] = (unsigned char)(int8_t)q;
                }
            }
        }
    return pack;
}

}  // namespace

bool q6_k_supported(int k, int n) {
    return k >= 256 && k <= 4096 && k % 256 == 0 && n >= 32 && n <= 32000 && n % 32 == 0;
}
size_t q6_k_size(int k, int n) { return q6_k_supported(k, n) ? aligned((size_t)k * n) + (size_t)(k / 16) * n * 4 : 0; }

struct Q6KWeight::Impl {
    Q6KInfo info;
    Q6KStatistics stats{};
    std::unique_ptr<Buffer> owned;
    void *storage = nullptr;
    bool ready = false;
};

Q6KWeight::Q6KWeight(int id, int k, int n, void *storage, size_t bytes) : impl_(new Impl{}) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    require(id >= 0 && id < device_total() && q6_k_supported(k, n));
    Impl &s = *impl_;
    s.info = {1, id, k, n, aligned((size_t)k * n), q6_k_size(k, n)};
    if (!storage) {
        s.owned.reset(new Buffer(id, s.info.payload_bytes));
        storage = s.owned->data();
        bytes = s.info.payload_bytes;
    }
    require((uintptr_t)storage % 256 == 0 && bytes >= s.info.payload_bytes);
    s.storage = storage;
}
Q6KWeight::~Q6KWeight() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    select(impl_->info.device);
    check(wait());
    delete impl_;
}
Q6KInfo Q6KWeight::info() const { return impl_->info; }
void *Q6KWeight::data() const { return impl_->storage; }
Q6KStatistics Q6KWeight::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    return impl_->stats;
}
void Q6KWeight::upload(const void *raw, size_t bytes) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Impl &s = *impl_;
    s.ready = false;
    auto t0 = std::chrono::steady_clock::now();
    const std::vector<unsigned char> pack = q6_pack(static_cast<const unsigned char *>(raw), bytes, s.info);
    s.stats.pack_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    select(s.info.device);
    check(wait());
    t0 = std::chrono::steady_clock::now();
    check(copy(s.storage, pack.data(), pack.size(), host_to_device));
    check(wait());
    s.stats.upload_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    ++s.stats.uploads;
    s.stats.upload_bytes += pack.size();
    s.ready = true;
}

struct Q6KWorkspace::Impl {
    int id = -1;
    std::unique_ptr<Buffer> quant;  // [k] int8, then 256-aligned [k/256] f32 chunk scales
    Q6KStatistics stats{};
};
Q6KWorkspace::Q6KWorkspace() : impl_(new Impl{}) {}
Q6KWorkspace::~Q6KWorkspace() {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    if (impl_->id >= 0) {
        select(impl_->id);
        check(wait());
    }
    delete impl_;
}
Q6KStatistics Q6KWorkspace::statistics() const {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Q6KStatistics s = impl_->stats;
    if (impl_->quant) s.workspace_bytes += impl_->quant->size();
    return s;
}
// One arithmetic path only: the HBM-partials diagnostic mode of the reference
// (KUNLUN_Q6_K_LEGACY=1) computes the same values, so no row is counted here.
size_t Q6KWorkspace::legacy_calls() const { return 0; }

void q6_k_matmul(Q6KWorkspace &workspace, int id, void *y, const Q6KWeight &weight, const void *x, int m,
                 InputType type) {
    std::lock_guard<std::recursive_mutex> lock(runtime_mutex());
    Q6KWorkspace::Impl &s = *workspace.impl_;
    const Q6KInfo a = weight.info();
    require(a.abi_version == 1 && weight.impl_->ready && a.device == id && q6_k_supported(a.k, a.n));
    require(m > 0 && m <= 512 && (type == InputType::f32 || type == InputType::f16));
    const int dtype = type == InputType::f16 ? 1 : 0;
    require(id >= 0 && id < device_total() && y && x && (uintptr_t)y % 64 == 0 && (uintptr_t)x % (dtype ? 2 : 4) == 0);
    const size_t xb = (size_t)a.k * m * (dtype ? 2 : 4), yb = (size_t)a.n * m * 4;
    require(!spans_overlap(x, xb, y, yb) && !spans_overlap(x, xb, weight.data(), a.payload_bytes) &&
            !spans_overlap(y, yb, weight.data(), a.payload_bytes));
    if (s.id < 0) s.id = id;
    require(s.id == id);
    select(id);
    const size_t need = aligned((size_t)a.k) + (size_t)(a.k / 256) * 4;
    if (!s.quant || s.quant->size() < need) {
        if (s.quant) check(wait());
        s.quant.reset(new Buffer(id, need));
    }
    int8_t *q = static_cast<int8_t *>(s.quant->data());
    float *scales = reinterpret_cast<float *>(static_cast<char *>(s.quant->data()) + aligned((size_t)a.k));
    const int8_t *w = static_cast<const int8_t *>(weight.data());
    const float *ws = reinterpret_cast<const float *>(static_cast<const char *>(weight.data()) + a.scale_offset);
    cudaStream_t stream = k200::library_stream(id);
    for (int row = 0; row < m; ++row) {
        const void *input = static_cast<const char *>(x) + (size_t)row * a.k * (dtype ? 2 : 4);
        float *output = static_cast<float *>(y) + (size_t)row * a.n;
        check((int)k200::launch_q6_quant(input, dtype, a.k, q, scales, stream));
        check((int)k200::launch_q6_gemv(output, w, ws, q, scales, a.k, a.n, k200::device_info(id), stream));
        ++s.stats.calls;
    }
    check(wait());
    k200::count_matmul(id);
}

}  // namespace kunlun
