// Glue that exposes the reference's own CPU code to the Python tests through a
// C ABI.  TEST INFRASTRUCTURE ONLY: built by oracle/Makefile into oracle/_ref/
// from the reference sources where they lie (REF=<reference checkout>); never
// linked into the product.
//
// Compiled reference units:
//   bench/native-q4-reference.h   Weights / input / Activation / reference()
//   src/q4-common-pack.h          common Q4 ABI v1 Pack and inverse
//   src/q4-layout.cpp             native_q4_size / pack_native_q4
// q4-layout.cpp needs a few kunlun:: runtime symbols; the pack functions only
// use aligned() and require(), the rest are never called from here and abort.
#include <kunlun/k200.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "native-q4-reference.h"
#include "q4-common-pack.h"

namespace kunlun {
namespace {
std::recursive_mutex glue_mutex;
[[noreturn]] void unavailable() {
    std::fprintf(stderr, "k200 reference glue: runtime call not available on the CPU\n");
    std::abort();
}
}  // namespace
std::recursive_mutex &runtime_mutex() { return glue_mutex; }
void check(int status) { if (status) unavailable(); }
void require(bool ok) { if (!ok) { std::fprintf(stderr, "k200 reference glue: require failed\n"); std::abort(); } }
void select(int) { unavailable(); }
int wait() { unavailable(); }
int copy(void *, const void *, size_t, CopyKind) { unavailable(); }
size_t aligned(size_t n) { require(n <= SIZE_MAX - 255); return (n + 255) & ~size_t(255); }
}  // namespace kunlun

extern "C" {

// native_q4_bench::Weights: raw Q4_0 fixture, decoded f32 weights, the
// bench's own native packing, and the per-row i8 scales it derives.
int ref_fixture(int k, int n, unsigned char *q4, float *decoded, unsigned char *native,
                float *row_scales) {
    native_q4_bench::Weights w(k, n);
    if (q4) std::memcpy(q4, w.q4.data(), w.q4.size());
    if (decoded) std::memcpy(decoded, w.decoded.data(), w.decoded.size() * 4);
    if (native) std::memcpy(native, w.native.data(), w.native.size());
    if (row_scales) std::memcpy(row_scales, w.row_scales.data(), w.row_scales.size() * 4);
    return 1;
}

void ref_input(int k, int batch, int pattern, float *x) {
    auto v = native_q4_bench::input(k, batch, pattern);
    std::memcpy(x, v.data(), v.size() * 4);
}

// native_q4_bench::Activation (linear components, scales, represented input).
void ref_activation(const float *x, int k, int batch, int bits, int components, signed char *linear,
                    float *scales, float *represented) {
    std::vector<float> in(x, x + (size_t)k * batch);
    native_q4_bench::Activation a(in, k, batch, bits, components, false, represented != nullptr);
    std::memcpy(linear, a.linear.data(), a.linear.size());
    for (int i = 0; i < 3; ++i) scales[i] = a.scale[i];
    if (represented) std::memcpy(represented, a.represented.data(), a.represented.size() * 4);
}

void ref_reference(const float *w, const float *x, int k, int n, int batch, double *y) {
    std::vector<float> wv(w, w + (size_t)k * n), xv(x, x + (size_t)k * batch);
    auto r = native_q4_bench::reference(wv, xv, k, n, batch);
    std::memcpy(y, r.data(), r.size() * 8);
}

// The reference FP64 GEMV over `threads` host threads: the unmodified
// reference() (whose OpenMP team size is fixed at 6 in its source) is called on
// disjoint row slices from ceil(threads/6) host threads.  The slices are built
// once (create), so a run times only reference() itself.
struct RefGemv {
    int k = 0, n = 0;
    std::vector<int> first;
    std::vector<std::vector<float>> slices;
};

void *ref_gemv_create(const float *w, int k, int n, int threads) {
    auto *g = new RefGemv();
    g->k = k;
    g->n = n;
    int parts = threads <= 6 ? 1 : (threads + 5) / 6;
    if (parts > n) parts = n;
    for (int s = 0; s < parts; ++s) {
        int a = (int)((long long)n * s / parts), b = (int)((long long)n * (s + 1) / parts);
        g->first.push_back(a);
        g->slices.emplace_back(w + (size_t)a * k, w + (size_t)b * k);
    }
    g->first.push_back(n);
    return g;
}

void ref_gemv_run(void *handle, const float *x, int batch, double *y) {
    auto *g = static_cast<RefGemv *>(handle);
    std::vector<float> xv(x, x + (size_t)g->k * batch);
    std::vector<std::thread> pool;
    for (size_t s = 0; s < g->slices.size(); ++s) {
        pool.emplace_back([g, s, batch, y, &xv] {
            int rows = g->first[s + 1] - g->first[s];
            auto r = native_q4_bench::reference(g->slices[s], xv, g->k, rows, batch);
            for (int b = 0; b < batch; ++b)
                for (int i = 0; i < rows; ++i) y[(size_t)b * g->n + g->first[s] + i] = r[(size_t)b * rows + i];
        });
    }
    for (auto &t : pool) t.join();
}

void ref_gemv_destroy(void *handle) { delete static_cast<RefGemv *>(handle); }

size_t ref_native_q4_size(int k, int n) { return kunlun::native_q4_size(k, n); }
int ref_pack_native_q4(void *dst, size_t bytes, const void *q4, int k, int n) {
    return kunlun::pack_native_q4(dst, bytes, q4, k, n) ? 1 : 0;
}

// common_q4::Pack with the library's ABI choice (Micro32Bank, K-major) unless
// another layout/scale order is requested.  Returns 0 on a rejected shape.
int ref_common_pack(const unsigned char *raw, size_t length, int k, int n, int layout, int scale_order,
                    unsigned char *out, size_t out_bytes, long long *info6) {
    try {
        common_q4::Pack p(raw, length, k, n, common_q4::Layout(layout),
                          common_q4::ScaleOrder(scale_order), true);
        if (info6) {
            info6[0] = p.info.k; info6[1] = p.info.n; info6[2] = p.info.kp; info6[3] = p.info.np;
            info6[4] = (long long)p.info.scale_offset; info6[5] = (long long)p.info.payload_bytes;
        }
        if (out) {
            if (out_bytes < p.bytes.size()) return 0;
            std::memcpy(out, p.bytes.data(), p.bytes.size());
        }
        return 1;
    } catch (...) {
        return 0;
    }
}

}  // extern "C"
