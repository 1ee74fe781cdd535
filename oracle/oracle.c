/*
 * CPU oracle for the k200 matmul hot path -- TEST INFRASTRUCTURE ONLY.
 * Not linked into the product.  See oracle.h for the contract and the pins.
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
static float bits_to_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

uint32_t ko_xorshift32(uint32_t *state) {
    /* bench/native-q4-reference.h:14 */
    uint32_t s = *state;
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    *state = s;
    return s;
}

void ko_fill_uniform(uint32_t seed, float *out, size_t count, float lo, float hi) {
    uint32_t state = seed ? seed : 1u;
    double span = (double)hi - (double)lo;
    for (size_t i = 0; i < count; ++i) {
        double u = (double)(ko_xorshift32(&state) >> 8) * (1.0 / 16777216.0);
        out[i] = (float)((double)lo + span * u);
    }
}

void ko_fill_normal(uint32_t seed, float *out, size_t count, float mean, float std) {
    uint32_t state = seed ? seed : 1u;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < count; i += 2) {
        double u1 = ((double)(ko_xorshift32(&state) >> 8) + 1.0) * (1.0 / 16777217.0);
        double u2 = (double)(ko_xorshift32(&state) >> 8) * (1.0 / 16777216.0);
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(mean + std * r * cos(two_pi * u2));
        if (i + 1 < count) out[i + 1] = (float)(mean + std * r * sin(two_pi * u2));
    }
}

/* ---- scalar formats ----------------------------------------------------- */
float ko_half_to_float(uint16_t h) {
    /* kernels/kunlun-matvec.xpu:4-18 */
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, sign = (uint32_t)(h & 0x8000u) << 16;
    if (e == 0) {
        if (m == 0) return bits_to_float(sign);
        int shift = 0;
        while ((m & 1024u) == 0) { m <<= 1; ++shift; }
        return bits_to_float(sign | ((uint32_t)(113 - shift) << 23) | ((m & 1023u) << 13));
    }
    return bits_to_float(sign | ((e == 31 ? 255u : e + 112u) << 23) | (m << 13));
}

uint16_t ko_float_to_half(float f) {
    uint32_t x = float_to_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;                       /* 24-bit significand -> subnormal */
        uint32_t half = man >> shift;
        uint32_t rest = man & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rest > mid || (rest == mid && (half & 1u))) ++half;
        return (uint16_t)(sign | half);
    }
    uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rest = man & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) ++half; /* may carry into exp: OK */
    return (uint16_t)half;
}

void ko_f32_to_f16(const float *in, uint16_t *out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = ko_float_to_half(in[i]);
}

/* ---- fixtures ----------------------------------------------------------- */
static int nibble(const uint8_t *block, int j) {
    /* bench/native-q4-reference.h:16: element j<16 in the low nibble of byte j,
     * element j>=16 in the high nibble of byte j-16; value nibble-8. */
    return ((block[2 + (j % 16)] >> (j < 16 ? 0 : 4)) & 15) - 8;
}

void ko_fixture_q4(int k, int n, uint8_t *q4) {
    /* bench/native-q4-reference.h:30-41 (no external weight file) */
    uint32_t state = 0x7340d123u;
    int blocks = k / 32;
    for (int row = 0; row < n; ++row) {
        for (int b = 0; b < blocks; ++b) {
            uint8_t *p = q4 + ((size_t)row * blocks + b) * 18;
            uint32_t h = ko_xorshift32(&state);
            float d = ldexpf((float)(8 + (h % 9)) / 1024.f, (int)((h >> 4) % 7) - 3);
            if (h & 0x80000000u) d = -d;
            if ((row * 13 + b) % 257 == 0) d = 0;
            uint16_t hd = ko_float_to_half(d);
            p[0] = (uint8_t)(hd & 255u);
            p[1] = (uint8_t)(hd >> 8);
            for (int j = 0; j < 16; ++j) p[j + 2] = (uint8_t)ko_xorshift32(&state);
        }
    }
}

void ko_fixture_input(int k, int batch, int pattern, float *x) {
    /* bench/native-q4-reference.h:58-69 */
    uint32_t state = 0x09200abcu;
    size_t count = (size_t)k * batch;
    for (size_t j = 0; j < count; ++j) {
        float value = (float)((int)(ko_xorshift32(&state) % 20001u) - 10000) / 8192.f;
        if (pattern == 3) value = (float)((double)(int32_t)ko_xorshift32(&state) / 2147483648.0);
        if (pattern == 4) {
            uint32_t bits = ko_xorshift32(&state);
            bits = (bits & 0x807fffffu) | ((107u + (ko_xorshift32(&state) % 32u)) << 23);
            value = bits_to_float(bits);
        }
        if (pattern == 1 && j % 113 == 0) value *= 1000;
        if (pattern == 2) value = 0;
        x[j] = value;
    }
}

void ko_library_bench_weights(int k, int n, float *w, uint8_t *q4) {
    /* bench/library-bench.cpp:89-100 */
    if (w)
        for (int r = 0; r < n; ++r)
            for (int j = 0; j < k; ++j) w[(size_t)r * k + j] = (float)(((r + j) % 16) - 8) * .0625f;
    if (q4) {
        size_t blocks = (size_t)n * k / 32;
        for (size_t block = 0; block < blocks; ++block) {
            q4[block * 18] = 0x00;
            q4[block * 18 + 1] = 0x2c; /* fp16 0x2c00 = 0.0625 */
            for (int j = 0; j < 16; ++j) {
                int row = (int)(block * 32 / (size_t)k), col = (int)(block * 32 % (size_t)k) + j;
                q4[block * 18 + 2 + j] = (uint8_t)(((row + col) % 16) | (((row + col + 16) % 16) << 4));
            }
        }
    }
}

void ko_library_bench_input(int k, int batch, float *x) {
    /* bench/library-bench.cpp:101: x[j] = sin(j * .017f) in float */
    for (size_t j = 0; j < (size_t)k * batch; ++j) x[j] = sinf((float)j * .017f);
}

/* ---- Q4_0 --------------------------------------------------------------- */
void ko_q4_0_quantize(const float *w, int n, int k, uint8_t *q4) {
    /* ggml quantize_row_q4_0 (published): d = v/-8 for the element v of
     * largest magnitude (first on ties), id = 1/d (0 if d == 0),
     * q = min(15, (int8)(x*id + 8.5)), elements 0..15 low nibbles,
     * 16..31 high nibbles, fp16 d first. */
    int blocks = k / 32;
    for (int r = 0; r < n; ++r) {
        for (int b = 0; b < blocks; ++b) {
            const float *x = w + (size_t)r * k + (size_t)b * 32;
            uint8_t *p = q4 + ((size_t)r * blocks + b) * 18;
            float amax = 0.f, vmax = 0.f;
            for (int j = 0; j < 32; ++j) {
                float a = fabsf(x[j]);
                if (amax < a) { amax = a; vmax = x[j]; }
            }
            float d = vmax / -8.f;
            float id = d != 0.f ? 1.0f / d : 0.0f;
            uint16_t hd = ko_float_to_half(d);
            p[0] = (uint8_t)(hd & 255u);
            p[1] = (uint8_t)(hd >> 8);
            for (int j = 0; j < 16; ++j) {
                float x0 = x[j] * id, x1 = x[16 + j] * id;
                int xi0 = (int)(int8_t)(x0 + 8.5f), xi1 = (int)(int8_t)(x1 + 8.5f);
                if (xi0 > 15) xi0 = 15;
                if (xi1 > 15) xi1 = 15;
                p[2 + j] = (uint8_t)(xi0 | (xi1 << 4));
            }
        }
    }
}

void ko_q4_0_dequantize(const uint8_t *q4, int n, int k, float *w) {
    /* kernels/kunlun-matvec.xpu:51-59 */
    int blocks = k / 32;
    for (int r = 0; r < n; ++r)
        for (int b = 0; b < blocks; ++b) {
            const uint8_t *p = q4 + ((size_t)r * blocks + b) * 18;
            float d = ko_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
            for (int j = 0; j < 32; ++j) w[(size_t)r * k + b * 32 + j] = (float)nibble(p, j) * d;
        }
}

/* Decode one row of any legacy weight type into f32 (exact). */
static void decode_row(const void *w, int type, int k, int row, float *out) {
    if (type == 0) {
        memcpy(out, (const float *)w + (size_t)row * k, (size_t)k * 4);
    } else if (type == 1) {
        const uint16_t *h = (const uint16_t *)w + (size_t)row * k;
        for (int j = 0; j < k; ++j) out[j] = ko_half_to_float(h[j]);
    } else {
        ko_q4_0_dequantize((const uint8_t *)w + (size_t)row * (k / 32) * 18, 1, k, out);
    }
}

void ko_matmul_gold(const void *w, int type, const float *x, int k, int n, int batch, double *y) {
    /* bench/library-bench.cpp:121-123 (double accumulation, serial j).  Rows
     * run in parallel and four columns share a pass over the row, each with
     * its own serial sum, so every output is the same as the serial loop's. */
#ifdef _OPENMP
#pragma omp parallel
#endif
    {
        float *row = (float *)malloc((size_t)k * 4);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int r = 0; r < n; ++r) {
            decode_row(w, type, k, r, row);
            int b = 0;
            for (; b + 4 <= batch; b += 4) {
                const float *x0 = x + (size_t)b * k, *x1 = x0 + k, *x2 = x1 + k, *x3 = x2 + k;
                double g0 = 0, g1 = 0, g2 = 0, g3 = 0;
                for (int j = 0; j < k; ++j) {
                    const double wj = (double)row[j];
                    g0 += wj * (double)x0[j];
                    g1 += wj * (double)x1[j];
                    g2 += wj * (double)x2[j];
                    g3 += wj * (double)x3[j];
                }
                y[(size_t)b * n + r] = g0;
                y[(size_t)(b + 1) * n + r] = g1;
                y[(size_t)(b + 2) * n + r] = g2;
                y[(size_t)(b + 3) * n + r] = g3;
            }
            for (; b < batch; ++b) {
                double gold = 0;
                for (int j = 0; j < k; ++j) gold += (double)row[j] * (double)x[(size_t)b * k + j];
                y[(size_t)b * n + r] = gold;
            }
        }
        free(row);
    }
}

void ko_matvec_model(const void *w, int type, const float *x, int k, int n, int batch, float *y) {
    /* kernels/kunlun-matvec.xpu:37-77.  Per 32-block: acc[l] = q[l]*x[l];
     * acc[l] = acc[l] + q[j+l]*x[j+l] for j = 8,16,24; s = serial sum of acc;
     * sum = sum + d*s. */
    float *row = (float *)malloc((size_t)k * 4);
    for (int r = 0; r < n; ++r) {
        const uint8_t *q4row = (const uint8_t *)w + (size_t)r * (k / 32) * 18;
        if (type != 2) decode_row(w, type, k, r, row);
        for (int c = 0; c < batch; ++c) {
            const float *xv = x + (size_t)c * k;
            float sum = 0;
            for (int b = 0; b < k / 32; ++b) {
                float q[32], d = 1.f;
                if (type == 2) {
                    const uint8_t *p = q4row + (size_t)b * 18;
                    d = ko_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
                    for (int j = 0; j < 32; ++j) q[j] = (float)nibble(p, j);
                } else {
                    for (int j = 0; j < 32; ++j) q[j] = row[b * 32 + j];
                }
                float acc[8];
                for (int l = 0; l < 8; ++l) acc[l] = q[l] * xv[b * 32 + l];
                for (int j = 8; j < 32; j += 8)
                    for (int l = 0; l < 8; ++l) {
                        float prod = q[j + l] * xv[b * 32 + j + l];
                        acc[l] = acc[l] + prod;
                    }
                float s = 0;
                for (int l = 0; l < 8; ++l) s = s + acc[l];
                float t = d * s;
                sum = sum + t;
            }
            y[(size_t)c * n + r] = sum;
        }
    }
    free(row);
}

void ko_reference_fp64(const float *w, const float *x, int k, int n, int batch, double *y,
                       int threads) {
    /* bench/native-q4-reference.h:98-108 */
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_num_procs();
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
    for (int row = 0; row < n; ++row)
        for (int b = 0; b < batch; ++b) {
            double sum = 0;
            for (int j = 0; j < k; ++j) sum += (double)w[(size_t)row * k + j] * (double)x[(size_t)b * k + j];
            y[(size_t)b * n + row] = sum;
        }
    (void)threads;
}

void ko_q4_gemv_fp64(const uint8_t *q4, const float *x, int k, int n, int batch, float *y,
                     int threads) {
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_num_procs();
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
    for (int row = 0; row < n; ++row) {
        float wrow[16384];
        ko_q4_0_dequantize(q4 + (size_t)row * (k / 32) * 18, 1, k, wrow);
        for (int b = 0; b < batch; ++b) {
            double sum = 0;
            for (int j = 0; j < k; ++j) sum += (double)wrow[j] * (double)x[(size_t)b * k + j];
            y[(size_t)b * n + row] = (float)sum;
        }
    }
    (void)threads;
}

/* ---- rowwise INT8 ------------------------------------------------------- */
size_t ko_aligned(size_t n) { return (n + 255) & ~(size_t)255; }
size_t ko_packed_i8_size(int k, int n) {
    return ko_aligned((size_t)k * n) + ko_aligned((size_t)n * 4) + 256;
}

static int round_half_away_127(float value) {
    /* (int)(value + (value >= 0 ? .5f : -.5f)) clamped to +-127,
     * src/k200.cpp:114,217,224 and kernels/native-q4/quant.h:10 */
    float t = value + (value >= 0 ? .5f : -.5f);
    int q = (int)t;
    if (q > 127) q = 127;
    if (q < -127) q = -127;
    return q;
}

int ko_i8_pack_rows(const float *w, int k, int n, int8_t *q, float *scales) {
    /* src/k200.cpp:107-116 */
    for (int r = 0; r < n; ++r) {
        float maximum = 0;
        for (int j = 0; j < k; ++j) {
            float v = w[(size_t)r * k + j];
            if (!isfinite(v)) return 0;
            float a = fabsf(v);
            maximum = maximum > a ? maximum : a;
        }
        scales[r] = maximum > 0 ? maximum / 127 : 1;
        float inv = maximum > 0 ? 127 / maximum : 0;
        for (int j = 0; j < k; ++j) {
            float value = w[(size_t)r * k + j] * inv;
            q[(size_t)r * k + j] = (int8_t)round_half_away_127(value);
        }
    }
    return 1;
}

int ko_a8_tensor(const float *x, size_t count, int8_t *q0, int8_t *q1, float *max0_out,
                 float *max1_out) {
    /* src/k200.cpp:212-225 */
    float max0 = 0, max1 = 0;
    for (size_t j = 0; j < count; ++j) {
        if (!isfinite(x[j])) return 0;
        float a = fabsf(x[j]);
        max0 = max0 > a ? max0 : a;
    }
    if (max0 == 0) max0 = 1;
    float inv0 = 127 / max0, step0 = max0 / 127;
    float *residual = (float *)malloc(count * sizeof(float) + 4);
    for (size_t j = 0; j < count; ++j) {
        float value = x[j] * inv0;
        q0[j] = (int8_t)round_half_away_127(value);
        float back = (float)q0[j] * step0;
        residual[j] = x[j] - back;
        float a = fabsf(residual[j]);
        max1 = max1 > a ? max1 : a;
    }
    if (max1 == 0) max1 = 1;
    float inv1 = 127 / max1;
    for (size_t j = 0; j < count; ++j) {
        float value = residual[j] * inv1;
        q1[j] = (int8_t)round_half_away_127(value);
    }
    free(residual);
    *max0_out = max0;
    *max1_out = max1;
    return 1;
}

void ko_i8_matmul(const int8_t *wq, const float *scales, const int8_t *q0, const int8_t *q1,
                  float max0, float max1, int k, int n, int batch, float *y, int32_t *p0,
                  int32_t *p1) {
    /* src/k200.cpp:231-232 + kernels/kunlun-combine.xpu:19.  The int32 dots
     * are exact in any order; the combine runs per output as written there. */
    float scale0 = max0 / 127.0f, scale1 = max1 / 127.0f;
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(dynamic, 64)
#endif
    for (int c = 0; c < batch; ++c)
        for (int r = 0; r < n; ++r) {
            int32_t d0 = 0, d1 = 0;
            const int8_t *wr = wq + (size_t)r * k;
            const int8_t *a0 = q0 + (size_t)c * k, *a1 = q1 + (size_t)c * k;
#ifdef _OPENMP
#pragma omp simd reduction(+ : d0, d1)
#endif
            for (int j = 0; j < k; ++j) {
                d0 += (int32_t)a0[j] * wr[j];
                d1 += (int32_t)a1[j] * wr[j];
            }
            if (p0) p0[(size_t)c * n + r] = d0;
            if (p1) p1[(size_t)c * n + r] = d1;
            float primary = (float)d0, residual = (float)d1;
            float t0 = primary * scale0;
            float t1 = residual * scale1;
            float t = t0 + t1;
            y[(size_t)c * n + r] = t * scales[r];
        }
}

/* ---- native Q4 ---------------------------------------------------------- */
int ko_native_q4_supported(int k, int n) {
    return k > 0 && k <= 16384 && k % 32 == 0 && n > 0 && n <= 90000000 / k;
}
size_t ko_native_q4_size(int k, int n) {
    if (!ko_native_q4_supported(k, n)) return 0;
    size_t rows = ((size_t)n + 31) & ~(size_t)31;
    return ko_aligned(rows * k / 2) + ko_aligned(rows * (k / 32) * 2);
}
int ko_pack_native_q4(uint8_t *dst, size_t bytes, const uint8_t *q4, int k, int n) {
    /* src/q4-layout.cpp:15-37: [N32 tile][K32 block][16 K pairs][32 N lanes]
     * signed int4 (nibble-8), FP16 scales after the aligned payload at
     * (tile_block*32 + row%32)*2. */
    size_t need = ko_native_q4_size(k, n);
    if (!need || bytes < need || !dst || !q4) return 0;
    size_t payload = ko_aligned((((size_t)n + 31) & ~(size_t)31) * k / 2);
    memset(dst, 0, need);
    int blocks = k / 32;
    for (int row = 0; row < n; ++row)
        for (int b = 0; b < blocks; ++b) {
            const uint8_t *block = q4 + ((size_t)row * blocks + b) * 18;
            size_t tile_block = (size_t)(row / 32) * blocks + b;
            memcpy(dst + payload + (tile_block * 32 + row % 32) * 2, block, 2);
            for (int j = 0; j < 16; ++j) {
                int lo = nibble(block, 2 * j), hi = nibble(block, 2 * j + 1);
                dst[tile_block * 512 + j * 32 + row % 32] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            }
        }
    return 1;
}

static float load_activation(const void *x, int dtype, size_t i) {
    return dtype ? ko_half_to_float(((const uint16_t *)x)[i]) : ((const float *)x)[i];
}

void ko_native_a8(const void *x, int k, int dtype, int8_t *q0, int8_t *q1, float *params) {
    /* kernels/kunlun-native-q4-max.xpu:6-16: max of |x| bit patterns
     * (f16 input: max of the f16 bits, then converted);
     * kernels/native-q4/quant.h:7-9: 0 -> 1.f;
     * kernels/kunlun-native-q4-main.xpu:9-19: q0 = round(x*inverse),
     * r = x - float(q0)*scale;
     * kernels/kunlun-native-q4-residual.xpu:11-18: q1 = round(r*inverse1),
     * params = {max0/127, max1/127, max0, max1}. */
    uint32_t m0 = 0;
    for (int j = 0; j < k; ++j) {
        uint32_t u = dtype ? (uint32_t)(((const uint16_t *)x)[j] & 0x7fffu)
                           : (float_to_bits(((const float *)x)[j]) & 0x7fffffffu);
        if (u > m0) m0 = u;
    }
    if (dtype) m0 = float_to_bits(ko_half_to_float((uint16_t)m0));
    float maximum0 = m0 ? bits_to_float(m0) : 1.f;
    float scale0 = maximum0 / 127.f, inverse0 = 127.f / maximum0;
    float *r = (float *)malloc((size_t)k * 4 + 4);
    uint32_t m1 = 0;
    for (int j = 0; j < k; ++j) {
        float v = load_activation(x, dtype, (size_t)j);
        float scaled = inverse0 * v;
        int q = round_half_away_127(scaled);
        q0[j] = (int8_t)q;
        float back = scale0 * (float)q;
        r[j] = v - back;
        uint32_t u = float_to_bits(r[j]) & 0x7fffffffu;
        if (u > m1) m1 = u;
    }
    float maximum1 = m1 ? bits_to_float(m1) : 1.f;
    float inverse1 = 127.f / maximum1;
    for (int j = 0; j < k; ++j) {
        float scaled = inverse1 * r[j];
        q1[j] = (int8_t)round_half_away_127(scaled);
    }
    free(r);
    params[0] = maximum0 / 127.f;
    params[1] = maximum1 / 127.f;
    params[2] = maximum0;
    params[3] = maximum1;
}

static float block_partial(int32_t dot0, int32_t dot1, float s0, float s1, float d) {
    float a = (float)dot0 * s0;
    float b = (float)dot1 * s1;
    float e = a + b;
    return e * d;
}

void ko_native_q4_gemv(const uint8_t *native, int k, int n, const int8_t *q0, const int8_t *q1,
                       const float *params, float *y) {
    int blocks = k / 32;
    size_t payload = ko_aligned((((size_t)n + 31) & ~(size_t)31) * k / 2);
    for (int row = 0; row < n; ++row) {
        float sum = 0;
        for (int b = 0; b < blocks; ++b) {
            size_t tile_block = (size_t)(row / 32) * blocks + b;
            const uint8_t *s = native + payload + (tile_block * 32 + row % 32) * 2;
            float d = ko_half_to_float((uint16_t)(s[0] | (s[1] << 8)));
            int32_t dot0 = 0, dot1 = 0;
            for (int j = 0; j < 16; ++j) {
                uint8_t v = native[tile_block * 512 + j * 32 + row % 32];
                int lo = (v & 15) >= 8 ? (v & 15) - 16 : (v & 15);
                int hi = (v >> 4) >= 8 ? (v >> 4) - 16 : (v >> 4);
                dot0 += lo * q0[b * 32 + 2 * j] + hi * q0[b * 32 + 2 * j + 1];
                dot1 += lo * q1[b * 32 + 2 * j] + hi * q1[b * 32 + 2 * j + 1];
            }
            float partial = block_partial(dot0, dot1, params[0], params[1], d);
            sum = sum + partial;
        }
        y[row] = sum;
    }
}

/* ---- common Q4 ABI v1 --------------------------------------------------- */
static int round_up(int v, int a) { return (v + a - 1) / a * a; }

int ko_common_describe(int k, int n, ko_common_info *a) {
    /* src/q4-common-pack.h:16-20 (Micro32Bank, K-major scales) */
    if (k < 1 || k > 16384 || n < 1 || n > 32000) return 0;
    a->k = k;
    a->n = n;
    a->kp = round_up(k, k < 512 ? 512 : 256);
    a->np = round_up(n, 256);
    a->scale_offset = (size_t)a->kp * a->np / 2;
    a->payload_bytes = a->scale_offset + (size_t)a->kp * a->np / 16;
    return 1;
}

size_t ko_common_weight_index(const ko_common_info *a, int col, int pair) {
    /* src/q4-common-pack.h:23-27 (Micro32Bank) */
    int kb = pair / 16, p = pair % 16, row = (col % 32 / 16) * 8 + p / 2, bank = col % 16;
    size_t tile = (size_t)(col / 32) * (a->kp / 32);
    return (tile + kb) * 512 + (size_t)(bank * 16 + row) * 2 + p % 2;
}

size_t ko_common_scale_index(const ko_common_info *a, int col, int kb) {
    /* src/q4-common-pack.h:31 (K-major) */
    return a->scale_offset + ((size_t)kb * a->np + col) * 2;
}

int ko_common_pack(const uint8_t *raw, size_t length, int k, int n, uint8_t *out) {
    /* src/q4-common-pack.h:34-41 */
    ko_common_info a;
    if (!ko_common_describe(k, n, &a)) return 0;
    int blocks = (k + 31) / 32;
    if (!raw || length != (size_t)n * blocks * 18) return 0;
    memset(out, 0, a.payload_bytes);
    for (int c = 0; c < n; ++c)
        for (int b = 0; b < blocks; ++b) {
            const uint8_t *src = raw + ((size_t)c * blocks + b) * 18;
            size_t si = ko_common_scale_index(&a, c, b);
            out[si] = src[0];
            out[si + 1] = src[1];
            for (int p = 0; p < 16; ++p) {
                int v0 = nibble(src, p * 2), v1 = nibble(src, p * 2 + 1);
                out[ko_common_weight_index(&a, c, b * 16 + p)] = (uint8_t)((v0 & 15) | ((v1 & 15) << 4));
            }
        }
    return 1;
}

static int common_q(const ko_common_info *a, const uint8_t *packed, int c, int j) {
    int v = (packed[ko_common_weight_index(a, c, j / 2)] >> (j % 2 * 4)) & 15;
    return v >= 8 ? v - 16 : v;
}

int ko_common_inverse(const uint8_t *packed, int k, int n, uint8_t *raw) {
    /* src/q4-common-pack.h:47-52 */
    ko_common_info a;
    if (!ko_common_describe(k, n, &a)) return 0;
    int blocks = (k + 31) / 32;
    for (int c = 0; c < n; ++c)
        for (int b = 0; b < blocks; ++b) {
            size_t o = ((size_t)c * blocks + b) * 18, si = ko_common_scale_index(&a, c, b);
            raw[o] = packed[si];
            raw[o + 1] = packed[si + 1];
            for (int j = 0; j < 16; ++j)
                raw[o + 2 + j] = (uint8_t)((common_q(&a, packed, c, b * 32 + j) + 8) |
                                           ((common_q(&a, packed, c, b * 32 + j + 16) + 8) << 4));
        }
    return 1;
}

void ko_common_q4_gemv(const uint8_t *packed, int k, int n, const int8_t *q0, const int8_t *q1,
                       const float *params, float *y) {
    ko_common_info a;
    if (!ko_common_describe(k, n, &a)) return;
    int blocks = (k + 31) / 32;
    for (int c = 0; c < n; ++c) {
        float sum = 0;
        for (int b = 0; b < blocks; ++b) {
            size_t si = ko_common_scale_index(&a, c, b);
            float d = ko_half_to_float((uint16_t)(packed[si] | (packed[si + 1] << 8)));
            int32_t dot0 = 0, dot1 = 0;
            for (int j = 0; j < 32 && b * 32 + j < k; ++j) {
                int w = common_q(&a, packed, c, b * 32 + j);
                dot0 += w * q0[b * 32 + j];
                dot1 += w * q1[b * 32 + j];
            }
            float partial = block_partial(dot0, dot1, params[0], params[1], d);
            sum = sum + partial;
        }
        y[c] = sum;
    }
}

void ko_row_a8(const void *x, int m, int k, int dtype, int8_t *q, float *row_scale) {
    /* .../frozen/quant-row-serial-fused.xpu:8-23 */
    for (int row = 0; row < m; ++row) {
        uint32_t maximum = 0;
        for (int j = 0; j < k; ++j) {
            float v = load_activation(x, dtype, (size_t)row * k + j);
            uint32_t u = float_to_bits(v) & 0x7fffffffu;
            if (u > maximum) maximum = u;
        }
        float mx = maximum ? bits_to_float(maximum) : 1.f;
        float scale = mx / 127.f, inv = 127.f / mx;
        for (int j = 0; j < k; ++j) {
            float scaled = inv * load_activation(x, dtype, (size_t)row * k + j);
            q[(size_t)row * k + j] = (int8_t)round_half_away_127(scaled);
        }
        row_scale[row] = scale;
    }
}

void ko_common_q4_gemm(const uint8_t *packed, int k, int n, const int8_t *q, const float *row_scale,
                       int m, float *y) {
    ko_common_info a;
    if (!ko_common_describe(k, n, &a)) return;
    int blocks = (k + 31) / 32;
    for (int r = 0; r < m; ++r)
        for (int c = 0; c < n; ++c) {
            float sum = 0;
            for (int b = 0; b < blocks; ++b) {
                size_t si = ko_common_scale_index(&a, c, b);
                float d = ko_half_to_float((uint16_t)(packed[si] | (packed[si + 1] << 8)));
                int32_t dot = 0;
                for (int j = 0; j < 32 && b * 32 + j < k; ++j)
                    dot += common_q(&a, packed, c, b * 32 + j) * q[(size_t)r * k + b * 32 + j];
                float t = (float)dot * d;
                sum = sum + t;
            }
            y[(size_t)r * n + c] = sum * row_scale[r];
        }
}
