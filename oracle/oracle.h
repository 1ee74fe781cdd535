/*
 * CPU oracle for the k200 matmul hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference library's arithmetic for
 * Y[batch,n] = X[batch,k] . W^T[n,k] (UnagiDojyou/kunlunK200_lib v0.7.12).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library; the product (libkunlunk200.so) never does.
 *
 * Every function cites the reference file:line it restates.  Floating-point
 * statements are written one IEEE operation per C operation and the file is
 * compiled with -ffp-contract=off, so no fused multiply-add sneaks in.
 *
 * Parity pins (see tests/test_oracle_pins.py):
 *   - fixtures, decode, native pack, common pack, A8 activation model and the
 *     FP64 reference are checked against the reference's own sources compiled
 *     from where they lie (oracle/_ref, built by oracle/Makefile) and against
 *     committed golden vectors (tests/golden/);
 *   - the GGML Q4_0 f32 -> block quantiser is not part of the reference (the
 *     reference only decodes Q4_0); it restates ggml's published
 *     quantize_row_q4_0 and is "parity unpinned" by the reference's tests.
 */
#ifndef K200_ORACLE_H
#define K200_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- generators ---------------------------------------------------------- */
/* xorshift32, bench/native-q4-reference.h:14 */
uint32_t ko_xorshift32(uint32_t *state);
/* uniform [lo,hi) from xorshift32: u = (r >> 8) * 2^-24 */
void ko_fill_uniform(uint32_t seed, float *out, size_t count, float lo, float hi);
/* normal(mean,std) by Box-Muller over two xorshift32 uniforms */
void ko_fill_normal(uint32_t seed, float *out, size_t count, float mean, float std);
/* Weights fixture of bench/native-q4-reference.h:25-55 (random Q4_0 blocks,
 * seed 0x7340d123) -> raw GGML Q4_0 bytes [n][k/32][18]. */
void ko_fixture_q4(int k, int n, uint8_t *q4);
/* Input fixture of bench/native-q4-reference.h:58-69 (seed 0x09200abc). */
void ko_fixture_input(int k, int batch, int pattern, float *x);
/* library-bench closed form, bench/library-bench.cpp:89-101 */
void ko_library_bench_weights(int k, int n, float *w, uint8_t *q4);
void ko_library_bench_input(int k, int batch, float *x);

/* ---- scalar formats ------------------------------------------------------ */
/* half_to_float, kernels/kunlun-matvec.xpu:4-18 (exact, incl. subnormal/Inf/NaN) */
float ko_half_to_float(uint16_t h);
/* IEEE binary32 -> binary16, round to nearest even (used to build F16 inputs) */
uint16_t ko_float_to_half(float f);
void ko_f32_to_f16(const float *in, uint16_t *out, size_t count);

/* ---- Q4_0 ---------------------------------------------------------------- */
/* ggml quantize_row_q4_0 (published algorithm; not in the reference) */
void ko_q4_0_quantize(const float *w, int n, int k, uint8_t *q4);
/* Q4_0 block decode, kernels/kunlun-matvec.xpu:51-59: (nibble - 8) * d */
void ko_q4_0_dequantize(const uint8_t *q4, int n, int k, float *w);

/* ---- legacy matmul (WeightType f32=0, f16=1, q4_0=2) ----------------------- */
/* library-bench gold, bench/library-bench.cpp:121-123: double sum of w*x over
 * the decoded weights, any batch. */
void ko_matmul_gold(const void *w, int type, const float *x, int k, int n, int batch,
                    double *y);
/* kunlun_matvec's FP32 operation order, kernels/kunlun-matvec.xpu:37-77
 * (8-lane products, three lane adds, serial lane reduce, sum += d*s). */
void ko_matvec_model(const void *w, int type, const float *x, int k, int n, int batch,
                     float *y);
/* FP64 reference of bench/native-q4-reference.h:98-108 over decoded weights,
 * run with `threads` OpenMP threads (0 = all). */
void ko_reference_fp64(const float *w, const float *x, int k, int n, int batch, double *y,
                       int threads);
/* Same as ko_reference_fp64 but decodes Q4_0 weights on the fly (the CPU
 * baseline of the Q4_0 GEMV: no decoded-weight copy is materialised). */
void ko_q4_gemv_fp64(const uint8_t *q4, const float *x, int k, int n, int batch, float *y,
                     int threads);

/* ---- rowwise INT8 -------------------------------------------------------- */
size_t ko_aligned(size_t bytes);                       /* src/k200.cpp:98 */
size_t ko_packed_i8_size(int k, int n);                /* src/k200.cpp:99 */
/* upload_i8_rows' row quantiser, src/k200.cpp:102-123.  Returns 0 if a value
 * is non-finite (the reference aborts). */
int ko_i8_pack_rows(const float *w, int k, int n, int8_t *q, float *scales);
/* Per-tensor two-pass activation quantiser, src/k200.cpp:209-229.  Returns 0
 * on a non-finite input (the reference aborts). */
int ko_a8_tensor(const float *x, size_t count, int8_t *q0, int8_t *q1, float *max0,
                 float *max1);
/* Exact int32 dots of both components against the int8 rows
 * (xdnn fc<int8> with unit scales, src/k200.cpp:231) followed by the
 * combine formula of kernels/kunlun-combine.xpu:19 in f32:
 *   y = (float(p0)*(max0/127) + float(p1)*(max1/127)) * scale[row]. */
void ko_i8_matmul(const int8_t *wq, const float *scales, const int8_t *q0, const int8_t *q1,
                  float max0, float max1, int k, int n, int batch, float *y, int32_t *p0,
                  int32_t *p1);

/* ---- native Q4 layout (src/q4-layout.cpp) ---------------------------------- */
int ko_native_q4_supported(int k, int n);              /* q4-layout.cpp:7-9 */
size_t ko_native_q4_size(int k, int n);                /* q4-layout.cpp:10-14 */
int ko_pack_native_q4(uint8_t *dst, size_t bytes, const uint8_t *q4, int k, int n); /* :15-37 */
/* Two-component A8 quantiser of kunlun-native-q4-{max,main,residual}.xpu with
 * the 64-element chunked maxima (the maxima compare |x| bit patterns).
 * dtype 0 = f32 input, 1 = f16 input.  params = {max0/127, max1/127, max0, max1}.
 * q0/q1 are linear [k] int8. */
void ko_native_a8(const void *x, int k, int dtype, int8_t *q0, int8_t *q1, float *params);
/* W4A8x2 GEMV on the native layout: per K32 block
 *   partial = (float(dot0)*s0 + float(dot1)*s1) * d_w
 * then y = sum of partials in increasing block order from 0 (the SD MAC of
 * kernels/native-q4/pipeline.h:32-44,62-67 and q4_sum_partial mode 1,
 * kernels/kunlun-native-q4-sum.xpu:13-24). */
void ko_native_q4_gemv(const uint8_t *native, int k, int n, const int8_t *q0, const int8_t *q1,
                       const float *params, float *y);

/* ---- common Q4 ABI v1 (src/q4-common-pack.h) ------------------------------- */
typedef struct {
    int k, n, kp, np;
    size_t scale_offset, payload_bytes;
} ko_common_info;
int ko_common_describe(int k, int n, ko_common_info *info);       /* :16-20 */
size_t ko_common_weight_index(const ko_common_info *a, int col, int pair); /* :23-27 */
size_t ko_common_scale_index(const ko_common_info *a, int col, int kb);    /* :31 */
int ko_common_pack(const uint8_t *q4, size_t bytes, int k, int n, uint8_t *out); /* :34-41 */
int ko_common_inverse(const uint8_t *packed, int k, int n, uint8_t *q4);         /* :47-52 */
/* Common-layout GEMV (M=1): same arithmetic as ko_native_q4_gemv. */
void ko_common_q4_gemv(const uint8_t *packed, int k, int n, const int8_t *q0, const int8_t *q1,
                       const float *params, float *y);
/* Row-A8 quantiser (quant_row_serial, .../frozen/quant-row-serial-fused.xpu:8-23):
 * per row scale = max|x|/127 (1 if 0), q = round_quant(x * (127/max)). */
void ko_row_a8(const void *x, int m, int k, int dtype, int8_t *q, float *row_scale);
/* Row-A8 x W4 GEMM: per row, per K32 block float(dot)*d_w summed in
 * increasing block order in f32, times the row scale (q40_finish). */
void ko_common_q4_gemm(const uint8_t *packed, int k, int n, const int8_t *q, const float *row_scale,
                       int m, float *y);

#ifdef __cplusplus
}
#endif
#endif
