/*
 * k200_c.h -- C ABI of libkunlunk200.so.0 (B200 / sm_100a).
 *
 * Plain pointers, sizes and ints: the entry points an FFI (ctypes, cgo, JNI,
 * N-API) binds to reach the kunlun:: matmul hot path without C++ name
 * mangling.  Each function replaces the reference interface cited beside it
 * (UnagiDojyou/kunlunK200_lib v0.7.12, include/kunlun/k200.h and
 * src/k200.cpp) and keeps its argument meaning and error behaviour:
 * contract violations abort with a diagnostic exactly as kunlun::require()
 * does; device statuses are returned as ints (0 = success).
 *
 * Device pointers are CUDA device addresses.  `stream`-free: work goes to the
 * library stream of the device (k200_stream returns it for callers that need
 * to order their own work or record events on it).
 */
#ifndef K200_C_H
#define K200_C_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime: k200.h:10-23, src/k200.cpp:48-95 ---------------------------- */
const char *k200_version(void);                         /* kunlun::version, k200.cpp:634 */
int k200_device_count(int *count);                      /* kunlun::device_count, k200.cpp:63-66 */
void k200_select(int device);                           /* kunlun::select, k200.cpp:67 */
int k200_wait(void);                                    /* kunlun::wait, k200.cpp:68 */
void k200_check(int status);                            /* kunlun::check, k200.cpp:53-55 */
void k200_require(int condition);                       /* kunlun::require, k200.cpp:56-58 */
/* kind: 0 host_to_device, 1 device_to_host, 2 device_to_device */
int k200_copy(void *dst, const void *src, size_t bytes, int kind); /* kunlun::copy, k200.cpp:69-75 */
void k200_peer(int dst_device, void *dst, int src_device, const void *src, size_t bytes); /* kunlun::peer, k200.cpp:89-95 */
void *k200_allocate(int device, size_t bytes);          /* kunlun::allocate, k200.cpp:76-83 */
void k200_release(int device, void *ptr, size_t bytes); /* kunlun::release, k200.cpp:84-87 */
size_t k200_allocated_bytes(int device);                /* kunlun::allocated_bytes, k200.cpp:88 */
void k200_lock(void);                                   /* runtime_mutex().lock(), k200.cpp:48 */
void k200_unlock(void);                                 /* runtime_mutex().unlock() */

/* ---- kernel handle: k200.h:62-88 (kunlun::Kernel) -------------------------- */
void *k200_kernel_create(void);                         /* Kernel::Kernel, k200.cpp:249 */
void k200_kernel_destroy(void *kernel);                 /* Kernel::~Kernel, k200.cpp:250-267 */

/* ---- rowwise int8 packing: k200.h:90-96, src/k200.cpp:98-123 --------------- */
size_t k200_aligned(size_t bytes);
size_t k200_packed_i8_size(int k, int rows);
float *k200_packed_i8_scales(void *weights, int k, int rows);
float *k200_packed_i8_maxima(void *weights, int k, int rows);
void k200_upload_i8_rows(int device, void *weights, int k, int rows, int first_row, int count,
                         const float *host_input);

/* ---- matmul: k200.h:98-105, src/k200.cpp:268-279 --------------------------- */
/* type: 0 f32, 1 f16, 2 q4_0, 3 rowwise_i8 (kunlun::WeightType values) */
void k200_matmul(void *kernel, int device, void *y, const void *w, const void *x, int k, int n, int batch,
                 int type, const float *scales, const float *maxima, int tile);

/* ---- elementwise: k200.h:106-107, src/k200.cpp:280-323 --------------------- */
/* op: 0 add, 1 multiply, 2 silu, 3 rms_norm, 4 scale (kunlun::ElementwiseOp values) */
void k200_elementwise(void *kernel, int device, void *y, const void *a, const void *b, int count, int width,
                      int b_count, int op, float parameter);

/* ---- statistics: k200.h:345-350 -------------------------------------------- */
size_t k200_matmul_count(int device);                   /* Statistics::matmuls[device] */
size_t k200_peer_copies(void);
size_t k200_peer_bytes(void);

/* ---- additions with no reference counterpart -------------------------------- */
/* The library stream of `device` (a cudaStream_t), for event timing and for
 * ordering caller work against library work. */
void *k200_stream(int device);
/* Issue all further work of `device` on `stream` (a cudaStream_t; NULL
 * restores the library's own stream).  wait() then synchronises that stream.
 * Lets a caller order library work inside its own stream or capture it in a
 * CUDA graph; calls that grow scratch (the first rowwise_i8 matmul of a new
 * size) synchronise and must not run during a capture. */
void k200_set_stream(int device, void *stream);
/* Declare that on `device` no kernel immediately preceding a matmul on the
 * library stream writes that matmul's weights (true for inference with
 * resident weights).  Matmul kernels then stream their first weight chunks
 * while the preceding kernel is still finishing (programmatic dependent
 * launch); activations and outputs are still touched only after it
 * completes.  Default off; KUNLUN_STATIC_WEIGHTS=1 turns it on at start-up. */
void k200_set_static_weights(int device, int enabled);
/* Asynchronous copy on the library stream of the current device (pinned host
 * memory makes it truly asynchronous); completion via k200_wait(). */
int k200_copy_async(void *dst, const void *src, size_t bytes, int kind);
/* Copy by a kernel on the library stream of the current device; dst and src
 * are device memory or pinned host memory (which the kernel accesses over
 * the bus).  Unlike k200_copy_async, the copy takes part in the kernels'
 * programmatic-launch chain: a matmul issued after an input copy streams its
 * weights while the copy runs.  Completion via k200_wait(); 0 or a CUDA
 * error code. */
int k200_copy_kernel(void *dst, const void *src, size_t bytes);
/* CUDA graphs of library work.  k200_graph_begin starts capturing the
 * library stream of `device`; the calls that follow on this thread that only
 * submit work (k200_copy_async, k200_matmul, k200_matmul_q4_gather, ...) are
 * recorded instead of run, and k200_graph_end turns the record into a
 * replayable graph (*graph, a cudaGraphExec_t).  k200_graph_launch replays it
 * on the library stream (completion via k200_select + k200_wait), with the
 * pointers, shapes and host buffers it was recorded with: a decode step of
 * H2D input, the chained matmuls and D2H output becomes one launch, and the
 * kernels keep their programmatic-launch overlap.  Calls that complete
 * before returning (k200_wait, k200_copy, elementwise, ...) or that grow
 * scratch (the first matmul of a Kernel at a new size) fail during a
 * capture, so run the sequence once before recording it.  Other threads must
 * not submit work to the device while it is being recorded (hold k200_lock).
 * Replays do not move the matmul counters.  0 or a CUDA error code. */
int k200_graph_begin(int device);
int k200_graph_end(int device, void **graph);
int k200_graph_launch(int device, void *graph);
int k200_graph_destroy(void *graph);
/* GGML Q4_0 quantiser on the device: f32 [n][k] (device) -> 18-byte blocks
 * [n][k/32] (device).  Asynchronous on the library stream. */
void k200_quantize_q4_0(int device, void *q4, const float *w, int k, int n);
/* upload_i8_rows from DEVICE f32 rows (same packing and arithmetic as
 * k200_upload_i8_rows).  Asynchronous on the library stream. */
void k200_pack_i8_rows_device(int device, void *weights, int k, int rows, int first_row, int count,
                              const float *device_input);

/* Rowwise-int8 matmul that allocates nothing.  No counterpart in the
 * reference: kunlun::matmul keeps the quantised activations in scratch owned
 * by the Kernel and grows it with cudaMalloc/cudaFree (after a full
 * synchronisation) whenever batch*k grows.  Callers that cannot allocate at
 * call time -- those that have handed all free device memory to their own
 * pool, or that cannot afford the device-wide synchronisation cudaFree
 * implies in the middle of a serving loop -- use this instead.  The scratch is
 * one fixed array per device in the library's device image, so:
 *   - batch*k must be <= K200_NOALLOC_MAX_ELEMENTS; larger calls return
 *     K200_NOALLOC_TOO_LARGE (with a message on stderr) and do nothing;
 *   - the device must already be set up by k200_select(device), else
 *     K200_NOALLOC_NOT_READY.  That first select on a device is where the
 *     array's memory is taken: it creates the device's stream and error word
 *     and loads the module holding the array (CUDA loads modules lazily), so
 *     a caller that hands the rest of the device to its own pool should
 *     select the device before doing so;
 *   - overlapping calls on one device race on that array: calls issued on the
 *     same stream are ordered, but calls whose work can run concurrently
 *     (issued on different streams, see k200_set_stream) are not, and must be
 *     serialised by the caller.  (Each process has its own copy.)
 * Arguments, packing and results are those of k200_matmul with type 3
 * (rowwise_i8); results are bit-identical, and the same kernels run (the
 * tcgen05 int8 GEMM from batch 4, unless KUNLUN_TC=0).  Returns 0 once the work is
 * submitted (completion via k200_select + k200_wait), a K200_NOALLOC_* status,
 * or a CUDA error code.  Contract violations abort as in k200_matmul. */
#define K200_NOALLOC_MAX_ELEMENTS 2097152
#define K200_NOALLOC_TOO_LARGE (-2)
#define K200_NOALLOC_NOT_READY (-3)
int k200_matmul_i8_noalloc(int device, void *y, const void *w, const void *x, int k, int n, int batch,
                           const float *scales, const float *maxima);

/* ---- native Q4 layout: k200.h:127-131,203-224; src/q4-layout.cpp:7-45;
 *      src/k200.cpp:545-617 ------------------------------------------------- */
/* type: 0 f32 input, 1 f16 input (kunlun::InputType values) */
int k200_native_q4_layout_supported(int k, int n);           /* native_q4_layout_supported, q4-layout.cpp:7-9 */
size_t k200_native_q4_size(int k, int n);                    /* native_q4_size, q4-layout.cpp:10-14 */
int k200_pack_native_q4(void *destination, size_t bytes, const void *q4, int k, int n); /* host pack, q4-layout.cpp:15-37 */
void k200_upload_native_q4(int device, void *weights, const void *q4, int k, int n);   /* q4-layout.cpp:38-44 */
const char *k200_native_q4_reason(int k, int n, int batch, int type);                  /* k200.cpp:545-552 */
void *k200_native_q4_workspace_create(void);                 /* NativeQ4Workspace::NativeQ4Workspace */
void k200_native_q4_workspace_destroy(void *workspace);      /* NativeQ4Workspace::~NativeQ4Workspace */
/* out = {accelerated, fallback, hbm_workspace_bytes, l3_workspace_bytes} */
void k200_native_q4_statistics(void *workspace, size_t out[4]);  /* NativeQ4Workspace::statistics */
/* Completes before returning; 1: W4A8x2 path, 0: exact FP32 fallback. */
int k200_native_q4_matmul(void *workspace, int device, void *y, const void *weights, const void *input, int k, int n,
                          int batch, int type);              /* native_q4_matmul, k200.cpp:553-617 */

/* ---- common Q4 ABI v1: k200.h:226-335; src/q4-common.inc:1-334 ----------- */
typedef struct {
    uint32_t abi_version, quant_type, layout, scale_order;
    int k, n, kp, np, device;
    size_t scale_offset, payload_bytes;
} k200_common_q4_info;                                       /* kunlun::CommonQ4Info */
int k200_common_q4_supported(int k, int n);                  /* q4-common.inc:4 */
size_t k200_common_q4_size(int k, int n);                    /* q4-common.inc:5-8 */
/* Host pack of n rows of Q4_0 blocks into the payload (the packing
 * k200_common_q4_weight_upload performs; src/q4-common-pack.h:34-41).  No
 * device work; 1 on success, 0 on a bad shape or buffer size. */
int k200_common_q4_pack(const void *q4, size_t bytes, int k, int n, void *out, size_t out_bytes);
void *k200_common_q4_weight_create(int device, int k, int n, void *storage, size_t bytes); /* q4-common.inc:16-25 */
void k200_common_q4_weight_destroy(void *weight);
void k200_common_q4_weight_upload(void *weight, const void *q4, size_t bytes);          /* q4-common.inc:32-44 */
void *k200_common_q4_weight_data(void *weight);
void k200_common_q4_weight_info(void *weight, k200_common_q4_info *out);
void *k200_common_q4_workspace_create(void);
void k200_common_q4_workspace_destroy(void *workspace);
/* X [m,k] (type 0 f32, 1 f16), Y [m,n] f32; completes before returning. */
void k200_common_q4_matmul(void *workspace, int device, void *y, const void *weight, const void *input, int m,
                           int type);                        /* common_q4_matmul, q4-common.inc:319-334 */
/* The last call's quantised activations: *values, *scales, out = {rows, kp, components}. */
void k200_common_q4_quantization(void *workspace, const void **values, const void **scales, int out[3]);
/* out = {paths[0..7], calls, chunks} */
void k200_common_q4_statistics(void *workspace, size_t out[10]);

/* Activation lease and gate/up pair (kunlun::CommonQ4ActivationLease,
   common_q4_prepare, common_q4_matmul_shared, common_q4_matmul_pair:
   src/q4-activation.inc:1-98, src/q4-pair.inc:1-80).  The int results are
   1 = done, 0 = declined (nothing written). */
void *k200_common_q4_lease_create(void);
void k200_common_q4_lease_destroy(void *lease);
void k200_common_q4_lease_reset(void *lease);
int k200_common_q4_lease_matches(void *lease, int device, int k, int rows, int type, uint64_t generation);
size_t k200_common_q4_lease_chunks(void *lease);
/* chunk `index`: *values, *scales, out = {first, rows, padded_rows, kp, components}, bytes = {values, scales} */
void k200_common_q4_lease_chunk(void *lease, size_t index, const void **values, const void **scales, int out[5],
                                size_t bytes[2]);
int k200_common_q4_prepare(void *workspace, int device, const void *input, int k, int rows, int type,
                           uint64_t generation, void *lease);
int k200_common_q4_matmul_shared(void *workspace, int device, void *y, void *weight, void *lease, uint64_t generation);
int k200_common_q4_matmul_pair(void *workspace, int device, void *y0, void *y1, void *weight0, void *weight1,
                               void *lease, uint64_t generation);
/* out = {calls, declined, l3_partial_bytes}; the last status is a kunlun::CommonQ4PairStatus value */
void k200_common_q4_pair_statistics(void *workspace, size_t out[3]);
int k200_common_q4_pair_last_status(void *workspace);
/* out = {prepare_calls, quantized_chunks, quant_kernel_launches, prepared_matmuls, prepared_chunks,
          invalidations, rejected_calls, hbm_activation_bytes} */
void k200_common_q4_activation_statistics(void *workspace, size_t out[8]);

/* Q6_K typed GEMV (kunlun::Q6KWeight, Q6KWorkspace, q6_k_matmul:
   src/q6-k.inc:1-142).  type 0 = f32, 1 = f16 activations. */
int k200_q6_k_supported(int k, int n);
size_t k200_q6_k_size(int k, int n);
void *k200_q6_k_weight_create(int device, int k, int n, void *storage, size_t bytes);
void k200_q6_k_weight_destroy(void *weight);
void k200_q6_k_weight_upload(void *weight, const void *q6, size_t bytes);
void *k200_q6_k_weight_data(void *weight);
void *k200_q6_k_workspace_create(void);
void k200_q6_k_workspace_destroy(void *workspace);
/* out = {calls, uploads or 0, upload_bytes or 0, workspace_bytes} of the workspace */
void k200_q6_k_workspace_statistics(void *workspace, size_t out[4]);
void k200_q6_k_matmul(void *workspace, int device, void *y, void *weight, const void *x, int m, int type);

/* Row gathers; 1 = rows written, 0 = contract violation or an index outside
   [0, n) (no output written).  Replace kunlun::get_rows_f32
   (src/get-rows-f32.inc:1-29) and kunlun::common_q4_get_rows
   (src/get-rows.inc:1-26). */
int k200_get_rows_f32(void *kernel, int device, void *output, size_t output_bytes, const void *input,
                      size_t input_bytes, const int32_t *indices, size_t index_bytes, int k, int n, int rows);
int k200_common_q4_get_rows(void *kernel, int device, void *output, size_t output_bytes, void *weight,
                            const int32_t *indices, size_t index_bytes, int rows);

/* Fused SiLU(gate) * up over rows at byte strides; type 0 = f32, 1 = f16.
   Replace kunlun::swiglu_reason / kunlun::swiglu (src/k200.cpp:324-368);
   k200_swiglu returns 1 when done, 0 for an unsupported layout or pointer
   contract (nothing submitted). */
const char *k200_swiglu_reason(int width, int rows, int gate_stride, int up_stride, int output_stride, int type);
int k200_swiglu(void *kernel, int device, void *y, size_t y_bytes, const void *gate, size_t gate_bytes,
                const void *up, size_t up_bytes, int width, int rows, int gate_stride, int up_stride,
                int output_stride, int type);

/* ---- row-sharded batch-1 Q4_0 matmul with a fused all-gather over peer memory
 * Replaces the gather of a row split: the reference's consumers split output
 * rows over devices and move the slices with kunlun::peer copies
 * (src/k200.cpp:89-95; "Row Split", docs/common-q4.md:23,31).  Here the GEMV
 * of each rank stores its rows straight into every rank's memory over NVLink,
 * so no separate collective runs.  One process per GPU; every rank maps the
 * other ranks' tag arrays with k200_ipc_open.
 *
 * An exchange is, on every rank, an output buffer y of batch * rows floats
 * ([batch][rows]), a tag array of batch * rows 64-bit words and two counter
 * words, all zeroed before the first call.  Values travel as tagged words
 * {f32 bits in the low half, epoch in the high half}, each stored with one
 * single-copy-atomic 8-byte store into every rank's tag array; the epoch
 * counts this rank's launches on the exchange (the counter's second word).
 * A reader therefore needs no flag: it waits on the device until each word
 * it reads carries its own rank's current epoch.  k200_gather describes an
 * exchange from this rank: tags[r] is rank r's tag array as an address valid
 * on this device (own allocation or IPC mapping); y and counter are this
 * rank's own.  k200_matmul_q4_gather (batch 1) stores this rank's rows
 * [row_begin, row_begin + n) as tagged words on every rank and as plain
 * floats into this rank's y; k200_gather_wait then waits for every word of
 * the exchange and writes all batch * rows values into this rank's y.
 * wait_for (optional) names the exchange whose output is x (x must point
 * into wait_for's y): the GEMV reads x's tagged words, each as it arrives,
 * and x's elements past batch * rows (padding) plainly from y.  A wait that
 * runs out (several seconds) posts 0x4b03 to the device's error word
 * (k200_wait returns it) and the call completes without waiting further.
 * Calls on one exchange must be issued in the same order on every rank, on
 * one stream per rank.  A rank that reuses an exchange while another rank
 * may still read the previous contents races: alternate two exchanges (a
 * rank cannot run further ahead than one use, because its next reader waits
 * for every rank's words). */
#define K200_GATHER_MAX_RANKS 8
#define K200_GATHER_UNSUPPORTED (-4)
typedef struct {
    int ranks, rank;
    unsigned long long *tags[K200_GATHER_MAX_RANKS]; /* every rank's tag array */
    float *y;                                          /* this rank's output buffer */
    unsigned *counter;                                 /* this rank's two counter words */
    int rows;  /* rows of every rank's buffers: row_begin + n must not exceed it */
    int batch; /* columns: [batch][rows] values (1 for k200_matmul_q4_gather) */
} k200_gather;
/* IPC of a device allocation's base address (64-byte handles). */
int k200_ipc_handle(const void *device_ptr, void *handle);
int k200_ipc_open(int device, const void *handle, void **device_ptr);
int k200_ipc_close(int device, void *device_ptr);
/* Zeroed scratch the GEMV needs for a shard of n rows (0: shape not handled). */
size_t k200_matmul_q4_gather_scratch(int device, int k, int n);
/* Y rows [row_begin, row_begin + n) = W . x for this rank's n rows of Q4_0
 * weights W (batch 1, K % 256 == 0, 16-byte aligned W and x); scratch as
 * above, left zeroed.  0, K200_GATHER_UNSUPPORTED or a CUDA error code. */
int k200_matmul_q4_gather(int device, const k200_gather *out, int row_begin, const void *w, const void *x, int k,
                          int n, void *scratch, size_t scratch_bytes, const k200_gather *wait_for);
/* Waits for every tagged word of an exchange to carry this rank's current
 * epoch and writes the values into this rank's y (the end of a sequence, or
 * before the host reads y). */
int k200_gather_wait(int device, const k200_gather *exchange);
/* Row gather for any row-sharded matmul (any weight type and batch, any
 * split of the rows, uneven ones included): this rank's slice, [batch][n]
 * floats at `shard` (device memory, e.g. the y of a k200_matmul over this
 * rank's n weight rows), is stored as tagged words into columns
 * [row_begin, row_begin + n) of every rank's [batch][rows] tag array and as
 * plain floats into this rank's y; readers wait with k200_gather_wait (or
 * wait_for).  batch must equal the exchange's batch.  Asynchronous on the
 * library stream; 0 or a CUDA error code.  Replaces the reference
 * consumers' per-slice kunlun::peer copies of a row split
 * (src/k200.cpp:89-95, docs/common-q4.md "Row Split"). */
int k200_gather_rows(int device, const k200_gather *out, int row_begin, const float *shard, int n, int batch);

#ifdef __cplusplus
}
#endif
#endif
