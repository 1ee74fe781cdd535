// All-gather of a row-sharded matmul's output over peer memory
// (k200_gather_rows): this rank's slice Y[:, row_begin : row_begin + n] of a
// [batch][rows] output, computed into a local [batch][n] buffer by any
// matmul (any weight type, any batch), is stored as tagged words {f32,
// epoch} into every rank's [batch][rows] tag array of the exchange (its own,
// and over NVLink the others' through IPC mappings; exchange.cuh) and as
// plain values into this rank's own output.  Readers wait on the device for
// the words' epoch (k200_gather_wait, which also writes the plain rows, or
// the X of a k200_matmul_q4_gather).  Any split of the rows works, uneven
// ones included (8193 rows over 2 ranks: 4097 + 4096): every slice lands at
// its own offset, so nothing is padded or cropped.
//
// The reference has no multi-device matmul: its consumers split rows across
// devices and move the slices with kunlun::peer copies (src/k200.cpp:89-95,
// docs/common-q4.md "Row Split"); this is that exchange as one kernel.
#include <cstdint>

#include "device_common.cuh"
#include "exchange.cuh"
#include "k200_internal.h"

namespace k200 {

namespace {

// Grid-stride pass over the [batch][n] slice, two columns at a time (one
// 16-byte store of two tagged words per rank) when the offsets allow it,
// after the launch is counted in.
__global__ void __launch_bounds__(256) gather_rows_kernel(float *y, const float *shard, int n, int batch, int rows,
                                                          const __grid_constant__ GatherLaunch xg, int vec2) {
    pdl_wait_prior();  // the counter and the tags' previous contents belong to earlier kernels
    const unsigned epoch = exchange_epoch(xg.counter) + 1u;
    // every thread has read the epoch: the block counts in before its stores
    // (the last one raises the epoch, which only kernels after this launch read)
    __syncthreads();
    if (threadIdx.x == 0) count_launch(xg.counter, gridDim.x, epoch);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long first = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    if (vec2) {
        const int nh = n >> 1, rh = rows >> 1;
        const long long pairs = static_cast<long long>(batch) * nh;
        for (long long i = first; i < pairs; i += stride) {
            const long long b = i / nh, j = i - b * nh;
            const float2 v = reinterpret_cast<const float2 *>(shard)[i];
            reinterpret_cast<float2 *>(y)[b * rh + j] = v;
            const unsigned long long w0 = tag_word(v.x, epoch), w1 = tag_word(v.y, epoch);
            for (int r = 0; r < xg.ranks; ++r) {
                unsigned long long *t = xg.tags[r] + 2 * (b * rh + j);
                asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(t), "l"(w0), "l"(w1) : "memory");
            }
        }
    } else {
        const long long total = static_cast<long long>(batch) * n;
        for (long long i = first; i < total; i += stride) {
            const long long b = i / n, j = i - b * n;
            const float v = shard[i];
            y[b * rows + j] = v;
            const unsigned long long w = tag_word(v, epoch);
            for (int r = 0; r < xg.ranks; ++r) st_tag(xg.tags[r] + b * rows + j, w);
        }
    }
}

}  // namespace

cudaError_t launch_gather_rows(const GatherLaunch &xg, float *y, const float *shard, int n, int batch, int rows,
                               const DeviceInfo &dev, cudaStream_t stream) {
    if (xg.ranks < 1 || n < 1 || batch < 1 || rows < n || !y || !xg.counter) return cudaErrorInvalidValue;
    bool vec2 = n % 2 == 0 && rows % 2 == 0 && (reinterpret_cast<uintptr_t>(shard) & 7) == 0 &&
                (reinterpret_cast<uintptr_t>(y) & 7) == 0;
    for (int r = 0; r < xg.ranks; ++r) vec2 = vec2 && (reinterpret_cast<uintptr_t>(xg.tags[r]) & 15) == 0;
    const long long work = static_cast<long long>(batch) * n / (vec2 ? 2 : 1);
    const long long want = (work + 255) / 256;
    const int grid = static_cast<int>(want < dev.sm_count * 4LL ? (want < 1 ? 1 : want) : dev.sm_count * 4LL);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gather_rows_kernel, y, shard, n, batch, rows, xg, vec2 ? 1 : 0);
}

}  // namespace k200
