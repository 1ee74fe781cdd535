// All-gather of a row-sharded matmul's output over peer memory
// (k200_gather_rows): this rank's slice Y[:, row_begin : row_begin + n] of a
// [batch][rows] output, computed into a local [batch][n] buffer by any
// matmul (any weight type, any batch), is stored into every rank's full
// output buffer (its own and, over NVLink, the others' through IPC
// mappings), then the exchange's next epoch is published in every rank's
// flag array (peer_flags.cuh).  Readers wait for the epoch on the device
// (k200_gather_wait, or the wait of k200_matmul_q4_gather).  Any split of the
// rows works, uneven ones included (8193 rows over 2 ranks: 4097 + 4096):
// every slice lands at its own offset, so nothing is padded or cropped.
//
// The reference has no multi-device matmul: its consumers split rows across
// devices and move the slices with kunlun::peer copies (src/k200.cpp:89-95,
// docs/common-q4.md "Row Split"); this is that exchange as one kernel.
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"
#include "peer_flags.cuh"

namespace k200 {

namespace {

// Grid-stride copy of the [batch][n] slice into every rank's [batch][rows]
// buffer (xg.y[r] already points at column row_begin), four columns at a
// time when the rows allow 16-byte stores, then the epoch.
__global__ void __launch_bounds__(256) gather_rows_kernel(const float *shard, int n, int batch, int rows,
                                                          const GatherLaunch xg, int vec4) {
    const long long total = static_cast<long long>(batch) * n;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    if (vec4) {
        const int nq = n >> 2, rq = rows >> 2;
        const long long quads = static_cast<long long>(batch) * nq;
        for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < quads; i += stride) {
            const long long b = i / nq, j = i - b * nq;
            const float4 v = reinterpret_cast<const float4 *>(shard)[i];
            for (int r = 0; r < xg.ranks; ++r) reinterpret_cast<float4 *>(xg.y[r])[b * rq + j] = v;
        }
    } else {
        for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
            const long long b = i / n, j = i - b * n;
            const float v = shard[i];
            for (int r = 0; r < xg.ranks; ++r) xg.y[r][b * rows + j] = v;
        }
    }
    __syncthreads();  // every store of the block before its arrival
    if (threadIdx.x == 0) publish_epoch(xg, gridDim.x);
}

}  // namespace

cudaError_t launch_gather_rows(const GatherLaunch &xg, const float *shard, int n, int batch, int rows,
                               const DeviceInfo &dev, cudaStream_t stream) {
    if (xg.ranks < 1 || n < 1 || batch < 1 || rows < n) return cudaErrorInvalidValue;
    bool vec4 = n % 4 == 0 && rows % 4 == 0 && (reinterpret_cast<uintptr_t>(shard) & 15) == 0;
    for (int r = 0; r < xg.ranks; ++r) vec4 = vec4 && (reinterpret_cast<uintptr_t>(xg.y[r]) & 15) == 0;
    const long long work = static_cast<long long>(batch) * n / (vec4 ? 4 : 1);
    const long long want = (work + 255) / 256;
    const int grid = static_cast<int>(want < dev.sm_count * 4LL ? (want < 1 ? 1 : want) : dev.sm_count * 4LL);
    gather_rows_kernel<<<grid, 256, 0, stream>>>(shard, n, batch, rows, xg, vec4 ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace k200
