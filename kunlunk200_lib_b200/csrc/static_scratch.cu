// Fixed device scratch of the allocation-free rowwise-int8 matmul
// (k200_matmul_i8_noalloc).
//
// k200_matmul keeps the quantised activations of the rowwise-int8 path in a
// Kernel-owned buffer that it grows with cudaMalloc (and frees with cudaFree)
// when a larger batch*k arrives.  This array is the alternative for callers
// that cannot allocate at call time: it is sized at compile time, allocated
// by the driver when the module loads on a device, and shared by every call
// on that device.
//
// Layout (bytes): [0, 2*kNoAllocMaxElements) the two int8 activation
// components, q0 then q1, each batch*k long; at kNoAllocParamsOffset the
// 256-byte parameter block {max0, max1} (offset 0) and the three reduction
// words of the multi-CTA quantiser (offset 64).
#include "k200_internal.h"

namespace k200 {

static __device__ __align__(256) unsigned char noalloc_scratch[kNoAllocScratchBytes];

cudaError_t noalloc_scratch_address(void **ptr) { return cudaGetSymbolAddress(ptr, noalloc_scratch); }

}  // namespace k200
