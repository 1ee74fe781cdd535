// Tagged words of an all-gather exchange over peer memory (k200_gather).
//
// Every value a rank contributes to an exchange travels as one 64-bit word
// {f32 bits (low half), epoch (high half)}, stored with a single relaxed
// system-scope store into every rank's tag array (its own, and the others'
// over NVLink through IPC mappings).  A 64-bit access is single-copy atomic,
// so a reader that sees the epoch it expects also sees that launch's value:
// no fence, flag or counter has to travel between GPUs, and a reader waits
// only for the words it reads (as they arrive) rather than for a whole
// launch.  This is the low-latency form of the gather that the reference's
// consumers do with kunlun::peer copies (src/k200.cpp:89-95).
//
// Epochs: every rank keeps a private {arrivals, epoch} counter per exchange.
// A launch that stores into the exchange tags its words with epoch + 1 (read
// after the previous kernel of its stream completed); each block counts itself
// in as soon as all of its threads have read the epoch, and the last one
// raises the counter's epoch (only kernels after this launch read it).  Every rank
// issues the same sequence of launches per exchange, so the ranks' epochs
// agree.  A reader expects its own rank's current epoch of the exchange.
// Tag arrays start zeroed (epoch 0: nothing published yet).
//
// Users: the batch-1 Q4_0 GEMV with the fused gather (gemv_q4_mma.cu), the
// row gather (gather.cu) and the wait that turns an exchange's tags into
// plain rows (gemv_q4_mma.cu, gather_wait_kernel).
#pragma once
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

// Polls of a tagged word, with short sleeps: several seconds in all, because
// ranks are separate processes whose hosts can fall behind one another (a
// pause in one process) while another rank's GPU already waits.  A thread
// also gives up early once another thread has posted the timeout.
constexpr uint32_t kTagBudget = 1u << 23;

__device__ __forceinline__ unsigned long long tag_word(float v, unsigned epoch) {
    return (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ unsigned tag_epoch(unsigned long long w) { return static_cast<unsigned>(w >> 32); }
__device__ __forceinline__ float tag_value(unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); }

__device__ __forceinline__ void st_tag(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tag(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// two adjacent words (16-byte aligned); each is single-copy atomic on its own
__device__ __forceinline__ void ld_tag2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// This rank's current epoch of an exchange (after the kernels of this stream
// that published it have completed).
__device__ __forceinline__ unsigned exchange_epoch(const unsigned *counter) {
    return *reinterpret_cast<const volatile unsigned *>(counter + 1);
}

// The value of word *p once it carries `epoch` (w: a first load of it).  A
// wait that runs out posts kErrPeerTimeout and returns the stale value.
__device__ __forceinline__ float await_tag(const unsigned long long *p, unsigned long long w, unsigned epoch,
                                           int *err) {
    for (uint32_t spin = 0; tag_epoch(w) != epoch; ++spin) {
        if (spin >= kTagBudget ||
            ((spin & 255u) == 255u && *reinterpret_cast<volatile int *>(err) == kErrPeerTimeout)) {
            atomicExch(err, kErrPeerTimeout);
            break;
        }
        __nanosleep(128);
        w = ld_tag(p);
    }
    return tag_value(w);
}

// A block of a launch that stores words of `epoch` counts itself in (one
// thread, after a barrier behind every thread's read of the epoch): the last
// block to arrive resets the arrivals and raises the exchange's epoch for the
// launches that follow on this stream (which read it only after this launch
// has completed).
__device__ __forceinline__ void count_launch(unsigned *counter, int blocks, unsigned epoch) {
    if (atomicAdd(counter, 1u) + 1u == static_cast<unsigned>(blocks)) {
        counter[0] = 0u;
        counter[1] = epoch;
    }
}

}  // namespace k200
