// Epoch flags of an all-gather exchange over peer memory (k200_gather):
// every rank has a flag array with one word per rank, written by the other
// GPUs, and a private {arrivals, epoch} counter.  A launch that stored its
// rows into every rank's buffer publishes the exchange's next epoch in slot
// `rank` of every rank's array once all of its blocks are done; a launch that
// reads gathered rows first waits until every slot of its own array has
// reached its own epoch.  Used by the batch-1 Q4_0 GEMV with the fused
// gather (gemv_q4_mma.cu) and by the row gather (gather.cu).
#pragma once
#include <cstdint>

#include "device_common.cuh"
#include "k200_internal.h"

namespace k200 {

// Flags live in every rank's memory and are written by other GPUs:
// system-scope acquire loads and release stores.
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Polls of another rank's flag, with short sleeps (a flag that arrives is
// seen within a fraction of a microsecond): several seconds in all, because
// ranks are separate processes whose hosts can fall behind one another (a
// pause in one process) while the other rank's GPU already waits.
constexpr uint32_t kFlagBudget = 1u << 23;

// Waits until every rank's entry of this rank's flag array has reached this
// rank's own entry (epochs only grow; compared modulo 2^32).  Single thread;
// posts kErrPeerTimeout and stops waiting when the budget runs out.
__device__ __forceinline__ void wait_peer_flags(const unsigned *flags, int ranks, int rank, int *err) {
    const unsigned target = ld_acquire_sys(flags + rank);
    for (int r = 0; r < ranks; ++r) {
        if (r == rank) continue;
        for (uint32_t spin = 0; static_cast<int>(ld_acquire_sys(flags + r) - target) < 0; ++spin) {
            if (spin >= kFlagBudget) {
                atomicExch(err, kErrPeerTimeout);
                break;
            }
            __nanosleep(200);
        }
    }
}

// Called by one thread of every block of a launch after the block's stores
// (ordered before it by a block barrier).  Each block releases its stores at
// GPU scope and counts itself in (a relaxed device-scope atomic after an
// acq_rel fence); the block that arrives last has thereby synchronised with
// every other block, so one system-scope acq_rel fence in it orders all of
// the launch's stores (fences are cumulative) before the flag stores that
// follow, which need no release semantics of their own.  It resets the
// count, raises the exchange's epoch and stores it into slot `rank` of every
// rank's flag array.  System-scope fences are the expensive part (each waits
// microseconds for NVLink): one per launch instead of one per block, and none
// per flag store, halves the publish phase of a sharded GEMV.
__device__ __forceinline__ void publish_epoch(const GatherLaunch &xg, int blocks) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    const unsigned arrived = atomicAdd(xg.counter, 1u) + 1u;
    if (arrived == static_cast<unsigned>(blocks)) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        xg.counter[0] = 0u;  // the next launch's blocks arrive after this one completes
        const unsigned epoch = xg.counter[1] + 1u;
        xg.counter[1] = epoch;
        for (int r = 0; r < xg.ranks; ++r) st_relaxed_sys(xg.flags[r] + xg.rank, epoch);
    }
}

}  // namespace k200
