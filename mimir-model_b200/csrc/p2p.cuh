// p2p.cuh -- exchanges between the ranks of a tensor-parallel group through
// peer memory (NVLink / NVSwitch), fused into the kernels that produce and
// consume the exchanged activations.
//
// Every rank's session arena is exported with CUDA IPC and mapped by every
// other rank, and the arenas share one layout, so buffer X of rank r lives
// at base[r] + (X - local base).  A producer kernel stores its slice into
// every rank's copy of the buffer and does nothing else; the consumer kernel
// that follows it on the same stream publishes -- its first thread writes the
// step's epoch into slot `slot`, entry `k` (this rank), of every rank's flag
// array after a system-scope fence, one fence per exchange -- and then waits
// until all N entries of the slot hold the epoch (bounded by the context's
// wait limit, then DEV_TIMEOUT in the status word and the kernel goes on with
// what it reads).  The epoch advances once per
// forward, so flags never need resetting.  A rank can be at most one
// exchange ahead of another (each exchange waits for every rank's previous
// one), which is what keeps a producer from overwriting a buffer a slower
// rank still reads.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Address of a rank's copy of a buffer at arena offset `off`.
template <class T>
__device__ __forceinline__ T *peer_ptr(const P2P &x, int r, long long off) {
    return (T *)(uintptr_t)(x.base[r] + (uint64_t)off);
}

// Writes this forward's epoch into entry k of the slot on every rank.  The
// data this rank produced for the slot was stored by the kernel that
// precedes the caller in stream order, which has completed by the caller's
// griddepcontrol.wait; the system-scope fence orders those stores before the
// flag for the other GPUs.
__device__ __forceinline__ void p2p_publish(const P2P &x) {
    __threadfence_system();
    const unsigned e = *(volatile const unsigned *)x.epoch;
    for (int r = 0; r < x.N; r++) st_release_sys(peer_ptr<unsigned>(x, r, x.off_flags) + x.slot * x.N + x.k, e);
}

// Consumer side of an exchange, called by every block after
// griddepcontrol.wait: the grid's first thread publishes this rank's part
// (see p2p_publish), then each block's thread 0 waits until every rank has
// published the slot for this forward; the block synchronises afterwards.
__device__ __forceinline__ void p2p_publish_wait(const P2P &x) {
    if (threadIdx.x != 0) return;
    if (blockIdx.x == 0 && blockIdx.y == 0) p2p_publish(x);
    const unsigned e = *(volatile const unsigned *)x.epoch;
    const unsigned *f = peer_ptr<unsigned>(x, x.k, x.off_flags) + x.slot * x.N;
    const uint64_t t0 = global_ns(), limit = dev_wait_limit(x.status);
    // relaxed polls of the (local) flag words, one acquire fence once all match
    for (int r = 0; r < x.N; r++) {
        for (uint32_t i = 0;; i++) {
            if (*(volatile const unsigned *)(f + r) == e) break;
            if ((i & 63) == 63 && global_ns() - t0 > limit) {
                atomicOr(x.status, (unsigned)DEV_TIMEOUT);
                return;
            }
        }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace mimgpu
