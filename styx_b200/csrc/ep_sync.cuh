// Expert parallelism over NVLink peer memory: the device side of styx_ep.
//
// Every rank holds the slot rows of its own experts, weighted (w[s] * d[s][r];
// exactly 0 for another rank's slots).  A call moves them with plain stores
// into row `rank` of every peer's inbox, in the half picked by the parity of
// the call's generation, and then adds, per CTA, the rows it pushed to the
// sender's counter in each peer (a release add at system scope after a
// system fence).  A receiver waits (bounded) until every peer's counter has
// reached gen * H -- every row of the call -- and sums, per column, the ranks
// then the slots, in slot order, into x.  Each slot has one non-zero
// contributor, so the sum equals the single-device block bit for bit.
//
// The generation is this rank's count of completed calls + 1, read from its
// own memory after the grid dependency and advanced by the CTA that ends the
// call last, so a launch carries no per-call value and a recorded graph
// replays correctly.  A peer can be one call ahead (it writes the other
// half) but not two: its next push needs this rank's push of the call it is
// in.  Counters only grow, and every add of a call precedes every add of the
// sender's next call (its kernels are stream-ordered), so a counter at
// gen * H or above means every row of call gen has landed.
// Nothing here loads another GPU's memory: peers are only stored to.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace styx {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_add_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// the generation of the call in progress (after the grid dependency)
__device__ __forceinline__ unsigned long long ep_generation(const EpPeers &ep) {
    return __ldcg(ep.calls) + 1ull;
}

// After the CTA's stores to the peers (and a __syncthreads): thread p (p !=
// rank, p < world) publishes the CTA's `rows` to peer p, then waits until
// peer p's counter here shows every row of call `gen`.  Returns false (and
// sets the error word) if a wait gave up.
__device__ __forceinline__ bool ep_signal_and_wait(const EpPeers &ep, unsigned long long gen, int rows, int *err) {
    const int t = threadIdx.x;
    bool fine = true;
    if (t < ep.world && t != ep.rank) {
        __threadfence_system();
        red_add_release_sys(ep.cnt[t] + ep.rank, static_cast<unsigned long long>(rows));
        const unsigned long long want = gen * static_cast<unsigned long long>(ep.H);
        const unsigned long long *c = ep.cnt[ep.rank] + t;
        const long long t0 = clock64();
        while (ld_acquire_sys(c) < want) {
            const long long dt = clock64() - t0;
            if (dt > kSpinCycles) {
                atomicExch(err, kErrWaitPeer);
                fine = false;
                break;
            }
            if (dt > 100000) __nanosleep(256);
        }
    }
    return fine;
}

// After every thread of the CTA has read the generation: the CTA that ends
// the call last advances this rank's call counter.
__device__ __forceinline__ void ep_call_done(const EpPeers &ep, unsigned long long gen, int ctas) {
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ep.done, 1u) == static_cast<unsigned>(ctas - 1)) {
            *ep.done = 0u;
            __threadfence();
            *ep.calls = gen;
            __threadfence();
        }
    }
}

// the inbox element of (sending rank p, slot s, column c) in the half of `gen`
__device__ __forceinline__ size_t ep_index(const EpPeers &ep, unsigned long long gen, int p, int s, int c) {
    const size_t row = static_cast<size_t>(ep.k) * ep.H;
    return (gen & 1ull) * static_cast<size_t>(ep.world) * row + static_cast<size_t>(p) * row +
           static_cast<size_t>(s) * ep.H + c;
}

}  // namespace styx
