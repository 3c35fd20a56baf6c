// Expert parallelism over NVLink peer memory: the device side of styx_ep.
//
// Every rank holds the slot rows of its own experts, weighted (w[s] * d[s][r];
// exactly 0 for another rank's slots).  A call sends each value as one
// 8-byte word -- the f32 bits in the low half, the call's generation (low
// 32 bits) in the high half -- with a relaxed system-scope store into row
// `rank` of every peer's inbox, in the half picked by the parity of the
// generation.  An aligned 8-byte store is single-copy atomic, so a receiver
// that reads its own word with a relaxed system-scope load and finds this
// call's generation there has the value as well: no fence, no flag and no
// counter on the path (the low-latency form of a tagged-word exchange).  It
// then sums, per column, the ranks then the slots, in slot order, into x.
// Each slot has one non-zero contributor, so the sum equals the
// single-device block bit for bit.
//
// The generation is this rank's count of completed calls + 1, read from its
// own memory after the grid dependency and advanced by the CTA that ends the
// call last, so a launch carries no per-call value and a recorded graph
// replays correctly.  A peer can be one call ahead (it writes the other
// half) but not two: its next words need this rank's words of the call it is
// in.  A word left from two calls back carries another generation.  Every
// wait is bounded; a wait that gives up sets the error word, and the
// thread's later waits of the call are skipped.  Nothing here loads another
// GPU's memory: peers are only stored to.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace styx {

__device__ __forceinline__ void ep_put(unsigned long long *p, unsigned tag, float v) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The value of word p once it carries `tag`; `live` false: a wait of this
// thread already gave up in this call (returns 0 without waiting).
__device__ __forceinline__ float ep_get(const unsigned long long *p, unsigned tag, bool &live, int *err) {
    unsigned long long w = ld_relaxed_sys(p);
    if (static_cast<unsigned>(w >> 32) != tag) {
        if (!live) return 0.f;
        const long long t0 = clock64();
        do {
            const long long dt = clock64() - t0;
            if (dt > kSpinCycles) {
                atomicExch(err, kErrWaitPeer);
                live = false;
                return 0.f;
            }
            if (dt > 100000) __nanosleep(256);
            w = ld_relaxed_sys(p);
        } while (static_cast<unsigned>(w >> 32) != tag);
    }
    return __uint_as_float(static_cast<unsigned>(w));
}

// the generation of the call in progress (after the grid dependency)
__device__ __forceinline__ unsigned long long ep_generation(const EpPeers &ep) {
    return __ldcg(ep.calls) + 1ull;
}

// After a __syncthreads that follows every read of the generation in the
// CTA: the CTA that ends the call last advances this rank's call counter.
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

// the inbox word of (sending rank p, slot s, column c) in the half of `gen`
__device__ __forceinline__ size_t ep_index(const EpPeers &ep, unsigned long long gen, int p, int s, int c) {
    const size_t row = static_cast<size_t>(ep.k) * ep.H;
    return (gen & 1ull) * static_cast<size_t>(ep.world) * row + static_cast<size_t>(p) * row +
           static_cast<size_t>(s) * ep.H + c;
}

}  // namespace styx
