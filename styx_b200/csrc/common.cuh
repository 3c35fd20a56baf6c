// common.cuh -- shared device helpers for the styx B200 MoE kernels.
//
// * PTX wrappers for mbarriers and 1-D bulk copies (cp.async.bulk, the TMA
//   engine's non-tensor form) used to stage expert slabs into shared memory.
// * Bounded waits: every spin on an mbarrier gives up after ~1 s of device
//   clock, sets the context's device error word and lets the kernel finish.
// * dp4a wrappers and the "digit" decomposition of activations used by the
//   quantised dot products (see qdot.cuh).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/styx_moe.h"

namespace styx {

constexpr uint32_t kSkip = 0xFFFFFFFFu;
constexpr int kIdsPerLayer = STYX_IDS_PER_LAYER;

// device error codes written to the error word
enum : int {
    kErrNone = 0,
    kErrWaitFull = 1,    // consumer gave up waiting for a bulk copy
    kErrWaitEmpty = 2,   // producer gave up waiting for a free stage
    kErrWaitRoute = 3,   // route: last-block handoff failed
    kErrBadId = 4,       // an expert id / hot index / arena slot out of range
    kErrBadPos = 5,      // a token position outside the KV caches
    kErrWaitPeer = 6,    // expert parallelism: a peer rank's rows of the call did not arrive
};

// ~1 s at the B200's 1.9 GHz SM clock
constexpr long long kSpinCycles = 2000000000LL;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// before a barrier's memory is initialised again (no phase or copy pending)
__device__ __forceinline__ void mbar_inval(uint64_t *bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// The same test, but a thread whose phase is not complete may be suspended
// (leaving its issue slots to the other warps) until the phase completes or
// about kSuspendNs have passed (0: plain polling, no suspension).
#ifndef STYX_MBAR_SUSPEND_NS
#define STYX_MBAR_SUSPEND_NS 20000
#endif
constexpr uint32_t kSuspendNs = STYX_MBAR_SUSPEND_NS;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in
// the error word) if the phase did not complete within kSpinCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (true) {
        if (kSuspendNs ? mbar_try_wait_suspend(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > kSpinCycles) {
            if (err) atomicExch(err, code);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// L2 eviction policies for bulk copies: expert slabs are read once per token
// (evict first), so that small tensors read every token (router rows, norms,
// id tables) stay resident (evict last).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// bulk_g2s with an L2 eviction policy
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

// Programmatic dependent launch (sm_90+): wait for the previous grid's
// memory, and allow the next grid to be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Warm L2 with [src, src + bytes) (no data comes back to the SM, so it is safe
// before the grid dependency resolves).  src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// the same with an L2 eviction policy
__device__ __forceinline__ void prefetch_l2_hint(const void *src, uint32_t bytes, uint64_t pol) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---------------------------------------------------------------- dp4a
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    return static_cast<int>(__dp4a(a, b, static_cast<unsigned>(c)));
}
// signed a (s8 lanes) x unsigned b (u8 lanes)
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
// unsigned a (u8 lanes) x signed b (s8 lanes)
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// byte i (0..3, i a run-time value) of w as an exact float, without I2F:
// the byte becomes the low mantissa byte of 2^23, then 2^23 is subtracted
__device__ __forceinline__ float byte_to_f(uint32_t w, uint32_t i) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | i)) - 8388608.f;
}

// ------------------------------------------------ unaligned smem loads
// 16 bytes from any 1-byte aligned address (shared or global): the aligned
// words that cover the range and a funnel shift.  Touches no byte outside
// the 4-byte words that hold [p, p+16).
__device__ __forceinline__ uint4 lds16_unaligned(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3];
    const uint32_t w4 = sh ? w[4] : 0u;
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh),
                      __funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh));
}
__device__ __forceinline__ uint2 lds8_unaligned(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3) * 8u;
    const uint32_t w0 = w[0], w1 = w[1];
    const uint32_t w2 = sh ? w[2] : 0u;
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// ------------------------------------------------------ digit vectors
// An activation vector v (length n, n % 32 == 0) is carried to the quantised
// dot products as three byte planes and a power-of-two scale per 32-element
// group g:
//   v[i] ~= s_g * (D1[i] + D2[i]/256 + D3[i]/65536)
// D1 = floor(v/s) in [-64, 63] (s8), D2 = floor(256*frac) in [0,255] (u8),
// D3 = round(256*frac') in [0,255] (u8).  s_g = 2^(e-5) for 2^e <= max|v_g|.
// The representation error is below s_g * 2^-16 <= max|v_g| * 2^-21, so a
// dot product against integer weight codes is exact to ~f32 precision while
// the inner loop runs on dp4a.
struct DigitsView {
    int8_t *d1;
    uint8_t *d2;
    uint8_t *d3;
    float *scale;   // n/32 group scales
};

// power-of-two group scale s for group max |v| = a, and 1/s (both exact)
__device__ __forceinline__ float digits_scale(float a, float &inv) {
    int se = 127;   // s = 1
    if (a > 0.f && a < INFINITY) {
        se = ((__float_as_uint(a) >> 23) & 0xFF) - 5;   // s = 2^(E-5)
        if (se < 1) se = 1;
    }
    inv = __uint_as_float(static_cast<uint32_t>(254 - se) << 23);
    return __uint_as_float(static_cast<uint32_t>(se) << 23);
}

// the three digits of one element (q = v * (1/s), exact for a power-of-two s).
// floor and round-to-nearest-even of values below 2^22 in magnitude come from
// one add of 1.5 * 2^23 with the matching rounding mode: the sum's unit is 1,
// so its low mantissa bits are the integer (no float-to-int conversion).
__device__ __forceinline__ void digits_of(float v, float inv, int &d1, int &d2, int &d3) {
    constexpr float kM = 12582912.0f;      // 1.5 * 2^23
    constexpr int kMi = 0x4B400000;        // its bit pattern
    const float q = v * inv;               // |q| < 64
    const float t1 = __fadd_rd(q, kM);     // kM + floor(q)
    const float f1 = t1 - kM;
    const float r1 = (q - f1) * 256.f;     // exact, in [0, 256)
    const float t2 = __fadd_rd(r1, kM);
    const float f2 = t2 - kM;
    const float r2 = (r1 - f2) * 256.f;    // in [0, 256)
    const float t3 = __fadd_rn(r2, kM);    // kM + rint(r2), ties to even
    d1 = __float_as_int(t1) - kMi;
    d2 = __float_as_int(t2) - kMi;
    d3 = min(__float_as_int(t3) - kMi, 255);
}

// one 32-element group, one element per lane of a full warp
__device__ __forceinline__ void digits_group_warp(float v, int lane, const DigitsView &dv, int g) {
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    float inv;
    const float s = digits_scale(a, inv);
    int d1, d2, d3;
    digits_of(v, inv, d1, d2, d3);
    const int i = g * 32 + lane;
    dv.d1[i] = static_cast<int8_t>(d1);
    dv.d2[i] = static_cast<uint8_t>(d2);
    dv.d3[i] = static_cast<uint8_t>(d3);
    // every lane stores the (same) scale: a lane-0 branch here would leave the
    // warp split, and each shuffle of the next group would pay for regrouping
    // it (~10x its cost on B200)
    dv.scale[g] = s;
}

// N independent 32-element groups at once, one element of each per lane,
// group j at index gidx[j] (< 0: skipped): the same digits as N calls of
// digits_group_warp, but the N shuffle chains of the group maxima run in
// lockstep, so their latencies overlap instead of adding up.
template <int N>
__device__ __forceinline__ void digits_groups_warp(const float (&v)[N], const int (&gidx)[N], int lane,
                                                   const DigitsView &dv) {
    float a[N];
#pragma unroll
    for (int j = 0; j < N; j++) a[j] = fabsf(v[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int j = 0; j < N; j++) a[j] = fmaxf(a[j], __shfl_xor_sync(0xffffffffu, a[j], o));
#pragma unroll
    for (int j = 0; j < N; j++) {
        if (gidx[j] < 0) continue;
        float inv;
        const float s = digits_scale(a[j], inv);
        int d1, d2, d3;
        digits_of(v[j], inv, d1, d2, d3);
        const int i = gidx[j] * 32 + lane;
        dv.d1[i] = static_cast<int8_t>(d1);
        dv.d2[i] = static_cast<uint8_t>(d2);
        dv.d3[i] = static_cast<uint8_t>(d3);
        dv.scale[gidx[j]] = s;
    }
}

// Digits of a whole vector v[n] (n % 32 == 0) by a group of `nthreads`
// threads (a multiple of 32, all of them calling): EPT elements per thread
// (8 or 16), 32/EPT threads per 32-element group sharing the group max by
// shuffles; same digits as digits_group_warp.  GLOBAL: v is read through L2
// (__ldcg), else v is shared memory.
// Digits of part pidx (elements pidx*EPT ..) of a vector whose values this
// thread holds in x; the 32/EPT threads of a group are adjacent lanes and
// all call together (on = false for padding parts).
template <int EPT>
__device__ __forceinline__ void digits_part(const float (&x)[EPT], bool on, int pidx, int8_t *pd1, uint8_t *pd2,
                                            uint8_t *pd3, float *scale) {
    static_assert(EPT == 8 || EPT == 16, "8 or 16 elements per thread");
    constexpr int TPG = 32 / EPT;                                // threads per group
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; i++) a = fmaxf(a, fabsf(x[i]));
#pragma unroll
    for (int o = 1; o < TPG; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    float inv;
    const float s = digits_scale(a, inv);
    uint32_t w1[EPT / 4], w2[EPT / 4], w3[EPT / 4];
#pragma unroll
    for (int i = 0; i < EPT / 4; i++) {
        uint32_t a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int d1, d2, d3;
            digits_of(x[4 * i + j], inv, d1, d2, d3);
            a1 |= (static_cast<uint32_t>(d1) & 0xFFu) << (8 * j);
            a2 |= static_cast<uint32_t>(d2) << (8 * j);
            a3 |= static_cast<uint32_t>(d3) << (8 * j);
        }
        w1[i] = a1;
        w2[i] = a2;
        w3[i] = a3;
    }
    if (on) {
        const size_t o = static_cast<size_t>(pidx) * EPT;
        if constexpr (EPT == 16) {
            *reinterpret_cast<uint4 *>(pd1 + o) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
            *reinterpret_cast<uint4 *>(pd2 + o) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
            *reinterpret_cast<uint4 *>(pd3 + o) = make_uint4(w3[0], w3[1], w3[2], w3[3]);
        } else {
            *reinterpret_cast<uint2 *>(pd1 + o) = make_uint2(w1[0], w1[1]);
            *reinterpret_cast<uint2 *>(pd2 + o) = make_uint2(w2[0], w2[1]);
            *reinterpret_cast<uint2 *>(pd3 + o) = make_uint2(w3[0], w3[1]);
        }
        scale[pidx / TPG] = s;   // the group's threads store the same value (no branch)
    }
}

template <int EPT, bool GLOBAL>
__device__ __forceinline__ void digits_vector(const float *v, int n, int8_t *pd1, uint8_t *pd2, uint8_t *pd3,
                                              float *scale, int t, int nthreads) {
    const int nparts = n / EPT;
    const int lim = ((nparts + 31) >> 5) << 5;                   // every lane of a warp iterates alike
    for (int pidx = t; pidx < lim; pidx += nthreads) {
        const bool on = pidx < nparts;
        float x[EPT];
#pragma unroll
        for (int i = 0; i < EPT / 4; i++) {
            const float4 *src = reinterpret_cast<const float4 *>(v + static_cast<size_t>(pidx) * EPT) + i;
            const float4 q = on ? (GLOBAL ? __ldcg(src) : *src) : make_float4(0.f, 0.f, 0.f, 0.f);
            x[4 * i] = q.x;
            x[4 * i + 1] = q.y;
            x[4 * i + 2] = q.z;
            x[4 * i + 3] = q.w;
        }
        digits_part<EPT>(x, on, pidx, pd1, pd2, pd3, scale);
    }
}

}  // namespace styx
