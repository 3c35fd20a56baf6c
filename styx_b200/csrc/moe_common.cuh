// moe_common.cuh -- device helpers of the single-kernel MoE block
// (moe_fused.cu): tagged exchange words, slab sources, the warp-wide top-k
// selection, deterministic block sums, 16-byte covers.
#pragma once

#include <cfloat>

#include "common.cuh"
#include "kernels.h"

namespace styx {

// warps of a single-kernel MoE block CTA
constexpr int kFusedWarps = 16;
constexpr int kFusedBlock = 32 * kFusedWarps;

// ---- tagged exchange words {f32 value bits (low), u32 tag (high)}
// written with a 64-bit atomic exchange: performed at L2 at once, not held
// in the SM's store path behind other traffic
__device__ __forceinline__ void st_slot(uint64_t *p, float v, uint32_t tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    atomicExch(reinterpret_cast<unsigned long long *>(p), w);
}
__device__ __forceinline__ uint64_t ld_slot(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// two adjacent tagged words (16-byte aligned), each read whole
__device__ __forceinline__ void ld_slot2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t slot_tag(uint64_t w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ float slot_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

__device__ __forceinline__ const uint8_t *fused_slot_src(const ExpSrc &t, int hot, int arena, int full) {
    if (hot >= 0)
        return (t.hot && static_cast<uint32_t>(hot) < t.nhot) ? t.hot + static_cast<uint64_t>(hot) * t.slab : nullptr;
    if (arena >= 0)
        return (t.arena && static_cast<uint32_t>(arena) < t.narena) ? t.arena + static_cast<uint64_t>(arena) * t.aslab
                                                                     : nullptr;
    if (full >= 0)
        return (t.full && static_cast<uint32_t>(full) < t.nfull) ? t.full + static_cast<uint64_t>(full) * t.slab
                                                                  : nullptr;
    return nullptr;
}

// logits a lane of warp 0 holds: up to STYX_MAX_EXPERTS / 32
constexpr int kLogitRegs = STYX_MAX_EXPERTS / 32;

// Order-preserving key of a float that is > -inf (NaN excluded by the
// caller): larger float -> larger key, never 0; -0 is folded into +0, which
// the comparison treats as equal.
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

// Selection as topk_softmax_f32.comp:39-46: k times the largest untaken
// logit by strict '>', the lowest index among equals, never -inf or NaN.
// Lane l holds the keys of elements l + 32 j, j < NP (0 = not eligible); each
// pick is a warp max over keys, then a warp min over the indices holding
// that key.  A lane's candidates have increasing indices, so its first
// maximal register is its lowest such index.  Lane s < k receives pick s
// (e = -1, ke = 0 when fewer than k logits are eligible).
template <int NP>
__device__ __forceinline__ void warp_pick(uint32_t *key, int k, int lane, int &e, uint32_t &ke) {
    for (int s = 0; s < k; s++) {
        uint32_t bk = key[0];
        int bj = 0;
#pragma unroll
        for (int j = 1; j < NP; j++)
            if (key[j] > bk) {
                bk = key[j];
                bj = j;
            }
        const uint32_t K = __reduce_max_sync(0xffffffffu, bk);
        if (K == 0) break;   // the remaining slots stay empty
        const uint32_t mine = (bk == K) ? static_cast<uint32_t>(lane + 32 * bj) : 0xffffffffu;
        const uint32_t I = __reduce_min_sync(0xffffffffu, mine);
        if (mine == I) {
#pragma unroll
            for (int j = 0; j < NP; j++)
                if (j == bj) key[j] = 0u;
        }
        if (lane == s) {
            e = static_cast<int>(I);
            ke = K;
        }
    }
}

// The same selection for at most 4 keys per lane (E <= 128): each lane first
// orders its own (key, index) pairs, key descending and index ascending among
// equal keys, so its candidate for every pick is its head and a pick costs
// two reductions and a shift on the winning lane.
__device__ __forceinline__ void cx_desc(uint32_t &ka, int &ia, uint32_t &kb, int &ib) {
    if (kb > ka || (kb == ka && ib < ia)) {
        const uint32_t tk = ka;
        ka = kb;
        kb = tk;
        const int ti = ia;
        ia = ib;
        ib = ti;
    }
}
__device__ __forceinline__ void warp_pick_sorted4(const uint32_t *key, int k, int lane, int &e, uint32_t &ke) {
    uint32_t k0 = key[0], k1 = key[1], k2 = key[2], k3 = key[3];
    int i0 = lane, i1 = lane + 32, i2 = lane + 64, i3 = lane + 96;
    cx_desc(k0, i0, k1, i1);
    cx_desc(k2, i2, k3, i3);
    cx_desc(k0, i0, k2, i2);
    cx_desc(k1, i1, k3, i3);
    cx_desc(k1, i1, k2, i2);
    for (int s = 0; s < k; s++) {
        const uint32_t K = __reduce_max_sync(0xffffffffu, k0);
        if (K == 0) break;   // the remaining slots stay empty
        const uint32_t mine = k0 == K ? static_cast<uint32_t>(i0) : 0xffffffffu;
        const uint32_t I = __reduce_min_sync(0xffffffffu, mine);
        if (mine == I) {
            k0 = k1;
            i0 = i1;
            k1 = k2;
            i1 = i2;
            k2 = k3;
            i2 = i3;
            k3 = 0u;
        }
        if (lane == s) {
            e = static_cast<int>(I);
            ke = K;
        }
    }
}

// Cross-CTA polls spin without pausing for this long (a normal wait ends
// well within it), then pause between reads so that a wait that runs out
// does not load L2 for its whole second.
constexpr long long kPollFreeCycles = 100000;

// A 32-thread named barrier: regroups a warp whose lanes ran a divergent
// spin, so the full-warp shuffles and reductions that follow do not pay for
// reconverging them.
__device__ __forceinline__ void warp_converge(int id) { asm volatile("bar.sync %0, 32;" ::"r"(id) : "memory"); }

// two block-wide deterministic sums at once (fixed tree over the 16 warps)
__device__ __forceinline__ float2 fblock_sum2(float2 v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
        v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    __syncthreads();
    if (lane == 0) {
        red[warp] = v.x;
        red[kFusedWarps + warp] = v.y;
    }
    __syncthreads();
    float a = lane < kFusedWarps ? red[lane] : 0.f, c = lane < kFusedWarps ? red[kFusedWarps + lane] : 0.f;
#pragma unroll
    for (int o = 8; o; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    return make_float2(__shfl_sync(0xffffffffu, a, 0), __shfl_sync(0xffffffffu, c, 0));
}

// sum(r * w * x) over one float4, with one fixed sequence of roundings
__device__ __forceinline__ float rwx4(float4 r, float4 w, float4 x) {
    float a = __fmul_rn(__fmul_rn(r.x, w.x), x.x);
    a = __fmaf_rn(__fmul_rn(r.y, w.y), x.y, a);
    a = __fmaf_rn(__fmul_rn(r.z, w.z), x.z, a);
    return __fmaf_rn(__fmul_rn(r.w, w.w), x.w, a);
}

// block-wide deterministic sum (fixed tree over the 16 warps; the same tree
// as fblock_sum2's second component)
__device__ __forceinline__ float fblock_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < kFusedWarps ? red[lane] : 0.f;
#pragma unroll
    for (int o = 8; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return __shfl_sync(0xffffffffu, t, 0);
}

// 16-byte aligned cover of [p, p + n)
__device__ __forceinline__ void cover16(const uint8_t *p, size_t n, uintptr_t &a, uint32_t &len) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(p);
    a = s & ~uintptr_t(15);
    len = static_cast<uint32_t>(((s + n + 15) & ~uintptr_t(15)) - a);
}

}  // namespace styx
