// moe_fused.cu -- the whole MoE block of one layer as ONE cooperative kernel.
//
// Grid = one CTA per SM (cooperative launch: all CTAs co-resident), 16 warps.
// A CTA's share of the layer's expert bytes (its gate/up rows and its down
// rows for all k slots) fits in shared memory at the shapes this kernel is
// planned for (the host checks), so every bulk copy is issued up front and
// the whole layer streams from HBM at once.  Phases of CTA b of G:
//   0  thread 0 bulk-copies this CTA's router rows (e = b, b+G, ...) and
//      ffn_norm into shared memory (inputs that do not depend on x);
//   1  RMSNorm of x (every CTA, same fixed order -> identical x_norm), the
//      router dot products of its rows -> logits[e]; x_norm -> dp4a digits
//      in shared memory; arrive on counter 0;
//   2  wait for counter 0 == G (bounded), read all logits, softmax + top-k
//      (rank form of topk_softmax_f32.comp): every CTA computes the same ids;
//      CTA 0 publishes the id rows and the weights;
//   3  thread 0 issues the CTA's gate/up chunks and then its down chunks;
//      warps: gate/up dot products on dp4a, SiLU(g)*u -> h (global);
//      arrive on counter 1;
//   4  wait for counter 1 == G (all of h written); h -> digits in shared
//      memory; down dot products from the prefetched rows; slot-ordered
//      combine x[r] += sum_s w[s] d[s][r] (moe_reduce_f32.comp).
// The counters live in the workspace; the last CTA through a wait resets the
// counter before it, so the workspace is reusable by the next launch.
// Every wait is bounded (~1 s) and reports through the device error word.
#include <cfloat>

#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

namespace styx {

constexpr int kFusedWarps = 16;
constexpr int kFusedBlock = 32 * kFusedWarps;
// shared-memory header: 33 mbarriers, reduction scratch, weights, ids,
// flags, per-slot source pointers; region A starts at kFusedHeader
constexpr int kHdrRed = 512;
constexpr int kHdrSrc = 896;
constexpr int kFusedHeaderBytes = 1280;
static_assert(kHdrSrc + 3 * 16 * 8 <= kFusedHeaderBytes, "fused header overflow");
static_assert(kFusedHeaderBytes == static_cast<int>(kFusedHeader), "host and device header sizes differ");
static_assert(33 * 8 <= kHdrRed, "mbarriers overlap the reduction scratch");

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// bounded wait until *p >= target; false (and error code) on timeout
__device__ bool spin_geq(const unsigned *p, unsigned target, int *err, int code) {
    const long long t0 = clock64();
    while (ld_acquire(p) < target) {
        if (clock64() - t0 > kSpinCycles) {
            if (err) atomicExch(err, code);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

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

// block-wide deterministic sum / max (fixed tree over the 16 warps)
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
__device__ __forceinline__ float fblock_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < kFusedWarps ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 8; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    return __shfl_sync(0xffffffffu, t, 0);
}

// shared-memory bytes reserved for n rows of rb bytes (room for the cover)
__device__ __forceinline__ size_t chunk_bytes(int n, int rb) {
    return (static_cast<size_t>(n) * rb + 32 + 15) & ~size_t(15);
}

// 16-byte aligned cover of [p, p + n)
__device__ __forceinline__ void cover16(const uint8_t *p, size_t n, uintptr_t &a, uint32_t &len) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(p);
    a = s & ~uintptr_t(15);
    len = static_cast<uint32_t>(((s + n + 15) & ~uintptr_t(15)) - a);
}

template <int QG, int QD>
__global__ void __launch_bounds__(kFusedBlock, 1) k_moe_fused(const FusedArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    uint64_t *full_gu = bar, *full_d = bar + 16, *bar_router = bar + 32;
    float *red = reinterpret_cast<float *>(smem + kHdrRed);  // 32 floats
    float *wts = red + 32;                                    // 16 floats
    int *sel = reinterpret_cast<int *>(wts + 16);             // 16 ints
    int *s_flag = sel + 16;                                   // 16 ints
    const uint8_t **src_g = reinterpret_cast<const uint8_t **>(smem + kHdrSrc);   // 16 pointers each
    const uint8_t **src_u = src_g + 16;
    const uint8_t **src_d = src_u + 16;
    uint8_t *region_a = smem + p.off_a;                       // router rows, norm, xn, x digits
    float *rrows = reinterpret_cast<float *>(region_a);
    float *snorm = rrows + p.rrows_floats;
    float *xn = snorm + p.H;
    int8_t *xd1 = reinterpret_cast<int8_t *>(xn + p.H);
    uint8_t *xd2 = reinterpret_cast<uint8_t *>(xd1) + p.H;
    uint8_t *xd3 = xd2 + p.H;
    float *xsc = reinterpret_cast<float *>(xd3 + p.H);
    const int kF = p.k * p.F;                                 // phase 4: h digits in region A
    int8_t *hd1 = reinterpret_cast<int8_t *>(region_a);
    uint8_t *hd2 = reinterpret_cast<uint8_t *>(hd1) + kF;
    uint8_t *hd3 = hd2 + kF;
    float *hsc = reinterpret_cast<float *>(hd3 + kF);
    float *dpart = reinterpret_cast<float *>(smem + p.off_part);
    uint8_t *gubuf = smem + p.off_ring;
    uint8_t *dbuf = smem + p.off_down;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int H = p.H, F = p.F, k = p.k, E = p.E;
    const long long T = static_cast<long long>(k) * F;
    const int gbeg = static_cast<int>(T * b / G), gend = static_cast<int>(T * (b + 1) / G);
    const int dbeg = static_cast<int>(static_cast<long long>(H) * b / G);
    const int dend = static_cast<int>(static_cast<long long>(H) * (b + 1) / G);
    const int n_dchunks = (dend - dbeg + p.rc - 1) / p.rc;
    const int n_rows_mine = b < E ? (E - 1 - b) / G + 1 : 0;   // router rows e = b + G*j

#define STYX_STAMP(i_)                                                     \
    do {                                                                   \
        if (tid == 0 && p.trace) p.trace[b * 16 + (i_)] = clock64();        \
    } while (0)
    STYX_STAMP(0);
    // ------------------------------------------------ phase 0
    if (tid == 0) {
        for (int i = 0; i < 16; i++) {
            mbar_init(&full_gu[i], 1);
            mbar_init(&full_d[i], 1);
        }
        mbar_init(bar_router, 1);
        fence_mbar_init();
        const uint32_t rb = static_cast<uint32_t>(H) * 4u;
        mbar_arrive_expect_tx(bar_router, rb * static_cast<uint32_t>(n_rows_mine + 1));
        bulk_g2s(snorm, p.norm_w, rb, bar_router);
        for (int j = 0; j < n_rows_mine; j++)
            bulk_g2s(rrows + static_cast<size_t>(j) * H, p.router + static_cast<size_t>(b + G * j) * H, rb,
                     bar_router);
    }
    pdl_wait();

    // ------------------------------------------------ phase 1: RMSNorm + router
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    const int H4 = H >> 2;
    float ss = 0.f;
    for (int i = tid; i < H4; i += kFusedBlock) {
        const float4 v = __ldcg(x4 + i);
        reinterpret_cast<float4 *>(xn)[i] = v;   // raw x for now
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = fblock_sum(ss, red);   // (its barriers also publish the mbarrier inits)
    STYX_STAMP(1);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(H) + p.eps);
    const bool rok = mbar_wait(bar_router, 0, p.err, kErrWaitRoute);
    STYX_STAMP(2);
    for (int i = tid; i < H4; i += kFusedBlock) {
        float4 v = reinterpret_cast<float4 *>(xn)[i];
        const float4 w = rok ? reinterpret_cast<const float4 *>(snorm)[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        v.x = v.x * scale * w.x;
        v.y = v.y * scale * w.y;
        v.z = v.z * scale * w.z;
        v.w = v.w * scale * w.w;
        reinterpret_cast<float4 *>(xn)[i] = v;
    }
    __syncthreads();
    for (int j = 0; j < n_rows_mine; j++) {
        float acc = 0.f;
        const float4 *r4 = reinterpret_cast<const float4 *>(rrows + static_cast<size_t>(j) * H);
        for (int i = tid; i < H4; i += kFusedBlock) {
            const float4 r = r4[i], v = reinterpret_cast<const float4 *>(xn)[i];
            acc += r.x * v.x + r.y * v.y + r.z * v.z + r.w * v.w;
        }
        acc = fblock_sum(acc, red);
        if (tid == 0) __stcg(p.logits + b + G * j, acc);
    }
    {   // x_norm digits (every CTA keeps its own copy for the gate/up dots)
        const DigitsView dv{xd1, xd2, xd3, xsc};
        for (int g = warp; g < (H >> 5); g += kFusedWarps) digits_group_warp(xn[g * 32 + lane], lane, dv, g);
    }
    if (b == 0)   // test / debug view of x_norm
        for (int i = tid; i < H; i += kFusedBlock) p.xnorm[i] = xn[i];
    __threadfence();
    __syncthreads();
    STYX_STAMP(3);
    if (tid == 0) {
        atomicAdd(p.counters + 0, 1u);
        s_flag[0] = spin_geq(p.counters + 0, static_cast<unsigned>(G), p.err, kErrWaitRoute) ? 1 : 0;
    }
    STYX_STAMP(4);
    __syncthreads();

    // ------------------------------------------------ phase 2: top-k
    float *lg = rrows;   // router rows are consumed; the logits go here
    for (int i = tid; i < E; i += kFusedBlock) lg[i] = __ldcg(p.logits + i);
    __syncthreads();
    STYX_STAMP(5);
    {
        float m = -INFINITY;
        for (int i = tid; i < E; i += kFusedBlock) m = fmaxf(m, lg[i]);
        const float mx = fblock_max(m, red);
        float se = 0.f;
        for (int i = tid; i < E; i += kFusedBlock) se += expf(lg[i] - mx);
        const float sum = fblock_sum(se, red);
        STYX_STAMP(6);
        if (tid < 16) sel[tid] = -1;
        __syncthreads();
        // rank of every finite logit (strict '>' first, equal values ordered
        // by index): the serial scan's s-th pick is the element of rank s
        for (int i = tid; i < E; i += kFusedBlock) {
            const float v = lg[i];
            if (v > -INFINITY) {
                int gt = 0, eq = 0;
                const float4 *l4 = reinterpret_cast<const float4 *>(lg);
                const int E4 = E >> 2;
#pragma unroll 4
                for (int j4 = 0; j4 < E4; j4++) {
                    const float4 u = l4[j4];
                    const int j = 4 * j4;
                    gt += (u.x > v) + (u.y > v) + (u.z > v) + (u.w > v);
                    eq += ((u.x == v) & (j < i)) + ((u.y == v) & (j + 1 < i)) + ((u.z == v) & (j + 2 < i)) +
                          ((u.w == v) & (j + 3 < i));
                }
                for (int j = E4 * 4; j < E; j++) {
                    const float u = lg[j];
                    gt += u > v;
                    eq += (u == v) & (j < i);
                }
                if (gt + eq < k) sel[gt + eq] = i;
            }
        }
        __syncthreads();
        STYX_STAMP(7);
        if (warp == 0) {
            // lane s < k: slot s's weight, id rows and slab sources
            const int s = lane;
            float w = 0.f;
            int e = -1;
            if (s < k) {
                e = sel[s];
                const float best = e >= 0 ? lg[e] : -INFINITY;
                w = expf(best - mx) / sum;
            }
            float wsum = 0.f;   // slot order, as topk_softmax_f32.comp:50
            for (int t = 0; t < k; t++) wsum += __shfl_sync(0xffffffffu, w, t);
            if (s < k) {
                const float wr = p.renorm ? w / wsum : w;
                wts[s] = wr;
                const uint32_t hot = (e >= 0 && p.remap) ? p.remap[e] : kSkip;
                int hi = -1, ai = -1, fi = -1;
                if (hot != kSkip) {
                    hi = static_cast<int>(hot);
                } else {
                    const uint32_t a = (e >= 0 && p.pmap) ? p.pmap[e] : kSkip;
                    if (a != kSkip) ai = static_cast<int>(a);
                    else fi = e;
                }
                src_g[s] = fused_slot_src(p.gate, hi, ai, fi);
                src_u[s] = fused_slot_src(p.up, hi, ai, fi);
                src_d[s] = fused_slot_src(p.down, hi, ai, fi);
                if (b == 0) {
                    if (e >= 0 && (!src_g[s] || !src_u[s] || !src_d[s])) atomicExch(p.err, kErrBadId);
                    p.weights[s] = wr;
                    p.ids64[s] = e;
                    p.ids64[16 + s] = hi;
                    p.ids64[32 + s] = ai;
                    p.ids64[48 + s] = fi;
                }
            }
            __syncwarp();
            // ---- issue every expert byte this CTA needs, one lane per copy:
            // gate/up chunks (lane ci), packed back to back (gate rows, then
            // up rows, each with room for the 16-byte cover) ...
            int ci = 0;
            size_t off = 0;
            for (int r = gbeg; r < gend; ci++) {
                const int sl = r / F, rr = r - sl * F;
                const int n = min(p.ch, min(gend - r, F - rr));
                const size_t up_off = chunk_bytes(n, p.rb_g);
                if (ci == lane) {
                    uint8_t *dst = gubuf + off;
                    if (src_g[sl] && src_u[sl]) {
                        uintptr_t ga, ua;
                        uint32_t gl, ul;
                        cover16(src_g[sl] + static_cast<size_t>(rr) * p.rb_g, static_cast<size_t>(n) * p.rb_g, ga, gl);
                        cover16(src_u[sl] + static_cast<size_t>(rr) * p.rb_u, static_cast<size_t>(n) * p.rb_u, ua, ul);
                        mbar_arrive_expect_tx(&full_gu[ci], gl + ul);
                        bulk_g2s(dst, reinterpret_cast<const void *>(ga), gl, &full_gu[ci]);
                        bulk_g2s(dst + up_off, reinterpret_cast<const void *>(ua), ul, &full_gu[ci]);
                    } else {
                        mbar_arrive(&full_gu[ci]);
                    }
                }
                off += up_off + chunk_bytes(n, p.rb_u);
                r += n;
            }
            // ... then the down rows of every slot (lane s)
            for (int c = 0; c < n_dchunks; c++) {
                const int r0 = dbeg + c * p.rc, n = min(p.rc, dend - r0);
                uintptr_t a = 0;
                uint32_t len = 0;
                if (s < k && src_d[s])
                    cover16(src_d[s] + static_cast<size_t>(r0) * p.rb_d, static_cast<size_t>(n) * p.rb_d, a, len);
                uint32_t total = len;
#pragma unroll
                for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                if (lane == 0) {
                    if (total == 0) mbar_arrive(&full_d[c]);
                    else mbar_arrive_expect_tx(&full_d[c], total);
                }
                __syncwarp();
                if (len)
                    bulk_g2s(dbuf + static_cast<size_t>(c) * p.dstage_bytes + static_cast<size_t>(s) * p.dslot_stride,
                             reinterpret_cast<const void *>(a), len, &full_d[c]);
            }
        }
        __syncthreads();
    }

    STYX_STAMP(8);
    // ------------------------------------------------ phase 3: gate/up + SiLU
    {
        const int units = p.units_g, gs = p.gs_g, rpw = 32 / gs;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        XUnit x;
        if (active) load_xunit<QG>(x, xd1, xd2, xd3, xsc, ug);
        bool ok = true;
        int ci = 0;
        size_t off = 0;
        for (int r = gbeg; r < gend; ci++) {
            const int s = r / F, rr = r - s * F;
            const int n = min(p.ch, min(gend - r, F - rr));
            if (ok) ok = mbar_wait(&full_gu[ci], 0, p.err, kErrWaitFull);
            if (ci == 0) STYX_STAMP(9);
            const uint8_t *gsrc = src_g[s], *usrc = src_u[s];
            const bool valid = ok && gsrc && usrc;
            const uint8_t *base = gubuf + off;
            const size_t up_off = chunk_bytes(n, p.rb_g);
            off += up_off + chunk_bytes(n, p.rb_u);
            const uint8_t *gb =
                base + (valid ? (reinterpret_cast<uintptr_t>(gsrc + static_cast<size_t>(rr) * p.rb_g) & 15) : 0);
            const uint8_t *ub = base + up_off +
                                (valid ? (reinterpret_cast<uintptr_t>(usrc + static_cast<size_t>(rr) * p.rb_u) & 15) : 0);
            for (int t = warp * rpw; t < n; t += kFusedWarps * rpw) {
                const int row = t + grp;
                float g = 0.f, u = 0.f;
                if (valid && active && row < n) {
                    g = unit_dot<QG>(gb + static_cast<size_t>(row) * p.rb_g, ug, x);
                    u = unit_dot<QG>(ub + static_cast<size_t>(row) * p.rb_u, ug, x);
                }
                for (int o = gs >> 1; o; o >>= 1) {
                    g += __shfl_xor_sync(0xffffffffu, g, o);
                    u += __shfl_xor_sync(0xffffffffu, u, o);
                }
                // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
                if (ug == 0 && row < n) __stcg(p.h + static_cast<size_t>(s) * F + rr + row, g / (1.0f + expf(-g)) * u);
            }
            r += n;
        }
    }
    __threadfence();
    __syncthreads();
    STYX_STAMP(10);
    if (tid == 0) {
        const unsigned prev = atomicAdd(p.counters + 1, 1u);
        // every CTA has passed the phase-1 wait once counter 1 is complete
        if (prev == static_cast<unsigned>(G) - 1) atomicExch(p.counters + 0, 0u);
        s_flag[1] = spin_geq(p.counters + 1, static_cast<unsigned>(G), p.err, kErrWaitRoute) ? 1 : 0;
        const unsigned prev2 = atomicAdd(p.counters + 2, 1u);
        if (prev2 == static_cast<unsigned>(G) - 1) {
            atomicExch(p.counters + 1, 0u);
            atomicExch(p.counters + 2, 0u);
        }
    }
    __syncthreads();
    STYX_STAMP(11);

    // ------------------------------------------------ phase 4: down + combine
    // h -> digits: two threads per 32-element group, all loads in flight
    digits_vector<8, true>(p.h, kF, hd1, hd2, hd3, hsc, tid, kFusedBlock);
    __syncthreads();
    STYX_STAMP(12);
    {
        const int units = p.units_d, gs = p.gs_d, rpw = 32 / gs;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        const bool multi = k > kFusedWarps;
        const int nwps = multi ? 1 : kFusedWarps / k;
        const int slot0 = multi ? warp : warp / nwps;
        const int sub = multi ? 0 : warp % nwps;
        const int sstep = multi ? kFusedWarps : 1 << 30;
        XUnit x;
        if (!multi && slot0 < k && active)
            load_xunit<QD>(x, hd1 + slot0 * F, hd2 + slot0 * F, hd3 + slot0 * F, hsc + slot0 * (F >> 5), ug);
        bool ok = s_flag[1] != 0;
        for (int c = 0; c < n_dchunks; c++) {
            const int r0 = dbeg + c * p.rc, n = min(p.rc, dend - r0);
            if (ok) ok = mbar_wait(&full_d[c], 0, p.err, kErrWaitFull);
            if (c == 0) STYX_STAMP(13);
            float *part = dpart + static_cast<size_t>(c & 1) * k * p.rc;
            for (int s = slot0; ok && s < k; s += sstep) {
                if (multi && active)
                    load_xunit<QD>(x, hd1 + s * F, hd2 + s * F, hd3 + s * F, hsc + s * (F >> 5), ug);
                const uint8_t *src = src_d[s];
                const uint8_t *base = dbuf + static_cast<size_t>(c) * p.dstage_bytes +
                                      static_cast<size_t>(s) * p.dslot_stride +
                                      (src ? (reinterpret_cast<uintptr_t>(src + static_cast<size_t>(r0) * p.rb_d) & 15) : 0);
                for (int t = sub * rpw; t < n; t += nwps * rpw) {
                    const int row = t + grp;
                    float v = 0.f;
                    if (src && active && row < n) v = unit_dot<QD>(base + static_cast<size_t>(row) * p.rb_d, ug, x);
                    for (int o = gs >> 1; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (ug == 0 && row < n) part[s * p.rc + row] = v;
                }
            }
            __syncthreads();
            STYX_STAMP(14);
            if (ok && tid < n) {
                float acc = 0.f;
                for (int s = 0; s < k; s++) acc = __fadd_rn(acc, __fmul_rn(wts[s], part[s * p.rc + tid]));
                p.x[r0 + tid] = __fadd_rn(p.x[r0 + tid], acc);
            }
        }
    }
    STYX_STAMP(15);
#undef STYX_STAMP
}

template <int QG, int QD>
static cudaError_t launch_fused_t(const FusedArgs &a, int grid, uint32_t smem, cudaStream_t st) {
    auto kern = k_moe_fused<QG, QD>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kFusedBlock, smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (occ < 1 || grid > occ * sms) return cudaErrorCooperativeLaunchTooLarge;
    void *args[] = {const_cast<FusedArgs *>(&a)};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(kern), dim3(grid), dim3(kFusedBlock), args,
                                       smem, st);
}

cudaError_t launch_fused(const FusedArgs &a, int qg, int qd, int grid, uint32_t smem, cudaStream_t st) {
#define STYX_FUSED_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return launch_fused_t<G_, D_>(a, grid, smem, st);
    STYX_FUSED_CASE(STYX_Q4_K, STYX_Q6_K)
    STYX_FUSED_CASE(STYX_Q4_K, STYX_Q4_K)
    STYX_FUSED_CASE(STYX_Q5_K, STYX_Q6_K)
    STYX_FUSED_CASE(STYX_Q5_K, STYX_Q5_K)
    STYX_FUSED_CASE(STYX_Q8_0, STYX_Q8_0)
    STYX_FUSED_CASE(STYX_Q6_K, STYX_Q6_K)
#undef STYX_FUSED_CASE
    return cudaErrorNotSupported;
}

bool fused_supported(int qg, int qd) {
    return (qg == STYX_Q4_K && (qd == STYX_Q6_K || qd == STYX_Q4_K)) ||
           (qg == STYX_Q5_K && (qd == STYX_Q6_K || qd == STYX_Q5_K)) || (qg == STYX_Q8_0 && qd == STYX_Q8_0) ||
           (qg == STYX_Q6_K && qd == STYX_Q6_K);
}

int fused_block_threads() { return kFusedBlock; }

}  // namespace styx
