// attn_fused.cu -- the attention half of a decode layer as ONE cooperative
// kernel (sm_100a): what styx_attn_block otherwise runs as seven launches
// (crates/model/src/moe.rs:1857-1972).
//
// 148 CTAs x 512 threads, one per SM.  Phases:
//   0  the CTA's rows of Wq|Wk|Wv and of Wo start streaming into shared
//      memory (bulk copies) before the grid dependency resolves: weights do
//      not depend on x
//   A  x -> RMSNorm(attn_norm) -> digits (every CTA, all of x)
//   B  the CTA's rows of q|k|v (dp4a dot products); each head's rows are
//      published with a per-head arrival count
//   C  CTA (kv head j, split s): waits for its q heads, k and v; per-head
//      RMSNorm + NEOX RoPE in shared memory; split 0 writes the K / V cache
//      row at pos; scores, softmax statistics and P.V over its cache rows
//      (row pos from shared memory); partials published with a count per kv
//      head
//   D  CTA h < n_heads merges head h's splits -> att[h]; one count for all
//   E  every CTA: att -> digits, its rows of Wo . att added to x (the
//      residual add fused)
// Exchanges are monotonic counters in the workspace, never reset (launch
// tag = launch number + 1 from a counter every CTA increments once): a
// phase waits until its counter reaches tag x (arrivals per launch).  Every
// wait is bounded (~1 s): it then records an error code and goes on, so the
// kernel always ends.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

namespace styx {
namespace {

constexpr int kAF = 512;                 // threads
constexpr int kAFWarps = kAF / 32;
constexpr int kHD = 128;                 // head_dim of the fused form
constexpr int kAFHeadsPerPass = 8;
constexpr long long kAFPollFree = 100000;   // cycles of tight polling before backing off

// 16-byte asynchronous copies global -> shared (no registers held while in flight)
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ unsigned long long ld_acq(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// one thread waits until *cnt >= target (bounded); false after giving up
__device__ bool wait_count(const unsigned long long *cnt, unsigned long long target, int *err) {
    const long long t0 = clock64();
    while (ld_acq(cnt) < target) {
        const long long dt = clock64() - t0;
        if (dt > kSpinCycles) {
            atomicExch(err, kErrWaitRoute);
            return false;
        }
        if (dt > kAFPollFree) __nanosleep(256);
    }
    return true;
}

__device__ __forceinline__ float af_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float af_warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// block sum over 512 threads (fixed tree), result in every thread
__device__ __forceinline__ float af_block_sum(float v, float *red) {
    v = af_warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < kAFWarps ? red[lane] : 0.f;
#pragma unroll
    for (int o = 8; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return __shfl_sync(0xffffffffu, t, 0);
}

// the 16-byte-aligned cover of [p, p + n)
__device__ __forceinline__ void af_cover(const uint8_t *p, size_t n, uintptr_t &a, uint32_t &len) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(p);
    a = s & ~uintptr_t(15);
    len = static_cast<uint32_t>(((s + n + 15) & ~uintptr_t(15)) - a);
}

// Segment i of the CTA's q|k|v rows: rows [beg, end) of matrix m (0 q, 1 k, 2 v)
struct Seg {
    int m, beg, end, out0;   // out0: index of the segment's first row in q|k|v
};

__device__ __forceinline__ int qkv_segments(const AttnFusedArgs &p, int r0, int r1, Seg (&s)[3]) {
    const int qd = p.n_heads * kHD, kvd = p.n_kv * kHD;
    const int lim[4] = {0, qd, qd + kvd, qd + 2 * kvd};
    int n = 0;
    for (int m = 0; m < 3; m++) {
        const int a = max(r0, lim[m]), b = min(r1, lim[m + 1]);
        if (a < b) s[n++] = Seg{m, a - lim[m], b - lim[m], a};
    }
    return n;
}

template <int QW, int QV>
__global__ void __launch_bounds__(kAF, 1) k_attn_fused(const __grid_constant__ AttnFusedArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int H = p.H, qd = p.n_heads * kHD, kvd = p.n_kv * kHD, gqa = p.n_heads / p.n_kv;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);        // [0] q|k|v rows, [1] o rows
    float *red = reinterpret_cast<float *>(smem + 64);         // 32 floats
    uint32_t *s_tag = reinterpret_cast<uint32_t *>(smem + 192);
    int *s_ok = reinterpret_cast<int *>(smem + 196);
    uint32_t *s_soff = reinterpret_cast<uint32_t *>(smem + 200);   // smem offset of each segment's first row
    int8_t *dg1 = reinterpret_cast<int8_t *>(smem + p.off_dig);
    const int dmax = max(H, qd);
    uint8_t *dg2 = reinterpret_cast<uint8_t *>(dg1) + dmax;
    uint8_t *dg3 = dg2 + dmax;
    float *dsc = reinterpret_cast<float *>(dg3 + dmax);
    float *fst = reinterpret_cast<float *>(smem + p.off_f32);  // f32 staging [dmax]
    uint8_t *w1 = smem + p.off_w1;                             // q|k|v rows; later attention scratch
    uint8_t *w2 = smem + p.off_w2;                             // o rows

    const int R = qd + 2 * kvd;
    const int r0 = static_cast<int>(static_cast<long long>(R) * b / G);
    const int r1 = static_cast<int>(static_cast<long long>(R) * (b + 1) / G);
    const int o0 = static_cast<int>(static_cast<long long>(H) * b / G);
    const int o1 = static_cast<int>(static_cast<long long>(H) * (b + 1) / G);
    Seg seg[3];
    const int nseg = qkv_segments(p, r0, r1, seg);
#define AF_STAMP(i_)                                                           \
    do {                                                                       \
        if (tid == 0 && p.trace) p.trace[b * kAttnTraceStamps + (i_)] = clock64(); \
    } while (0)
    AF_STAMP(0);

    // ------------------------------------------------ phase 0
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        // q|k|v rows: each segment's cover, one after another
        uint32_t total = 0, off = 0;
        uintptr_t a[3];
        uint32_t len[3];
        for (int i = 0; i < nseg; i++) {
            const uint8_t *m = seg[i].m == 0 ? p.wq : seg[i].m == 1 ? p.wk : p.wv;
            const int rb = seg[i].m == 2 ? p.rb_v : p.rb_q;
            af_cover(m + static_cast<size_t>(seg[i].beg) * rb, static_cast<size_t>(seg[i].end - seg[i].beg) * rb,
                     a[i], len[i]);
            s_soff[i] = off + static_cast<uint32_t>(reinterpret_cast<uintptr_t>(m + static_cast<size_t>(seg[i].beg) *
                                                                                     rb) - a[i]);
            off += len[i];
            total += len[i];
        }
        if (total) {
            mbar_arrive_expect_tx(&bar[0], total);
            off = 0;
            for (int i = 0; i < nseg; i++) {
                bulk_g2s(w1 + off, reinterpret_cast<const void *>(a[i]), len[i], &bar[0]);
                off += len[i];
            }
        } else {
            mbar_arrive(&bar[0]);
        }
        // o rows
        uintptr_t ao;
        uint32_t lo = 0;
        if (o1 > o0) af_cover(p.wo + static_cast<size_t>(o0) * p.rb_o, static_cast<size_t>(o1 - o0) * p.rb_o, ao, lo);
        s_soff[3] = lo ? static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.wo + static_cast<size_t>(o0) * p.rb_o) -
                                               ao)
                       : 0;
        if (lo) {
            mbar_arrive_expect_tx(&bar[1], lo);
            bulk_g2s(w2, reinterpret_cast<const void *>(ao), lo, &bar[1]);
        } else {
            mbar_arrive(&bar[1]);
        }
        // this launch's tag: every CTA of the previous launch on this
        // workspace took its number before any could exit (each waits for
        // the others' heads), and no CTA of this one is resident before one
        // of the previous exits (one CTA per SM)
        *s_tag = static_cast<uint32_t>(atomicAdd(p.gen, 1ull) / static_cast<unsigned long long>(G)) + 1u;
        *s_ok = 1;
    }
    // the RoPE table of this token's position (theta_i = pos * theta_scale^i,
    // in double) and the norm weights: neither depends on the previous grid,
    // so they are ready before it ends (warps 2-3 and one float4 per thread)
    double2 *rope_t = reinterpret_cast<double2 *>(smem + p.off_rope);   // [64] (cos, sin)
    if (tid >= 64 && tid < 64 + kHD / 2) {
        const int i = tid - 64;
        const double th = static_cast<double>(p.n_t - 1) * pow(p.theta_scale, static_cast<double>(i));
        double sn, cs;
        sincos(th, &sn, &cs);
        rope_t[i] = make_double2(cs, sn);
    }
    const int H4 = H >> 2;
    float4 wn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H4) wn = __ldg(reinterpret_cast<const float4 *>(p.attn_norm) + tid);
    pdl_trigger();
    pdl_wait();
    __syncthreads();
    const unsigned long long tag = *s_tag;
    AF_STAMP(1);
    // this CTA's first cache rows of K and V (before row pos), in flight
    // while phases A and B run: warp w copies rows w and w + 16
    float *kpre = reinterpret_cast<float *>(smem + p.off_kv);   // [kPreRows][128]
    float *vpre = kpre + kPreRows * kHD;
    const int S = p.n_splits;
    const bool attn_cta = b < p.n_kv * S;
    const int kvh = attn_cta ? b / S : 0, split = attn_cta ? b % S : 0;
    const int t0 = split * p.tps, t1 = attn_cta ? min(p.n_t, t0 + p.tps) : 0, nt = t1 - t0;
    const int pos = p.n_t - 1;
    for (int t = warp; t < min(nt, kPreRows); t += kAFWarps) {
        if (t0 + t == pos) continue;
        const size_t off = static_cast<size_t>(t0 + t) * kvd + kvh * kHD + 4 * lane;
        cp_async16(kpre + t * kHD + 4 * lane, p.kcache + off);
        cp_async16(vpre + t * kHD + 4 * lane, p.vcache + off);
    }
    cp_async_commit();

    // ------------------------------------------------ phase A: x -> RMSNorm -> digits
    // (H <= 2048: at most one float4 of x per thread)
    float4 xr = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H4) xr = __ldcg(reinterpret_cast<const float4 *>(p.x) + tid);
    const float ss = af_block_sum(xr.x * xr.x + xr.y * xr.y + xr.z * xr.z + xr.w * xr.w, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(H) + p.eps);
    if (tid < H4)
        reinterpret_cast<float4 *>(fst)[tid] = make_float4(xr.x * scale * wn.x, xr.y * scale * wn.y,
                                                           xr.z * scale * wn.z, xr.w * scale * wn.w);
    __syncthreads();
    {   // four groups' shuffle chains together
        const DigitsView dv{dg1, dg2, dg3, dsc};
        for (int g0 = warp; g0 < (H >> 5); g0 += 4 * kAFWarps) {
            float v[4];
            int gi[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int g = g0 + j * kAFWarps;
                gi[j] = g < (H >> 5) ? g : -1;
                v[j] = g < (H >> 5) ? fst[g * 32 + lane] : 0.f;
            }
            digits_groups_warp<4>(v, gi, lane, dv);
        }
    }
    __syncthreads();
    AF_STAMP(2);

    // ------------------------------------------------ phase B: q|k|v rows
    {
        bool ok = mbar_wait(&bar[0], 0, p.err, kErrWaitFull);
        AF_STAMP(3);
        const int units = H >> 6, gs = units >= 32 ? 32 : units >= 16 ? 16 : units >= 8 ? 8 : units >= 4 ? 4 : 2;
        const int rpw = 32 / gs, ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        for (int i = 0; i < nseg; i++) {
            const int n = seg[i].end - seg[i].beg;
            const uint8_t *base = w1 + s_soff[i];
            XUnit x;
            if (seg[i].m == 2) {
                if (active) load_xunit<QV>(x, dg1, dg2, dg3, dsc, ug);
            } else {
                if (active) load_xunit<QW>(x, dg1, dg2, dg3, dsc, ug);
            }
            const int rb = seg[i].m == 2 ? p.rb_v : p.rb_q;
            for (int t = warp * rpw * 2; t < n; t += kAFWarps * rpw * 2) {   // two rows in flight
                const int ra = t + grp, rc = t + rpw + grp;
                float va = 0.f, vc = 0.f;
                if (ok && active) {
                    if (seg[i].m == 2) {
                        if (ra < n) va = unit_dot<QV>(base + static_cast<size_t>(ra) * rb, ug, x);
                        if (rc < n) vc = unit_dot<QV>(base + static_cast<size_t>(rc) * rb, ug, x);
                    } else {
                        if (ra < n) va = unit_dot<QW>(base + static_cast<size_t>(ra) * rb, ug, x);
                        if (rc < n) vc = unit_dot<QW>(base + static_cast<size_t>(rc) * rb, ug, x);
                    }
                }
                __syncwarp();
                for (int o = gs >> 1; o; o >>= 1) {
                    va += __shfl_xor_sync(0xffffffffu, va, o);
                    vc += __shfl_xor_sync(0xffffffffu, vc, o);
                }
                if (ug == 0 && ra < n) p.qkv[seg[i].out0 + ra] = va;
                if (ug == 0 && rc < n) p.qkv[seg[i].out0 + rc] = vc;
            }
        }
        __syncthreads();
        AF_STAMP(13);
        if (tid == 0) {   // publish: rows of each head this CTA wrote
            __threadfence();
            for (int i = 0; i < nseg; i++) {
                const int lo = seg[i].out0, hi = seg[i].out0 + seg[i].end - seg[i].beg;
                for (int h = lo / kHD; h * kHD < hi; h++) {
                    const int n = min(hi, (h + 1) * kHD) - max(lo, h * kHD);
                    atomicAdd(p.head_cnt + h, static_cast<unsigned long long>(n));
                }
            }
        }
    }
    AF_STAMP(4);

    // ------------------------------------------------ phase C: attention partials
    cp_async_wait_all();
    if (attn_cta) {
        float *sq = reinterpret_cast<float *>(w1);                 // [gqa][128] q heads
        float *sk = sq + gqa * kHD;                                // [128] k (row pos)
        float *sv = sk + kHD;                                      // [128] v (row pos)
        const double2 *rope = rope_t;                              // [64] (cos, sin), computed at entry
        float *ssc = sv + 3 * kHD;                                 // [tps][gqa] (a table-sized gap after v)
        float *sml = ssc + p.tps * gqa;                            // [gqa][2]
        float *sacc = sml + ((2 * gqa + 3) & ~3);                  // [8][8][128]
        // wait for the gqa q heads, k head and v head of kvh (lanes of warp 0)
        if (warp == 0) {
            bool fine = true;
            if (lane < gqa + 2) {
                const int h = lane < gqa ? kvh * gqa + lane : lane == gqa ? p.n_heads + kvh : p.n_heads + p.n_kv + kvh;
                fine = wait_count(p.head_cnt + h, tag * kHD, p.err);
            }
            fine = __all_sync(0xffffffffu, fine);
            if (lane == 0 && !fine) *s_ok = 0;
        }
        __syncthreads();
        AF_STAMP(5);
        const bool ok = *s_ok;
        for (int i = tid; i < gqa * kHD; i += kAF) sq[i] = __ldcg(p.qkv + kvh * gqa * kHD + i);
        for (int i = tid; i < kHD; i += kAF) {
            sk[i] = __ldcg(p.qkv + qd + kvh * kHD + i);
            sv[i] = __ldcg(p.qkv + qd + kvd + kvh * kHD + i);
        }
        __syncthreads();
        // per-head RMSNorm + RoPE (warp per head): lane l owns elements
        // l, l+32 (first halves of its two pairs) and l+64, l+96
        for (int h = warp; h <= gqa; h += kAFWarps) {
            float *hv = h < gqa ? sq + h * kHD : sk;
            const float *nw = h < gqa ? p.q_norm : p.k_norm;
            float e0 = hv[lane], e1 = hv[lane + 32], e2 = hv[lane + 64], e3 = hv[lane + 96];
            if (nw) {
                const float s2 = af_warp_sum(e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3);
                const float sc = 1.0f / sqrtf(s2 / static_cast<float>(kHD) + p.eps);
                e0 = e0 * sc * nw[lane];
                e1 = e1 * sc * nw[lane + 32];
                e2 = e2 * sc * nw[lane + 64];
                e3 = e3 * sc * nw[lane + 96];
            }
            const double2 ra = rope[lane], rb = rope[lane + 32];
            const double a0 = e0, a1 = e1, a2 = e2, a3 = e3;
            hv[lane] = static_cast<float>(a0 * ra.x - a2 * ra.y);
            hv[lane + 64] = static_cast<float>(a0 * ra.y + a2 * ra.x);
            hv[lane + 32] = static_cast<float>(a1 * rb.x - a3 * rb.y);
            hv[lane + 96] = static_cast<float>(a1 * rb.y + a3 * rb.x);
        }
        __syncthreads();
        if (split == 0) {   // the cache rows of this token
            float *kr = p.kcache + static_cast<size_t>(pos) * kvd + kvh * kHD;
            float *vr = p.vcache + static_cast<size_t>(pos) * kvd + kvh * kHD;
            for (int i = tid; i < kHD; i += kAF) {
                kr[i] = sk[i];
                vr[i] = sv[i];
            }
        }
        // scores: one token per warp pass, lane c holds elements 4c..4c+3
        for (int t = warp; t < nt; t += kAFWarps) {
            const int tt = t0 + t;
            const float4 kv = tt == pos       ? *reinterpret_cast<const float4 *>(sk + 4 * lane)
                              : t < kPreRows ? *reinterpret_cast<const float4 *>(kpre + t * kHD + 4 * lane)
                                             : __ldg(reinterpret_cast<const float4 *>(
                                                   p.kcache + static_cast<size_t>(tt) * kvd + kvh * kHD) + lane);
            for (int g = 0; g < gqa; g++) {
                const float4 qv = *reinterpret_cast<const float4 *>(sq + g * kHD + 4 * lane);
                float d = qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
                d = af_warp_sum(d);
                if (lane == 0) ssc[t * gqa + g] = d * p.scale;
            }
        }
        __syncthreads();
        AF_STAMP(6);
        for (int g = warp; g < gqa; g += kAFWarps) {
            float m = -INFINITY;
            for (int t = lane; t < nt; t += 32) m = fmaxf(m, ssc[t * gqa + g]);
            m = af_warp_max(m);
            float l = 0.f;
            for (int t = lane; t < nt; t += 32) {
                const float pr = expf(ssc[t * gqa + g] - m);
                ssc[t * gqa + g] = pr;
                l += pr;
            }
            l = af_warp_sum(l);
            if (lane == 0) {
                sml[2 * g] = m;
                sml[2 * g + 1] = l;
            }
        }
        __syncthreads();
        for (int g0 = 0; g0 < gqa; g0 += kAFHeadsPerPass) {
            const int ng = min(kAFHeadsPerPass, gqa - g0);
            float4 acc[kAFHeadsPerPass];
#pragma unroll
            for (int g = 0; g < kAFHeadsPerPass; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int t = warp; t < nt; t += kAFWarps) {
                const int tt = t0 + t;
                const float4 vv = tt == pos       ? *reinterpret_cast<const float4 *>(sv + 4 * lane)
                                  : t < kPreRows ? *reinterpret_cast<const float4 *>(vpre + t * kHD + 4 * lane)
                                                 : __ldg(reinterpret_cast<const float4 *>(
                                                       p.vcache + static_cast<size_t>(tt) * kvd + kvh * kHD) + lane);
#pragma unroll
                for (int g = 0; g < kAFHeadsPerPass; g++) {
                    if (g < ng) {
                        const float pr = ssc[t * gqa + g0 + g];
                        acc[g].x += pr * vv.x;
                        acc[g].y += pr * vv.y;
                        acc[g].z += pr * vv.z;
                        acc[g].w += pr * vv.w;
                    }
                }
            }
            // 16 warps' accumulators -> 8 slots (warp w + 8 into w's), then summed
            if (warp >= 8) {
#pragma unroll
                for (int g = 0; g < kAFHeadsPerPass; g++)
                    *reinterpret_cast<float4 *>(sacc + ((warp - 8) * kAFHeadsPerPass + g) * kHD + 4 * lane) = acc[g];
            }
            __syncthreads();
            if (warp < 8) {
#pragma unroll
                for (int g = 0; g < kAFHeadsPerPass; g++) {
                    float4 *d = reinterpret_cast<float4 *>(sacc + (warp * kAFHeadsPerPass + g) * kHD + 4 * lane);
                    const float4 o = *d;
                    *d = make_float4(acc[g].x + o.x, acc[g].y + o.y, acc[g].z + o.z, acc[g].w + o.w);
                }
            }
            __syncthreads();
            for (int i = tid; i < ng * kHD; i += kAF) {
                const int g = i / kHD, c = i - g * kHD;
                float s = 0.f;
                for (int w = 0; w < 8; w++) s += sacc[(w * kAFHeadsPerPass + g) * kHD + c];
                p.part_acc[(static_cast<size_t>(kvh * gqa + g0 + g) * S + split) * kHD + c] = ok ? s : 0.f;
            }
            __syncthreads();
        }
        for (int g = tid; g < gqa; g += kAF) {
            const size_t ix = static_cast<size_t>(kvh * gqa + g) * S + split;
            p.part_ml[2 * ix] = ok ? sml[2 * g] : 0.f;
            p.part_ml[2 * ix + 1] = ok ? sml[2 * g + 1] : 1.f;
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(p.split_cnt + kvh, 1ull);
        }
    }
    AF_STAMP(7);

    // ------------------------------------------------ phase D: merge head b's splits
    if (b < p.n_heads) {
        float *w = reinterpret_cast<float *>(w1);   // [S] split weights
        if (tid == 0 && !wait_count(p.split_cnt + b / gqa, tag * static_cast<unsigned long long>(S), p.err))
            *s_ok = 0;
        __syncthreads();
        AF_STAMP(8);
        const float *ml = p.part_ml + static_cast<size_t>(b) * S * 2;
        // every load of the merge in flight at once: thread s < S its split's
        // (max, sum) pair (S <= kAttnMaxSplits < kAF), and thread (c, q) the
        // partials of column c for splits q, q+4, .. (the first kMergeRegs
        // of them into registers)
        const float *acc = p.part_acc + static_cast<size_t>(b) * S * kHD;
        const int c = tid & (kHD - 1), q = tid >> 7;
        constexpr int kMergeRegs = 16;
        float av[kMergeRegs];
#pragma unroll
        for (int i = 0; i < kMergeRegs; i++) {
            const int s = q + (kAF / kHD) * i;
            av[i] = s < S ? __ldcg(acc + static_cast<size_t>(s) * kHD + c) : 0.f;
        }
        float mv = -INFINITY, lv = 0.f;
        if (tid < S) {
            mv = __ldcg(ml + 2 * tid);
            lv = __ldcg(ml + 2 * tid + 1);
        }
        const float m = af_warp_max(mv);
        if (lane == 0) red[warp] = m;
        __syncthreads();
        float M = -INFINITY;
        for (int i = 0; i < kAFWarps; i++) M = fmaxf(M, red[i]);
        __syncthreads();
        float l = 0.f;
        if (tid < S) {
            const float ws = expf(mv - M);
            w[tid] = ws;
            l += ws * lv;
        }
        const float L = af_block_sum(l, red);
        const float inv = 1.0f / L;
        // column c summed by four threads (splits q, q+4, ..), then the four
        // partials in order
        {
            float o = 0.f;
#pragma unroll
            for (int i = 0; i < kMergeRegs; i++) {
                const int s = q + (kAF / kHD) * i;
                if (s < S) o += w[s] * av[i];
            }
            for (int s = q + (kAF / kHD) * kMergeRegs; s < S; s += kAF / kHD)
                o += w[s] * __ldcg(acc + static_cast<size_t>(s) * kHD + c);
            fst[q * kHD + c] = o;
        }
        __syncthreads();
        if (warp < kHD / 32) {   // head b's 4 groups of 32 -> digits, published for phase E
            const int c = warp * 32 + lane;
            const float o = (fst[c] + fst[kHD + c] + fst[2 * kHD + c] + fst[3 * kHD + c]) * inv;
            const DigitsView dv{p.att_d1 + b * kHD, p.att_d2 + b * kHD, p.att_d3 + b * kHD, p.att_sc + b * (kHD / 32)};
            digits_group_warp(o, lane, dv, warp);
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(p.att_cnt, 1ull);
        }
    }

    // ------------------------------------------------ phase E: x += Wo . att
    AF_STAMP(9);
    if (tid == 0 && !wait_count(p.att_cnt, tag * static_cast<unsigned long long>(p.n_heads), p.err)) *s_ok = 0;
    __syncthreads();
    AF_STAMP(10);
    {
        // att's digits, as the merging CTAs published them
        for (int i = tid; i < qd / 16; i += kAF) {
            reinterpret_cast<uint4 *>(dg1)[i] = __ldcg(reinterpret_cast<const uint4 *>(p.att_d1) + i);
            reinterpret_cast<uint4 *>(dg2)[i] = __ldcg(reinterpret_cast<const uint4 *>(p.att_d2) + i);
            reinterpret_cast<uint4 *>(dg3)[i] = __ldcg(reinterpret_cast<const uint4 *>(p.att_d3) + i);
        }
        for (int i = tid; i < qd / 32; i += kAF) dsc[i] = __ldcg(p.att_sc + i);
        __syncthreads();
        AF_STAMP(11);
        const bool ok = mbar_wait(&bar[1], 0, p.err, kErrWaitFull) && *s_ok;
        // the row's units in groups of 32 (one unit per lane, its digits
        // loaded once), each group on kAFWarps / ngrp warps that walk the
        // rows; the groups' sums are added in group order
        const int units = qd >> 6, ngrp = (units + 31) >> 5, wpg = kAFWarps / ngrp;
        const int grp = warp / wpg, u = grp * 32 + lane;
        const int n = o1 - o0;
        const uint8_t *base = w2 + s_soff[3];
        float *opart = fst;   // [ngrp][n]
        XUnit x;
        if (grp < ngrp && u < units) load_xunit<QW>(x, dg1, dg2, dg3, dsc, u);
        for (int row = warp % wpg; grp < ngrp && row < n; row += wpg) {
            float v = 0.f;
            if (ok && u < units) v = unit_dot<QW>(base + static_cast<size_t>(row) * p.rb_o, u, x);
            __syncwarp();
            v = af_warp_sum(v);
            if (lane == 0) opart[grp * n + row] = v;
        }
        __syncthreads();
        if (tid < n && ok) {
            float v = 0.f;
            for (int g = 0; g < ngrp; g++) v += opart[g * n + tid];
            p.x[o0 + tid] = p.x[o0 + tid] + v;
        }
    }
    AF_STAMP(12);
#undef AF_STAMP
    // no copies in flight at exit (both barriers completed above on the
    // normal path; after a timed-out wait, wait for them, bounded)
    if (tid == 0) {
        mbar_wait(&bar[0], 0, p.err, kErrWaitFull);
        mbar_wait(&bar[1], 0, p.err, kErrWaitFull);
    }
}

}  // namespace

bool attn_fused_supported(int qw, int qv) {
    return (qw == STYX_Q4_K && (qv == STYX_Q6_K || qv == STYX_Q4_K)) || (qw == STYX_Q8_0 && qv == STYX_Q8_0) ||
           (qw == STYX_Q5_K && (qv == STYX_Q6_K || qv == STYX_Q5_K)) || (qw == STYX_Q6_K && qv == STYX_Q6_K);
}

int attn_fused_threads() { return kAF; }

template <class Kern>
static cudaError_t launch_af(Kern kern, const AttnFusedArgs &a, int grid, uint32_t smem, bool coop, cudaStream_t st) {
    const cudaError_t e = resident_fit(reinterpret_cast<const void *>(kern), kAF, smem, grid);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kAF);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = coop ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_attn_fused(const AttnFusedArgs &a, int qw, int qv, int grid, uint32_t smem, bool coop,
                              cudaStream_t st) {
#define STYX_AF_CASE(W_, V_) \
    if (qw == W_ && qv == V_) return launch_af(k_attn_fused<W_, V_>, a, grid, smem, coop, st);
    STYX_AF_CASE(STYX_Q4_K, STYX_Q6_K)
    STYX_AF_CASE(STYX_Q4_K, STYX_Q4_K)
    STYX_AF_CASE(STYX_Q8_0, STYX_Q8_0)
    STYX_AF_CASE(STYX_Q5_K, STYX_Q6_K)
    STYX_AF_CASE(STYX_Q5_K, STYX_Q5_K)
    STYX_AF_CASE(STYX_Q6_K, STYX_Q6_K)
#undef STYX_AF_CASE
    return cudaErrorNotSupported;
}

}  // namespace styx
