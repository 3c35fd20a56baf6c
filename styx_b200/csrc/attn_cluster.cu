// attn_cluster.cu -- the attention half of a decode layer as one launch of
// thread-block clusters (sm_100a): one cluster of C CTAs (C <= 16) per kv
// head, head_dim 128.  What styx_attn_block otherwise runs as seven launches
// (crates/model/src/moe.rs:1857-1972) or as one cooperative kernel whose
// phases exchange through global counters.
//
// Nothing waits across clusters: the q heads of kv head j, its k and v rows,
// the attention of those heads over the cache and the Wo columns of those
// heads all belong to cluster j, so every exchange is a cluster barrier over
// distributed shared memory; the n_kv clusters' shares of Wo . att are added
// by whichever CTA completes a row block last (a counter per block).  The
// launch needs no co-resident grid.
//
// Phases of CTA r of cluster j (512 threads, one CTA per SM):
//   0  bulk copies of the CTA's rows of Wq (q rows [nq r/C, nq (r+1)/C) of
//      the cluster's heads), Wk and Wv (rows [128 r/C, 128 (r+1)/C) of kv
//      head j) -- weights, read before the grid dependency resolves; the
//      next kernel may launch (PDL); wait for the previous grid; the CTA's
//      first cache rows of K and V (its split of the sequence) start
//      landing (async copies);
//   A  x -> RMSNorm(attn_norm) -> dp4a digits (every CTA, all of x);
//   B  the CTA's q / k / v rows; every value is stored into every CTA of
//      the cluster; the CTA's Wo slice (its output rows, the cluster's
//      columns) starts landing where the q / k / v rows were; one cluster
//      barrier;
//   C  per-head RMSNorm + NEOX RoPE of the q heads and k (every CTA); the CTA
//      whose split holds the token's position writes the cache rows; scores,
//      softmax statistics and P.V over the CTA's cache rows; each head's
//      partial goes to CTA g of the cluster (head g); one cluster barrier;
//      CTA g merges head g and stores att[g] into every CTA; one cluster
//      barrier;
//   E  att -> digits; the CTA's o rows over the cluster's columns; the share
//      goes to the workspace; the last of the n_kv clusters for a row block
//      adds the shares in cluster order: x += Wo . att (rec_add fused).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <vector>

#include "cluster.cuh"
#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

namespace styx {
namespace {

constexpr int kAC = 512;   // threads
constexpr int kACWarps = kAC / 32;
constexpr int kHD = 128;   // head_dim
constexpr int kMrecvStride = 132;   // floats per received partial: acc[128], m, l, pad

__device__ __forceinline__ void cpa16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// the 16-byte-aligned cover of [p, p + n)
__device__ __forceinline__ void cover(const uint8_t *p, size_t n, uintptr_t &a, uint32_t &len) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(p);
    a = s & ~uintptr_t(15);
    len = static_cast<uint32_t>(((s + n + 15) & ~uintptr_t(15)) - a);
}

struct AcHdr {
    uint64_t bar;          // q / k / v rows
    float red[kACWarps];
    uint32_t soff[3];      // offset of each matrix's first row inside the weight region
    int last;              // this CTA completes its row block
};
static_assert(sizeof(AcHdr) <= kAttnClusterHeader, "attention cluster header overflows");

template <int QW, int QV>
__global__ void __launch_bounds__(kAC, 1) k_attn_cluster(const __grid_constant__ AttnClusterArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    AcHdr &hd = *reinterpret_cast<AcHdr *>(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = p.C, H = p.H, gqa = p.n_heads / p.n_kv, kvd = p.n_kv * kHD;
    const int j = blockIdx.x / C;                         // the cluster's kv head
    const int r = static_cast<int>(cluster_ctarank());
    const int nq = gqa * kHD;
    float *xf = reinterpret_cast<float *>(smem + p.off_x);            // [H]
    int8_t *dg1 = reinterpret_cast<int8_t *>(smem + p.off_dig);       // digits of x_norm
    uint8_t *dg2 = reinterpret_cast<uint8_t *>(dg1) + H;
    uint8_t *dg3 = dg2 + H;
    float *dsc = reinterpret_cast<float *>(dg3 + H);
    float *sq = reinterpret_cast<float *>(smem + p.off_q);            // [gqa][128] q heads
    float *sk = sq + nq;                                              // [128] k
    float *sv = sk + kHD;                                             // [128] v
    double2 *rope = reinterpret_cast<double2 *>(smem + p.off_rope);   // [64] (cos, sin)
    float *ssc = reinterpret_cast<float *>(smem + p.off_sc);          // [tps][gqa] scores, then probabilities
    float *sml = ssc + ((p.tps * gqa + 3) & ~3);                      // [gqa][2] max, sum
    float *sacc = reinterpret_cast<float *>(smem + p.off_acc);        // [hpw][gqa][128] P.V partials
    float *mrecv = reinterpret_cast<float *>(smem + p.off_mrecv);     // [C][132] partials of head r
    float *satt = reinterpret_cast<float *>(smem + p.off_att);        // [gqa][128] att
    int8_t *ad1 = reinterpret_cast<int8_t *>(smem + p.off_adig);      // digits of att
    uint8_t *ad2 = reinterpret_cast<uint8_t *>(ad1) + nq;
    uint8_t *ad3 = ad2 + nq;
    float *asc = reinterpret_cast<float *>(ad3 + nq);
    float *so = reinterpret_cast<float *>(smem + p.off_o);            // the CTA's o rows
    uint8_t *wbuf = smem + p.off_w;                                   // q|k|v rows, then the Wo slice
    float *kpre = reinterpret_cast<float *>(smem + p.off_kv);         // [npre][128]
    float *vpre = kpre + p.npre * kHD;

    const int q0 = nq * r / C, nqr = nq * (r + 1) / C - q0;       // q rows (of the cluster's heads)
    const int k0 = kHD * r / C, nkr = kHD * (r + 1) / C - k0;     // k rows and v rows (of kv head j)
    const int o0 = H * r / C, nor = H * (r + 1) / C - o0;         // o rows
    const int t0 = r * p.tps, t1 = min(p.n_t, t0 + p.tps), nt = max(0, t1 - t0);
    const int pos = p.n_t - 1;
    const int H4 = H >> 2;
    const uint32_t blk_o = static_cast<uint32_t>(p.rb_o / p.n_kv);   // bytes of the cluster's columns per Wo row

#define AC_STAMP(i_)                                                                       \
    do {                                                                                   \
        if (tid == 0 && p.trace) p.trace[blockIdx.x * kAttnTraceStamps + (i_)] = clock64(); \
    } while (0)
    AC_STAMP(0);
    // ------------------------------------------------ phase 0
    if (tid == 0) {
        mbar_init(&hd.bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {   // q, k, v rows: each matrix's cover, one after another
        const uint8_t *src[3] = {p.wq + static_cast<size_t>(j * nq + q0) * p.rb_q,
                                 p.wk + static_cast<size_t>(j * kHD + k0) * p.rb_q,
                                 p.wv + static_cast<size_t>(j * kHD + k0) * p.rb_v};
        const size_t bytes[3] = {static_cast<size_t>(nqr) * p.rb_q, static_cast<size_t>(nkr) * p.rb_q,
                                 static_cast<size_t>(nkr) * p.rb_v};
        uintptr_t a[3];
        uint32_t len[3], total = 0;
        for (int i = 0; i < 3; i++) {
            len[i] = 0;
            if (bytes[i]) cover(src[i], bytes[i], a[i], len[i]);
            hd.soff[i] = total + (len[i] ? static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src[i]) - a[i]) : 0u);
            total += len[i];
        }
        if (total) {
            mbar_arrive_expect_tx(&hd.bar, total);
            uint32_t off = 0;
            for (int i = 0; i < 3; i++)
                if (len[i]) {
                    bulk_g2s(wbuf + off, reinterpret_cast<const void *>(a[i]), len[i], &hd.bar);
                    off += len[i];
                }
        } else {
            mbar_arrive(&hd.bar);
        }
    }
    float4 wn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H4) wn = __ldg(reinterpret_cast<const float4 *>(p.attn_norm) + tid);
    cl_arrive_relaxed();   // this CTA runs: its shared memory may receive values once all have arrived
    pdl_trigger();
    pdl_wait();
    AC_STAMP(1);
    // this CTA's first cache rows of K and V (row pos is this launch's own)
    for (int t = warp; t < min(nt, p.npre); t += kACWarps) {
        if (t0 + t == pos) continue;
        const size_t off = static_cast<size_t>(t0 + t) * kvd + j * kHD + 4 * lane;
        cpa16(kpre + t * kHD + 4 * lane, p.kcache + off);
        cpa16(vpre + t * kHD + 4 * lane, p.vcache + off);
    }
    cpa_commit();

    // ------------------------------------------------ phase A: x -> RMSNorm -> digits
    {
        float4 xr = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tid < H4) xr = __ldcg(reinterpret_cast<const float4 *>(p.x) + tid);
        float ss = wsum(xr.x * xr.x + xr.y * xr.y + xr.z * xr.z + xr.w * xr.w);
        if (lane == 0) hd.red[warp] = ss;
        __syncthreads();
        float t = lane < kACWarps ? hd.red[lane] : 0.f;
#pragma unroll
        for (int o = 8; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        const float scale = 1.0f / sqrtf(__shfl_sync(0xffffffffu, t, 0) / static_cast<float>(H) + p.eps);
        if (tid < H4) {
            float4 v = xr;
            v.x = v.x * scale * wn.x;
            v.y = v.y * scale * wn.y;
            v.z = v.z * scale * wn.z;
            v.w = v.w * scale * wn.w;
            reinterpret_cast<float4 *>(xf)[tid] = v;
        }
        __syncthreads();
        const DigitsView dv{dg1, dg2, dg3, dsc};
        for (int g = warp; g < (H >> 5); g += kACWarps) digits_group_warp(xf[g * 32 + lane], lane, dv, g);
        __syncthreads();
    }
    AC_STAMP(2);
    cl_wait();   // every CTA of the cluster runs

    // ------------------------------------------------ phase B: q / k / v rows
    bool ok = mbar_wait(&hd.bar, 0, p.err, kErrWaitFull);
    AC_STAMP(3);
    {
        const int units = H >> 6, gs = units >= 32 ? 32 : units >= 16 ? 16 : units >= 8 ? 8 : units >= 4 ? 4 : 2;
        const int rpw = 32 / gs, ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        const uint32_t sq_s = smem_addr(sq);
        for (int m = 0; m < 3; m++) {
            const int n = m == 0 ? nqr : nkr;
            const int rb = m == 2 ? p.rb_v : p.rb_q;
            const uint8_t *base = wbuf + hd.soff[m];
            const uint32_t dst0 = sq_s + 4u * static_cast<uint32_t>(m == 0 ? q0 : m == 1 ? nq + k0 : nq + kHD + k0);
            XUnit x;
            if (active) {
                if (m == 2) load_xunit<QV>(x, dg1, dg2, dg3, dsc, ug);
                else load_xunit<QW>(x, dg1, dg2, dg3, dsc, ug);
            }
            for (int t = warp * rpw * 2; t < n; t += kACWarps * rpw * 2) {   // two rows in flight
                const int ra = t + grp, rc = t + rpw + grp;
                float va = 0.f, vc = 0.f;
                if (ok && active) {
                    if (m == 2) {
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
                for (int q = ug; q < C; q += gs) {   // into every CTA of the cluster
                    if (ra < n) cl_st(cl_map(dst0 + 4u * ra, q), va);
                    if (rc < n) cl_st(cl_map(dst0 + 4u * rc, q), vc);
                }
            }
        }
    }
    AC_STAMP(9);
    __syncthreads();   // the q / k / v rows are read: their space takes the Wo slice
    {   // the CTA's o rows, the cluster's columns: blk_o bytes at column offset j * blk_o of each row
        const int per_row = static_cast<int>(blk_o >> 4);
        for (int c = tid; c < nor * per_row; c += kAC) {
            const int row = c / per_row, part = c - row * per_row;
            cpa16(wbuf + static_cast<size_t>(row) * blk_o + part * 16,
                  p.wo + static_cast<size_t>(o0 + row) * p.rb_o + j * blk_o + part * 16);
        }
        cpa_commit();
    }
    AC_STAMP(10);
    cl_arrive();
    cl_wait();   // q heads, k and v complete in every CTA
    AC_STAMP(4);

    // ------------------------------------------------ phase C: attention over the CTA's cache rows
    if (tid < kHD / 2) {   // RoPE table: theta_i = pos * theta_scale^i, in double
        const double th = static_cast<double>(pos) * pow(p.theta_scale, static_cast<double>(tid));
        double sn, cs;
        sincos(th, &sn, &cs);
        rope[tid] = make_double2(cs, sn);
    }
    __syncthreads();
    // per-head RMSNorm + RoPE (warp per head): lane l owns elements l, l+32
    // (first halves of its two pairs) and l+64, l+96
    for (int h = warp; h <= gqa; h += kACWarps) {
        float *hv = h < gqa ? sq + h * kHD : sk;
        const float *nw = h < gqa ? p.q_norm : p.k_norm;
        float e0 = hv[lane], e1 = hv[lane + 32], e2 = hv[lane + 64], e3 = hv[lane + 96];
        if (nw) {
            const float s2 = wsum(e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3);
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
    AC_STAMP(11);
    cpa_wait<1>();   // the cache rows (the Wo slice may still be landing)
    __syncthreads();
    if (pos >= t0 && pos < t1 && tid < kHD) {   // the cache rows of this token
        p.kcache[static_cast<size_t>(pos) * kvd + j * kHD + tid] = sk[tid];
        p.vcache[static_cast<size_t>(pos) * kvd + j * kHD + tid] = sv[tid];
    }
    // scores: one token per warp pass, lane c holds elements 4c..4c+3
    for (int t = warp; t < nt; t += kACWarps) {
        const int tt = t0 + t;
        const float4 kv = tt == pos      ? *reinterpret_cast<const float4 *>(sk + 4 * lane)
                          : t < p.npre ? *reinterpret_cast<const float4 *>(kpre + t * kHD + 4 * lane)
                                       : __ldg(reinterpret_cast<const float4 *>(
                                             p.kcache + static_cast<size_t>(tt) * kvd + j * kHD) + lane);
        for (int g = 0; g < gqa; g++) {
            const float4 qv = *reinterpret_cast<const float4 *>(sq + g * kHD + 4 * lane);
            const float d = wsum(qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w);
            if (lane == 0) ssc[t * gqa + g] = d * p.scale;
        }
    }
    __syncthreads();
    AC_STAMP(12);
    for (int g = warp; g < gqa; g += kACWarps) {   // softmax statistics, probabilities in place
        float m = -INFINITY;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, ssc[t * gqa + g]);
        m = wmax(m);
        float l = 0.f;
        for (int t = lane; t < nt; t += 32) {
            const float pr = expf(ssc[t * gqa + g] - m);
            ssc[t * gqa + g] = pr;
            l += pr;
        }
        l = wsum(l);
        if (lane == 0) {
            sml[2 * g] = m;
            sml[2 * g + 1] = l;
        }
    }
    __syncthreads();
    {   // P.V: warp w takes head w / hpw and every hpw-th of the CTA's tokens
        const int hpw = kACWarps / gqa >= 1 ? kACWarps / gqa : 1;
        const int g = warp / hpw, sub = warp % hpw;
        if (g < gqa) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int t = sub; t < nt; t += hpw) {
                const int tt = t0 + t;
                const float4 vv = tt == pos      ? *reinterpret_cast<const float4 *>(sv + 4 * lane)
                                  : t < p.npre ? *reinterpret_cast<const float4 *>(vpre + t * kHD + 4 * lane)
                                               : __ldg(reinterpret_cast<const float4 *>(
                                                     p.vcache + static_cast<size_t>(tt) * kvd + j * kHD) + lane);
                const float pr = ssc[t * gqa + g];
                acc.x += pr * vv.x;
                acc.y += pr * vv.y;
                acc.z += pr * vv.z;
                acc.w += pr * vv.w;
            }
            *reinterpret_cast<float4 *>(sacc + (sub * gqa + g) * kHD + 4 * lane) = acc;
        }
        // (warps past gqa * hpw hold nothing)
        __syncthreads();
        AC_STAMP(13);
        // head g's partial (acc[128], m, l) into CTA g's receive rows, row r
        const uint32_t mr_s = smem_addr(mrecv) + 4u * static_cast<uint32_t>(r * kMrecvStride);
        for (int i = tid; i < gqa * (kHD + 2); i += kAC) {
            const int gg = i / (kHD + 2), c = i - gg * (kHD + 2);
            float v;
            if (c < kHD) {
                v = 0.f;
                for (int s2 = 0; s2 < hpw; s2++) v += sacc[(s2 * gqa + gg) * kHD + c];
            } else {
                v = sml[2 * gg + (c - kHD)];
            }
            cl_st(cl_map(mr_s + 4u * c, static_cast<uint32_t>(gg)), v);
        }
    }
    AC_STAMP(14);
    cl_arrive();
    cl_wait();   // CTA g < gqa holds every CTA's partial of head g
    AC_STAMP(5);
    if (r < gqa && tid < kHD) {   // merge head r and store att[r] into every CTA
        float M = -INFINITY;
        for (int s2 = 0; s2 < C; s2++) M = fmaxf(M, mrecv[s2 * kMrecvStride + kHD]);
        float L = 0.f, o = 0.f;
        for (int s2 = 0; s2 < C; s2++) {
            const float w = expf(mrecv[s2 * kMrecvStride + kHD] - M);   // 0 for an empty split
            L += w * mrecv[s2 * kMrecvStride + kHD + 1];
            o += w * mrecv[s2 * kMrecvStride + tid];
        }
        o = o / L;
        const uint32_t a = smem_addr(satt) + 4u * static_cast<uint32_t>(r * kHD + tid);
        for (int q = 0; q < C; q++) cl_st(cl_map(a, static_cast<uint32_t>(q)), o);
    }
    cl_arrive();
    cl_wait();   // att of every q head of the cluster in every CTA
    AC_STAMP(6);

    // ------------------------------------------------ phase E: x += Wo . att
    {
        const DigitsView dv{ad1, ad2, ad3, asc};
        for (int g = warp; g < (nq >> 5); g += kACWarps) digits_group_warp(satt[g * 32 + lane], lane, dv, g);
    }
    cpa_wait<0>();   // the Wo slice
    __syncthreads();
    AC_STAMP(7);
    {
        const int units = nq >> 6, gs = units >= 32 ? 32 : units >= 16 ? 16 : units >= 8 ? 8 : units >= 4 ? 4 : 2;
        const int rpw = 32 / gs, ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        XUnit x;
        if (active) load_xunit<QW>(x, ad1, ad2, ad3, asc, ug);
        for (int t = warp * rpw * 2; t < nor; t += kACWarps * rpw * 2) {
            const int ra = t + grp, rc = t + rpw + grp;
            float va = 0.f, vc = 0.f;
            if (ok && active) {
                if (ra < nor) va = unit_dot<QW>(wbuf + static_cast<size_t>(ra) * blk_o, ug, x);
                if (rc < nor) vc = unit_dot<QW>(wbuf + static_cast<size_t>(rc) * blk_o, ug, x);
            }
            __syncwarp();
            for (int o = gs >> 1; o; o >>= 1) {
                va += __shfl_xor_sync(0xffffffffu, va, o);
                vc += __shfl_xor_sync(0xffffffffu, vc, o);
            }
            if (ug == 0 && ra < nor) so[ra] = va;
            if (ug == 0 && rc < nor) so[rc] = vc;
        }
    }
    __syncthreads();
    for (int t = tid; t < nor; t += kAC) __stcg(p.opart + static_cast<size_t>(j) * H + o0 + t, so[t]);
    __syncthreads();
    if (tid == 0) {
        __threadfence();   // the block's share before its count
        const unsigned old = atomicAdd(p.cnt + r * kCntStride, 1u);
        const int last = old == static_cast<unsigned>(p.n_kv - 1);
        if (last) {
            p.cnt[r * kCntStride] = 0u;   // the next launch starts after this grid ends
            __threadfence();              // the other clusters' shares before the reads below
        }
        hd.last = last;
    }
    __syncthreads();
    if (hd.last)
        for (int t = tid; t < nor; t += kAC) {
            float v = 0.f;
            for (int jj = 0; jj < p.n_kv; jj++) v += jj == j ? so[t] : __ldcg(p.opart + static_cast<size_t>(jj) * H + o0 + t);
            p.x[o0 + t] = __ldcg(p.x + o0 + t) + v;
        }
    AC_STAMP(8);
#undef AC_STAMP
    // no bulk copy in flight at exit (complete above on the normal path)
    if (tid == 0 && !ok) mbar_wait(&hd.bar, 0, p.err, kErrWaitFull);
}

// the opt-in shared-memory size and the non-portable cluster sizes, once per
// kernel and device
template <class Kern>
cudaError_t prepare(Kern kern) {
    struct Done {
        const void *kern;
        int dev;
    };
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::vector<Done> done;
    const void *kp = reinterpret_cast<const void *>(kern);
    std::lock_guard<std::mutex> lock(mu);
    for (const Done &d : done)
        if (d.kern == kp && d.dev == dev) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.push_back(Done{kp, dev});
    return cudaSuccess;
}

void fill_cfg(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *at, int n_clusters, int C, uint32_t smem,
              cudaStream_t st) {
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3(static_cast<unsigned>(n_clusters * C));
    cfg.blockDim = dim3(kAC);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = static_cast<unsigned>(C);
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
}

template <int QW, int QV>
cudaError_t launch_one(const AttnClusterArgs &a, uint32_t smem, cudaStream_t st) {
    cudaError_t e = prepare(k_attn_cluster<QW, QV>);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[2];
    fill_cfg(cfg, at, a.n_kv, a.C, smem, st);
    return cudaLaunchKernelEx(&cfg, k_attn_cluster<QW, QV>, a);
}

// clusters of C CTAs with `smem` bytes each that the device holds at once;
// queried once per (kernel, device, C, smem) and cached
template <int QW, int QV>
int max_active(int C, uint32_t smem) {
    struct Fit {
        const void *kern;
        int dev, C;
        uint32_t smem;
        int n;
    };
    static std::mutex mu;
    static std::vector<Fit> fits;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const void *kp = reinterpret_cast<const void *>(k_attn_cluster<QW, QV>);
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Fit &f : fits)
            if (f.kern == kp && f.dev == dev && f.C == C && f.smem == smem) return f.n;
    }
    if (prepare(k_attn_cluster<QW, QV>) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[2];
    fill_cfg(cfg, at, 1, C, smem, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_attn_cluster<QW, QV>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    fits.push_back(Fit{kp, dev, C, smem, n});
    return n;
}

}  // namespace

#define STYX_AC_CASES(X)     \
    X(STYX_Q4_K, STYX_Q6_K)  \
    X(STYX_Q4_K, STYX_Q4_K)  \
    X(STYX_Q8_0, STYX_Q8_0)  \
    X(STYX_Q5_K, STYX_Q6_K)  \
    X(STYX_Q5_K, STYX_Q5_K)

bool attn_cluster_supported(int qw, int qv) {
#define STYX_AC_CASE(W_, V_) \
    if (qw == W_ && qv == V_) return true;
    STYX_AC_CASES(STYX_AC_CASE)
#undef STYX_AC_CASE
    return false;
}

int attn_cluster_max_active(int qw, int qv, int C, uint32_t smem) {
#define STYX_AC_CASE(W_, V_) \
    if (qw == W_ && qv == V_) return max_active<W_, V_>(C, smem);
    STYX_AC_CASES(STYX_AC_CASE)
#undef STYX_AC_CASE
    return 0;
}

cudaError_t launch_attn_cluster(const AttnClusterArgs &a, int qw, int qv, uint32_t smem, cudaStream_t st) {
#define STYX_AC_CASE(W_, V_) \
    if (qw == W_ && qv == V_) return launch_one<W_, V_>(a, smem, st);
    STYX_AC_CASES(STYX_AC_CASE)
#undef STYX_AC_CASE
    return cudaErrorNotSupported;
}

}  // namespace styx
