// moe_cluster.cu -- the whole MoE block of one layer as one launch of
// thread-block clusters: one cluster of C CTAs (C <= 16) per selected slot.
//
// Nothing waits across clusters.  Every cluster routes the token itself (the
// same code on the same data gives every cluster the same ids), the h vector
// of slot s never leaves the cluster that computes it, and the combine of the
// k slots is done by whichever CTA finishes a row block last.  So the launch
// needs no co-residency guarantee and no cooperative launch, and the only
// waits are the cluster's own barriers and the bulk copies' mbarriers.
//
// Phases of CTA r of cluster s (512 threads, one CTA per SM):
//   0  mbarriers; one bulk copy of the CTA's router rows e in [E r/C,
//      E (r+1)/C) into shared memory and the norm weights into registers --
//      model weights, not written by any kernel, read before the grid
//      dependency resolves; the next kernel may launch (PDL); wait for the
//      previous grid;
//   1  x and the remap / pmap tables; RMSNorm; the router dot products of
//      the CTA's rows (the tree sums of the single kernel, so the logits are
//      the same bits); each logit is stored into every CTA of the cluster
//      (st.shared::cluster) and one cluster barrier later every CTA holds
//      all E logits;
//   2  top-k by rank (the selection of topk_softmax_f32.comp:39-46); warp 0
//      resolves slot s's slabs and issues the bulk copies of the CTA's
//      gate/up rows [F r/C, F (r+1)/C) (in chunks) and down rows
//      [H r/C, H (r+1)/C) (into the router rows' space); meanwhile every
//      warp turns x_norm into dp4a digits and warp 1 computes the softmax
//      weights;
//   3  gate/up dot products as the chunks land, SiLU(g) * u -> h
//      (ops2.rs:305-308); each h value is stored into every CTA of the
//      cluster; one cluster barrier;
//   4  h -> digits; the CTA's down rows of slot s;
//   5  the rows go to the workspace (or, for expert parallelism, w[s] times
//      them to the caller's partial buffer); the CTA that completes a row
//      block last among the k clusters (one counter per block, reset to 0 by
//      that CTA) adds the slots in slot order, x[r] += sum_s w[s] d[s][r]
//      (moe_reduce_f32.comp:8-13).
// The arithmetic of every value is the single kernel's (moe_fused.cu): the
// same reduction trees, digit vectors and dot products, so both forms give
// the same bits.
#include <cfloat>
#include <mutex>
#include <vector>

#include "cluster.cuh"
#include "common.cuh"
#include "kernels.h"
#include "moe_common.cuh"
#include "qdot.cuh"

namespace styx {

namespace {

constexpr int kBarRouter = 0, kBarGu = 1, kBarDown = 9, kNumBars = 10;   // gate/up chunks: at most 8

struct ClHdr {
    uint64_t bar[16];
    float red[9 * kFusedWarps];   // per warp: up to 8 router partial sums, then sum(x^2)
    float wts[16];                // softmax weights in slot order (the picked logits until then)
    uint32_t pkey[16];            // key of pick s
    int pid[16];                  // expert of slot s (-1: empty)
    const uint8_t *src[3];        // slot s's gate, up, down slab
    int last;                     // this CTA completes its row block
};
static_assert(sizeof(ClHdr) <= kClusterHeader, "cluster kernel header overflows");

template <int QG, int QD>
__global__ void __launch_bounds__(kFusedBlock, 1) k_moe_cluster(const __grid_constant__ ClusterArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    ClHdr &hd = *reinterpret_cast<ClHdr *>(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = p.C, H = p.H, F = p.F, E = p.E, k = p.k;
    const int s = blockIdx.x / C;                    // the cluster's slot
    const int r = static_cast<int>(cluster_ctarank());   // this CTA's rank in the cluster
    const bool lead = blockIdx.x == 0;               // writes the id block and the debug views
    float *lg = reinterpret_cast<float *>(smem + p.off_lg);
    uint32_t *key = reinterpret_cast<uint32_t *>(lg + E);
    int *rnk = reinterpret_cast<int *>(key + E);
    uint32_t *sremap = reinterpret_cast<uint32_t *>(rnk + E);
    uint32_t *spmap = sremap + E;
    float *xv = reinterpret_cast<float *>(smem + p.off_x);
    int8_t *xd1 = reinterpret_cast<int8_t *>(smem + p.off_xd);
    uint8_t *xd2 = reinterpret_cast<uint8_t *>(xd1) + H;
    uint8_t *xd3 = xd2 + H;
    float *xsc = reinterpret_cast<float *>(xd3 + H);
    float *hf = reinterpret_cast<float *>(smem + p.off_hf);
    int8_t *hd1 = reinterpret_cast<int8_t *>(smem + p.off_hd);
    uint8_t *hd2 = reinterpret_cast<uint8_t *>(hd1) + F;
    uint8_t *hd3 = hd2 + F;
    float *hsc = reinterpret_cast<float *>(hd3 + F);
    float *yl = reinterpret_cast<float *>(smem + p.off_y);
    uint8_t *gubuf = smem + p.off_gu;
    uint8_t *dnbuf = smem + p.off_dn;   // the router rows, then the down rows

    const int e0 = E * r / C, nr = E * (r + 1) / C - e0;    // router rows
    const int g0 = F * r / C, ngr = F * (r + 1) / C - g0;   // gate/up rows
    const int d0 = H * r / C, ndr = H * (r + 1) / C - d0;   // down rows
    const int H4 = H >> 2;

#define STYX_CSTAMP(i_)                                                                    \
    do {                                                                                   \
        if (tid == 0 && p.trace) p.trace[blockIdx.x * kTraceStamps + (i_)] = clock64();   \
    } while (0)
    STYX_CSTAMP(0);
    // ------------------------------------------------ phase 0
    if (tid == 0) {
        for (int i = 0; i < kNumBars; i++) mbar_init(&hd.bar[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && nr > 0) {
        const uint32_t bytes = static_cast<uint32_t>(nr) * static_cast<uint32_t>(H) * 4u;
        mbar_arrive_expect_tx(&hd.bar[kBarRouter], bytes);
        bulk_g2s_hint(dnbuf, p.router + static_cast<size_t>(e0) * H, bytes, &hd.bar[kBarRouter], l2_evict_last());
    }
    float4 wn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H4) wn = __ldg(reinterpret_cast<const float4 *>(p.norm_w) + tid);
    cl_arrive_relaxed();   // this CTA runs: its shared memory may receive logits once all have arrived
    pdl_trigger();
    pdl_wait();
    STYX_CSTAMP(1);

    // ------------------------------------------------ phase 1: RMSNorm + router
    float4 xr = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H4) xr = __ldcg(reinterpret_cast<const float4 *>(p.x) + tid);
    for (int i = tid; i < E; i += kFusedBlock) {
        sremap[i] = p.remap ? __ldg(p.remap + i) : kSkip;
        spmap[i] = p.pmap ? __ldg(p.pmap + i) : kSkip;
    }
    float ss = 0.f;
    ss += xr.x * xr.x + xr.y * xr.y + xr.z * xr.z + xr.w * xr.w;
    bool rok = true;
    if (nr > 0) rok = mbar_wait(&hd.bar[kBarRouter], 0, p.err, kErrWaitFull);
    cl_wait();   // every CTA of the cluster runs
    STYX_CSTAMP(2);
    const float *rrows = reinterpret_cast<const float *>(dnbuf);
    const uint32_t lg_s = smem_addr(lg);
    float scale = 0.f;
    for (int jb = 0; jb == 0 || jb < nr; jb += 8) {
        const int nb = min(nr - jb, 8);
        float part[9];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            part[j] = 0.f;
            if (j < nb && tid < H4 && rok)
                part[j] = rwx4(reinterpret_cast<const float4 *>(rrows + static_cast<size_t>(jb + j) * H)[tid], wn, xr);
        }
        part[8] = jb == 0 ? ss : 0.f;
#pragma unroll
        for (int o = 16; o; o >>= 1)
#pragma unroll
            for (int j = 0; j < 9; j++) part[j] += __shfl_xor_sync(0xffffffffu, part[j], o);
        if (jb) __syncthreads();   // the previous pass is done with red
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 9; j++) hd.red[j * kFusedWarps + warp] = part[j];
        }
        __syncthreads();
        if (jb == 0) {
            float t = lane < kFusedWarps ? hd.red[8 * kFusedWarps + lane] : 0.f;
#pragma unroll
            for (int o = 8; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            scale = 1.0f / sqrtf(__shfl_sync(0xffffffffu, t, 0) / static_cast<float>(H) + p.eps);
        }
        if (warp < nb) {   // row jb + warp: its logit into every CTA of the cluster
            float t = lane < kFusedWarps ? hd.red[warp * kFusedWarps + lane] : 0.f;
#pragma unroll
            for (int o = 8; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            const float acc = scale * __shfl_sync(0xffffffffu, t, 0);
            const uint32_t a = lg_s + static_cast<uint32_t>(e0 + jb + warp) * 4u;
            for (int q = lane; q < C; q += 32) cl_st(cl_map(a, static_cast<uint32_t>(q)), acc);
        }
    }
    fence_proxy_async_cta();   // the router rows are read: their space may take bulk copies
    if (tid < H4) {
        float4 v = xr;
        v.x = v.x * scale * wn.x;
        v.y = v.y * scale * wn.y;
        v.z = v.z * scale * wn.z;
        v.w = v.w * scale * wn.w;
        reinterpret_cast<float4 *>(xv)[tid] = v;
        if (lead) reinterpret_cast<float4 *>(p.xnorm)[tid] = v;   // debug view
    }
    cl_arrive();
    cl_wait();   // every logit stored in every CTA; x_norm complete
    STYX_CSTAMP(3);

    // ------------------------------------------------ phase 2: top-k, copies, digits
    for (int i = tid; i < E; i += kFusedBlock) {
        const float v = lg[i];
        key[i] = v > -INFINITY ? order_key(v) : 0u;   // 0: never picked (-inf, NaN)
        rnk[i] = 0;
    }
    if (tid < 16) hd.pid[tid] = -1;
    __syncthreads();
    {   // rank of element i = eligible elements ahead of it: larger key, or the same key and a lower index
        const int P = E <= 128 ? 4 : (E <= 256 ? 2 : 1);
        for (int t = tid; t < E * P; t += kFusedBlock) {
            const int i = t % E, part = t / E;
            const uint32_t ki = key[i];
            if (!ki) continue;
            const int jlo = E * part / P, jhi = E * (part + 1) / P;
            int c = 0;
            for (int j = jlo; j < jhi; j++) {
                const uint32_t kj = key[j];
                c += (kj > ki) || (kj == ki && j < i);
            }
            atomicAdd(&rnk[i], c);
        }
    }
    __syncthreads();
    for (int i = tid; i < E; i += kFusedBlock)
        if (key[i] && rnk[i] < k) {
            hd.pid[rnk[i]] = i;
            hd.pkey[rnk[i]] = key[i];
        }
    __syncthreads();
    STYX_CSTAMP(4);
    if (warp == 0) {   // slot s: its slabs and every byte of them this CTA needs
        const int e = hd.pid[s];
        int hi = -1, ai = -1, fi = -1;
        if (e >= 0) {
            const uint32_t hot = sremap[e];
            if (hot != kSkip) {
                hi = static_cast<int>(hot);
            } else {
                const uint32_t am = spmap[e];
                if (am != kSkip) ai = static_cast<int>(am);
                else fi = e;
            }
        }
        const uint8_t *sg = fused_slot_src(p.gate, hi, ai, fi);
        const uint8_t *su = fused_slot_src(p.up, hi, ai, fi);
        const uint8_t *sd = fused_slot_src(p.down, hi, ai, fi);
        if (lane == 0) {
            hd.src[0] = sg;
            hd.src[1] = su;
            hd.src[2] = sd;
        }
        const uint64_t once = l2_evict_first();   // expert bytes are read once per token
        if (lane < p.ng) {   // gate/up chunk `lane`: its gate rows, then its up rows
            const int q0 = lane * p.chg, n = min(p.chg, ngr - q0);
            uintptr_t ag = 0, au = 0;
            uint32_t lgn = 0, lun = 0;
            if (n > 0 && sg && su) {
                cover16(sg + static_cast<size_t>(g0 + q0) * p.rb_g, static_cast<size_t>(n) * p.rb_g, ag, lgn);
                cover16(su + static_cast<size_t>(g0 + q0) * p.rb_u, static_cast<size_t>(n) * p.rb_u, au, lun);
            }
            uint64_t *bar = &hd.bar[kBarGu + lane];
            if (lgn + lun == 0) {
                mbar_arrive(bar);
            } else {
                uint8_t *cb = gubuf + static_cast<size_t>(lane) * p.gu_stride;
                mbar_arrive_expect_tx(bar, lgn + lun);
                bulk_g2s_hint(cb, reinterpret_cast<const void *>(ag), lgn, bar, once);
                bulk_g2s_hint(cb + p.gu_up_off, reinterpret_cast<const void *>(au), lun, bar, once);
            }
        } else if (lane == p.ng) {   // the CTA's down rows, one copy
            uintptr_t a = 0;
            uint32_t len = 0;
            if (sd && ndr > 0) cover16(sd + static_cast<size_t>(d0) * p.rb_d, static_cast<size_t>(ndr) * p.rb_d, a, len);
            uint64_t *bar = &hd.bar[kBarDown];
            if (len == 0) {
                mbar_arrive(bar);
            } else {
                mbar_arrive_expect_tx(bar, len);
                bulk_g2s_hint(dnbuf, reinterpret_cast<const void *>(a), len, bar, once);
            }
        }
        __syncwarp();
    } else if (warp == 1 && lead) {   // the id block: expert, hot index, arena slot, full id of every slot
        const int e = lane < k ? hd.pid[lane] : -1;
        if (lane < k) {
            int hi = -1, ai = -1, fi = -1;
            if (e >= 0) {
                const uint32_t hot = sremap[e];
                if (hot != kSkip) {
                    hi = static_cast<int>(hot);
                } else {
                    const uint32_t am = spmap[e];
                    if (am != kSkip) ai = static_cast<int>(am);
                    else fi = e;
                }
                if (!p.quiet && (!fused_slot_src(p.gate, hi, ai, fi) || !fused_slot_src(p.up, hi, ai, fi) ||
                                 !fused_slot_src(p.down, hi, ai, fi)))
                    atomicExch(p.err, kErrBadId);
            }
            p.ids64[lane] = e;
            p.ids64[16 + lane] = hi;
            p.ids64[32 + lane] = ai;
            p.ids64[48 + lane] = fi;
        }
    }
    STYX_CSTAMP(5);
    {   // x_norm -> digits, four groups' shuffle chains together
        const DigitsView dv{xd1, xd2, xd3, xsc};
        for (int gb = warp; gb < (H >> 5); gb += 4 * kFusedWarps) {
            float v[4];
            int gi[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int g = gb + j * kFusedWarps;
                gi[j] = g < (H >> 5) ? g : -1;
                v[j] = g < (H >> 5) ? xv[g * 32 + lane] : 0.f;
            }
            digits_groups_warp<4>(v, gi, lane, dv);
        }
    }
    if (warp == 1) {
        // softmax statistics over all E logits (lane-strided partials, fixed
        // shuffle tree) and the weights in slot order (topk_softmax_f32.comp:47-52)
        float mx = -INFINITY, sum = 0.f;
        for (int i = lane; i < E; i += 32) mx = fmaxf(mx, lg[i]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (int i = lane; i < E; i += 32) sum += expf(lg[i] - mx);
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float lsel = (lane < k && hd.pid[lane] >= 0) ? key_value(hd.pkey[lane]) : -INFINITY;
        const float w = lane < k ? expf(lsel - mx) / sum : 0.f;
        float wsum = 0.f;
        for (int t = 0; t < k; t++) wsum += __shfl_sync(0xffffffffu, w, t);
        if (lane < k) {
            const float wr = p.renorm ? w / wsum : w;
            hd.wts[lane] = wr;
            if (lead) p.weights[lane] = wr;
        }
    }
    if (lead)
        for (int i = tid; i < E; i += kFusedBlock) p.logits[i] = lg[i];   // debug view
    __syncthreads();   // digits, weights and slab sources visible
    STYX_CSTAMP(6);

    // ------------------------------------------------ phase 3: gate/up -> h
    bool ok = true;
    {
        const uint8_t *sg = hd.src[0], *su = hd.src[1];
        const int units = p.units_g, gs = p.gs_g, rpw = 32 / gs, stride = kFusedWarps * rpw;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        XUnit xu;
        if (active) load_xunit<QG>(xu, xd1, xd2, xd3, xsc, ug);
        const uint32_t hf_s = smem_addr(hf);
        int waited = -1;
        bool first = true;
        for (int qb = warp * rpw; qb < ngr; qb += stride) {
            const int q = qb + grp;
            const int ci = qb / p.chg;   // chg % rpw == 0: the warp's rows share a chunk
            if (ci != waited) {
                if (ok) ok = mbar_wait(&hd.bar[kBarGu + ci], 0, p.err, kErrWaitFull);
                waited = ci;
            }
            if (first) {
                STYX_CSTAMP(7);
                first = false;
            }
            float g = 0.f, u = 0.f;
            if (q < ngr && ok && sg && su && active) {
                const int t = q - ci * p.chg;
                const size_t row0 = static_cast<size_t>(g0 + ci * p.chg);
                const uint8_t *cb = gubuf + static_cast<size_t>(ci) * p.gu_stride;
                const uint8_t *gb = cb + (reinterpret_cast<uintptr_t>(sg + row0 * p.rb_g) & 15) +
                                    static_cast<size_t>(t) * p.rb_g;
                const uint8_t *ub = cb + p.gu_up_off + (reinterpret_cast<uintptr_t>(su + row0 * p.rb_u) & 15) +
                                    static_cast<size_t>(t) * p.rb_u;
                g = unit_dot<QG>(gb, ug, xu);
                u = unit_dot<QG>(ub, ug, xu);
            }
            __syncwarp();   // regroup the lanes after the waits and branches above
            for (int o = gs >> 1; o; o >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, o);
                u += __shfl_xor_sync(0xffffffffu, u, o);
            }
            // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
            const float hv = g / (1.0f + expf(-g)) * u;
            if (q < ngr) {
                const uint32_t a = hf_s + static_cast<uint32_t>(g0 + q) * 4u;
                for (int dst = ug; dst < C; dst += gs) cl_st(cl_map(a, static_cast<uint32_t>(dst)), hv);
                if (ug == 0 && p.h) __stcg(p.h + static_cast<size_t>(s) * F + g0 + q, hv);   // debug view
            }
        }
    }
    STYX_CSTAMP(8);
    cl_arrive();
    cl_wait();   // slot s's h complete in every CTA of the cluster
    STYX_CSTAMP(9);

    // ------------------------------------------------ phase 4: down rows of slot s
    {
        const int nparts = F >> 4, lim = ((nparts + 31) >> 5) << 5;
        for (int pidx = tid; pidx < lim; pidx += kFusedBlock) {
            const bool on = pidx < nparts;
            float v[16];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 q = on ? reinterpret_cast<const float4 *>(hf)[pidx * 4 + i] : make_float4(0.f, 0.f, 0.f, 0.f);
                v[4 * i] = q.x;
                v[4 * i + 1] = q.y;
                v[4 * i + 2] = q.z;
                v[4 * i + 3] = q.w;
            }
            digits_part<16>(v, on, pidx, hd1, hd2, hd3, hsc);
        }
    }
    __syncthreads();
    {
        const uint8_t *sd = hd.src[2];
        const int units = p.units_d, gs = p.gs_d, rpw = 32 / gs;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        XUnit xu;
        if (active) load_xunit<QD>(xu, hd1, hd2, hd3, hsc, ug);
        if (ok) ok = mbar_wait(&hd.bar[kBarDown], 0, p.err, kErrWaitFull);
        STYX_CSTAMP(10);
        const uint8_t *base = dnbuf + (sd ? (reinterpret_cast<uintptr_t>(sd + static_cast<size_t>(d0) * p.rb_d) & 15) : 0);
        // two rows per lane group per pass: independent dot products in flight
        for (int t = warp * 2 * rpw; t < ndr; t += kFusedWarps * 2 * rpw) {
            const int ra = t + grp, rb = t + rpw + grp;
            float va = 0.f, vb = 0.f;
            if (ok && sd && active && ra < ndr) va = unit_dot<QD>(base + static_cast<size_t>(ra) * p.rb_d, ug, xu);
            if (ok && sd && active && rb < ndr) vb = unit_dot<QD>(base + static_cast<size_t>(rb) * p.rb_d, ug, xu);
            __syncwarp();
            for (int o = gs >> 1; o; o >>= 1) {
                va += __shfl_xor_sync(0xffffffffu, va, o);
                vb += __shfl_xor_sync(0xffffffffu, vb, o);
            }
            if (ug == 0 && ra < ndr) yl[ra] = va;
            if (ug == 0 && rb < ndr) yl[rb] = vb;
        }
    }
    __syncthreads();
    STYX_CSTAMP(11);

    // ------------------------------------------------ phase 5: combine
    if (p.partial) {
        // expert parallelism: slot s's weighted rows; the ranks' sum (one
        // non-zero contributor per slot) then goes through the combine
        for (int t = tid; t < ndr; t += kFusedBlock)
            p.partial[static_cast<size_t>(s) * H + d0 + t] = __fmul_rn(hd.wts[s], yl[t]);
    } else {
        for (int t = tid; t < ndr; t += kFusedBlock) __stcg(p.y + static_cast<size_t>(s) * H + d0 + t, yl[t]);
        __syncthreads();
        if (tid == 0) {
            __threadfence();   // the block's rows before its count
            const unsigned old = atomicAdd(p.cnt + r * kCntStride, 1u);
            const int last = old == static_cast<unsigned>(k - 1);
            if (last) {
                p.cnt[r * kCntStride] = 0u;   // the next launch starts after this grid ends
                __threadfence();              // the other clusters' rows before the reads below
            }
            hd.last = last;
        }
        __syncthreads();
        if (hd.last) {
            for (int t = tid; t < ndr; t += kFusedBlock) {
                float acc = 0.f;
                for (int j = 0; j < k; j++) {
                    const float d = j == s ? yl[t] : __ldcg(p.y + static_cast<size_t>(j) * H + d0 + t);
                    acc = __fadd_rn(acc, __fmul_rn(hd.wts[j], d));
                }
                p.x[d0 + t] = __fadd_rn(__ldcg(p.x + d0 + t), acc);
            }
        }
    }
    STYX_CSTAMP(12);
    // No CTA leaves with copies in flight into its shared memory, even after
    // a wait above gave up (bounded).
    if (tid == 0) {
        bool fine = true;
        for (int c = 0; c < p.ng && fine; c++) fine = mbar_wait(&hd.bar[kBarGu + c], 0, p.err, kErrWaitFull);
        if (fine) mbar_wait(&hd.bar[kBarDown], 0, p.err, kErrWaitFull);
    }
#undef STYX_CSTAMP
}

struct AttrDone {
    const void *kern;
    int dev;
};

// the opt-in shared-memory size and the non-portable cluster sizes, once per
// kernel and device
template <class Kern>
cudaError_t prepare(Kern kern) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::vector<AttrDone> done;
    const void *kp = reinterpret_cast<const void *>(kern);
    std::lock_guard<std::mutex> lock(mu);
    for (const AttrDone &d : done)
        if (d.kern == kp && d.dev == dev) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.push_back(AttrDone{kp, dev});
    return cudaSuccess;
}

void fill_cfg(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *at, int k, int C, uint32_t smem, cudaStream_t st) {
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3(static_cast<unsigned>(k * C));
    cfg.blockDim = dim3(kFusedBlock);
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

template <int QG, int QD>
cudaError_t launch_one(const ClusterArgs &a, uint32_t smem, cudaStream_t st) {
    cudaError_t e = prepare(k_moe_cluster<QG, QD>);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[2];
    fill_cfg(cfg, at, a.k, a.C, smem, st);
    return cudaLaunchKernelEx(&cfg, k_moe_cluster<QG, QD>, a);
}

// clusters of C CTAs with `smem` bytes each that the device holds at once;
// queried once per (kernel, device, C, smem) and cached
template <int QG, int QD>
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
    const void *kp = reinterpret_cast<const void *>(k_moe_cluster<QG, QD>);
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Fit &f : fits)
            if (f.kern == kp && f.dev == dev && f.C == C && f.smem == smem) return f.n;
    }
    if (prepare(k_moe_cluster<QG, QD>) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[2];
    fill_cfg(cfg, at, 1, C, smem, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_moe_cluster<QG, QD>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    fits.push_back(Fit{kp, dev, C, smem, n});
    return n;
}

}  // namespace

#define STYX_CLUSTER_CASES(X)          \
    X(STYX_Q4_K, STYX_Q6_K)            \
    X(STYX_Q4_K, STYX_Q4_K)            \
    X(STYX_Q5_K, STYX_Q6_K)            \
    X(STYX_Q5_K, STYX_Q5_K)            \
    X(STYX_Q8_0, STYX_Q8_0)            \
    X(STYX_Q6_K, STYX_Q6_K)

cudaError_t launch_cluster(const ClusterArgs &a, int qg, int qd, uint32_t smem, cudaStream_t st) {
#define STYX_CL_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return launch_one<G_, D_>(a, smem, st);
    STYX_CLUSTER_CASES(STYX_CL_CASE)
#undef STYX_CL_CASE
    return cudaErrorNotSupported;
}

int cluster_max_active(int qg, int qd, int C, uint32_t smem) {
#define STYX_CL_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return max_active<G_, D_>(C, smem);
    STYX_CLUSTER_CASES(STYX_CL_CASE)
#undef STYX_CL_CASE
    return 0;
}

bool cluster_supported(int qg, int qd) { return fused_supported(qg, qd); }

}  // namespace styx
