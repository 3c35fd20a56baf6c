// moe_kernels.cu -- sm_100a kernels of the Qwen3-MoE block.
//
//   k_route      RMSNorm(x) -> router GEMV (one CTA per expert row) -> the
//                last CTA to finish runs softmax + top-k, writes the id rows,
//                and emits x_norm as dp4a digits for the expert kernels.
//   k_gate_up    per selected expert: gate and up rows streamed HBM -> shared
//                memory by 1-D bulk copies (TMA) through an mbarrier ring,
//                decoded in registers, dot products on dp4a, SiLU(g)*u.
//   k_down       output rows of all k slots streamed the same way; down dot
//                products against h (digits built per CTA in shared memory),
//                then the slot-ordered weighted combine into the residual.
//   k_matvec_id  the generic expert-indexed GEMV (MatVecIdPush semantics).
//
// Reference semantics: crates/model/src/moe.rs:1974-2062 and the shaders
// named beside each kernel.
#include <cfloat>

#include "common.cuh"
#include "kernels.h"
#include "ep_sync.cuh"
#include "qdot.cuh"

namespace styx {

// Source slab of slot s: hot row, then arena row, then full-tensor row (the
// three-way split of rec_matvec_id, moe.rs:1649-1700).  An index outside its
// source is skipped (nullptr) and reported; `report` is false on re-reads.
// With `quiet`, a full-tensor fallback with no full tensor (an expert another
// device holds, expert parallelism) is skipped without a report.
__device__ __forceinline__ const uint8_t *slot_src(const ExpSrc &t, const int32_t *ids64, int s, int *err,
                                                   bool report, bool quiet = false) {
    const uint32_t h = static_cast<uint32_t>(ids64[16 + s]);
    const uint32_t a = static_cast<uint32_t>(ids64[32 + s]);
    const uint32_t g = static_cast<uint32_t>(ids64[48 + s]);
    const uint8_t *p = nullptr;
    bool bad = false;
    if (h != kSkip) {
        if (t.hot && h < t.nhot) p = t.hot + static_cast<uint64_t>(h) * t.slab;
        else bad = true;
    } else if (a != kSkip) {
        if (t.arena && a < t.narena) p = t.arena + static_cast<uint64_t>(a) * t.aslab;
        else bad = true;
    } else if (g != kSkip) {
        if (t.full && g < t.nfull) p = t.full + static_cast<uint64_t>(g) * t.slab;
        else bad = t.full || !quiet;
    }
    if (bad && report && err) atomicExch(err, kErrBadId);
    return p;
}

// deterministic 256-thread reductions (fixed tree)
__device__ __forceinline__ float block_sum256(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < 8 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 4; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return __shfl_sync(0xffffffffu, t, 0);
}

__device__ __forceinline__ float block_max256(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < 8 ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 4; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    return __shfl_sync(0xffffffffu, t, 0);
}

// ----------------------------------------------------------- top-k
// shaders/topk_softmax_f32.comp:29-67 by ranks instead of k serial scans:
// element i (finite or +inf, i.e. > -inf) gets rank #{j: l_j > l_i} +
// #{j < i: l_j == l_i}; the serial scan's s-th pick (strict '>', first index
// wins ties, -inf/NaN never picked) is exactly the element of rank s.
// Softmax normaliser over all n; weights in selection order, optionally
// renormalised.  Called by all 256 threads; lg in shared memory.
__device__ void topk_block(const float *lg, int n, int k, int renorm, const uint32_t *remap,
                           const uint32_t *pmap, float *weights, int32_t *ids64, float *red,
                           int *sel) {
    const int tid = threadIdx.x;
    float m = -INFINITY;
    for (int i = tid; i < n; i += 256) m = fmaxf(m, lg[i]);
    const float mx = block_max256(m, red);
    float se = 0.f;
    for (int i = tid; i < n; i += 256) se += expf(lg[i] - mx);
    const float sum = block_sum256(se, red);
    if (tid < 16) sel[tid] = -1;
    __syncthreads();
    for (int i = tid; i < n; i += 256) {
        const float v = lg[i];
        if (v > -INFINITY) {
            int r = 0;
            for (int j = 0; j < n; j++) {
                const float u = lg[j];
                r += (u > v) | ((u == v) & (j < i));
            }
            if (r < k) sel[r] = i;
        }
    }
    __syncthreads();
    if (tid == 0) {
        float picked[16];
        float wsum = 0.f;
        for (int s = 0; s < k; s++) {
            const float best = sel[s] >= 0 ? lg[sel[s]] : -INFINITY;
            const float w = expf(best - mx) / sum;
            picked[s] = w;
            wsum += w;
        }
        for (int s = 0; s < k; s++) {
            weights[s] = renorm ? picked[s] / wsum : picked[s];
            const int e = sel[s];
            ids64[s] = e;
            const uint32_t hot = (e >= 0 && remap) ? remap[e] : kSkip;
            if (hot != kSkip) {
                ids64[16 + s] = static_cast<int32_t>(hot);
                ids64[32 + s] = -1;
                ids64[48 + s] = -1;
            } else {
                const uint32_t a = (e >= 0 && pmap) ? pmap[e] : kSkip;
                ids64[16 + s] = -1;
                ids64[32 + s] = a != kSkip ? static_cast<int32_t>(a) : -1;
                ids64[48 + s] = a != kSkip ? -1 : e;
            }
        }
    }
}

// ----------------------------------------------------------- route
__global__ void __launch_bounds__(256) k_route(const RouteArgs p) {
    extern __shared__ float xn[];   // H floats
    __shared__ float red[32];
    __shared__ float lg[STYX_MAX_EXPERTS];
    __shared__ int sel[16];
    __shared__ int s_last;
    const int tid = threadIdx.x, e = blockIdx.x;

    // RMSNorm (kernels.rs:58-67 with the ffn_norm multiply); every CTA
    // computes the same values in the same order
    float ss = 0.f;
    for (int c = tid; c < p.H; c += 256) {
        const float v = p.x[c];
        ss += v * v;
    }
    ss = block_sum256(ss, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(p.H) + p.eps);
    for (int c = tid; c < p.H; c += 256) {
        const float v = p.x[c] * scale;
        xn[c] = p.norm_w ? v * p.norm_w[c] : v;
    }
    __syncthreads();

    // logits[e] = router[e] . xnorm  (matvec_strided_f32.comp)
    const float4 *R = reinterpret_cast<const float4 *>(p.router + static_cast<size_t>(e) * p.H);
    float acc = 0.f;
    for (int c4 = tid; c4 < (p.H >> 2); c4 += 256) {
        const float4 r = __ldg(R + c4);
        const float4 v = reinterpret_cast<const float4 *>(xn)[c4];
        acc += r.x * v.x + r.y * v.y + r.z * v.z + r.w * v.w;
    }
    acc = block_sum256(acc, red);
    if (tid == 0) {
        p.logits[e] = acc;
        __threadfence();
        s_last = (atomicAdd(p.counter, 1u) == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // last CTA: softmax + top-k + id rows, x_norm and its digits
    for (int i = tid; i < p.E; i += 256) lg[i] = __ldcg(p.logits + i);
    __syncthreads();
    topk_block(lg, p.E, p.k, p.renorm, p.remap, p.pmap, p.weights, p.ids64, red, sel);
    for (int c = tid; c < p.H; c += 256) p.xnorm[c] = xn[c];
    const int warp = tid >> 5, lane = tid & 31;
    const DigitsView dv{p.xd1, p.xd2, p.xd3, p.xscale};
    for (int g = warp; g < (p.H >> 5); g += 8) digits_group_warp(xn[g * 32 + lane], lane, dv, g);
    if (tid == 0) *p.counter = 0u;
}

cudaError_t launch_route(const RouteArgs &a, cudaStream_t st) {
    const size_t smem = static_cast<size_t>(a.H) * sizeof(float);
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(k_route, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        attr_done = true;
    }
    k_route<<<a.E, 256, smem, st>>>(a);
    return cudaGetLastError();
}

// --------------------------------------------------------- gate / up
// One producer warp (lane 0 issues the bulk copies) and 8 consumer warps.
// CTA b owns row-pairs [T*b/G, T*(b+1)/G) of the T = k*F (slot, row) pairs;
// a chunk is <= ch consecutive rows of one slot: its gate rows and up rows
// are two contiguous byte ranges, each one bulk copy.
template <int QT>
__global__ void __launch_bounds__(kFusedThreads, 1) k_gate_up(const GateUpArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 16;
    uint8_t *stages = smem + 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long T = static_cast<long long>(p.k) * p.F;
    const int rbeg = static_cast<int>(T * blockIdx.x / gridDim.x);
    const int rend = static_cast<int>(T * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nst; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            int r = rbeg, ci = 0;
            while (r < rend) {
                const int s = r / p.F, rr = r - s * p.F;
                const int n = min(p.ch, min(rend - r, p.F - rr));
                const int st = ci % p.nst;
                if (ci >= p.nst && !mbar_wait(&empty[st], ((ci / p.nst) - 1) & 1, p.err, kErrWaitEmpty))
                    break;
                const uint8_t *gsrc = slot_src(p.gate, p.ids64, s, p.err, true, p.quiet);
                const uint8_t *usrc = slot_src(p.up, p.ids64, s, p.err, true, p.quiet);
                uint8_t *dst = stages + static_cast<size_t>(st) * p.stage_bytes;
                if (gsrc && usrc) {
                    const uintptr_t g0 = reinterpret_cast<uintptr_t>(gsrc + static_cast<size_t>(rr) * p.rb_g);
                    const uintptr_t ga = g0 & ~uintptr_t(15);
                    const uintptr_t gb = (g0 + static_cast<size_t>(n) * p.rb_g + 15) & ~uintptr_t(15);
                    const uintptr_t u0 = reinterpret_cast<uintptr_t>(usrc + static_cast<size_t>(rr) * p.rb_u);
                    const uintptr_t ua = u0 & ~uintptr_t(15);
                    const uintptr_t ub = (u0 + static_cast<size_t>(n) * p.rb_u + 15) & ~uintptr_t(15);
                    mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>((gb - ga) + (ub - ua)));
                    bulk_g2s(dst, reinterpret_cast<const void *>(ga), static_cast<uint32_t>(gb - ga), &full[st]);
                    bulk_g2s(dst + p.up_off, reinterpret_cast<const void *>(ua), static_cast<uint32_t>(ub - ua),
                             &full[st]);
                } else {
                    mbar_arrive(&full[st]);
                }
                r += n;
                ci++;
            }
        }
        return;
    }

    const int cw = warp - 1;
    const int rpw = 32 / p.gs;
    const int ug = lane & (p.gs - 1), grp = lane / p.gs;
    const bool active = ug < p.units;
    XUnit x;
    if (active) load_xunit<QT>(x, p.xd1, p.xd2, p.xd3, p.xscale, ug);

    int r = rbeg, ci = 0;
    while (r < rend) {
        const int s = r / p.F, rr = r - s * p.F;
        const int n = min(p.ch, min(rend - r, p.F - rr));
        const int st = ci % p.nst;
        if (!mbar_wait(&full[st], (ci / p.nst) & 1, p.err, kErrWaitFull)) break;
        const uint8_t *gsrc = slot_src(p.gate, p.ids64, s, p.err, false, p.quiet);
        const uint8_t *usrc = slot_src(p.up, p.ids64, s, p.err, false, p.quiet);
        const bool valid = gsrc && usrc;
        const uint8_t *base = stages + static_cast<size_t>(st) * p.stage_bytes;
        const uint8_t *gbase =
            base + (valid ? (reinterpret_cast<uintptr_t>(gsrc + static_cast<size_t>(rr) * p.rb_g) & 15) : 0);
        const uint8_t *ubase = base + p.up_off +
            (valid ? (reinterpret_cast<uintptr_t>(usrc + static_cast<size_t>(rr) * p.rb_u) & 15) : 0);
        for (int t = cw * rpw; t < n; t += kConsumerWarps * rpw) {
            const int row = t + grp;
            float g = 0.f, u = 0.f;
            if (valid && active && row < n) {
                g = unit_dot<QT>(gbase + static_cast<size_t>(row) * p.rb_g, ug, x);
                u = unit_dot<QT>(ubase + static_cast<size_t>(row) * p.rb_u, ug, x);
            }
            for (int o = p.gs >> 1; o; o >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, o);
                u += __shfl_xor_sync(0xffffffffu, u, o);
            }
            // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
            if (ug == 0 && row < n) p.h[static_cast<size_t>(s) * p.F + rr + row] = g / (1.0f + expf(-g)) * u;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        r += n;
        ci++;
    }
}

int gate_up_smem(const GateUpArgs &a) { return 256 + a.nst * static_cast<int>(a.stage_bytes); }

template <int QT>
static cudaError_t launch_gate_up_t(const GateUpArgs &a, int grid, cudaStream_t st) {
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(k_gate_up<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr_done = true;
    }
    k_gate_up<QT><<<grid, kFusedThreads, gate_up_smem(a), st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gate_up(const GateUpArgs &a, int qtype, int grid, cudaStream_t st) {
    switch (qtype) {
    case STYX_Q4_K: return launch_gate_up_t<STYX_Q4_K>(a, grid, st);
    case STYX_Q5_K: return launch_gate_up_t<STYX_Q5_K>(a, grid, st);
    case STYX_Q6_K: return launch_gate_up_t<STYX_Q6_K>(a, grid, st);
    case STYX_Q8_0: return launch_gate_up_t<STYX_Q8_0>(a, grid, st);
    default: return cudaErrorInvalidValue;
    }
}

// -------------------------------------------------------- down + combine
// CTA b owns output rows [H*b/G, H*(b+1)/G); a chunk is <= rc rows, copied
// for every slot (k bulk copies).  h is turned into digits once per CTA.
// moe_reduce_f32.comp:8-13: acc = sum_s w[s]*d[s][i] in slot order, x += acc.
// CW consumer warps after the producer warp: 8 for the MoE block's down
// rows, 16 for a dense GEMV (one slot, long rows: more warps keep more
// dot products in flight per scheduler).
template <int QT, int CW>
__global__ void __launch_bounds__(32 * (CW + 1), 1) k_down(const DownArgs p) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 16;
    float *wts = reinterpret_cast<float *>(smem + 2 * 16 * sizeof(uint64_t));   // 16 floats
    const int kF = p.k * p.F;
    int8_t *hd1 = reinterpret_cast<int8_t *>(smem + p.dig_off);
    uint8_t *hd2 = reinterpret_cast<uint8_t *>(hd1 + kF);
    uint8_t *hd3 = hd2 + kF;
    float *hsc = reinterpret_cast<float *>(hd3 + kF);
    float *dpart = reinterpret_cast<float *>(smem + p.part_off);
    uint8_t *stages = smem + p.stage_off;
    const int nparts = p.nst < 2 ? 2 : p.nst;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rbeg = static_cast<int>(static_cast<long long>(p.H) * blockIdx.x / gridDim.x);
    const int rend = static_cast<int>(static_cast<long long>(p.H) * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nst; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            int ci = 0;
            for (int r0 = rbeg; r0 < rend; r0 += p.rc, ci++) {
                const int n = min(p.rc, rend - r0);
                const int st = ci % p.nst;
                if (ci >= p.nst && !mbar_wait(&empty[st], ((ci / p.nst) - 1) & 1, p.err, kErrWaitEmpty))
                    break;
                uint8_t *dst = stages + static_cast<size_t>(st) * p.stage_bytes;
                uint32_t total = 0;
                for (int s = 0; s < p.k; s++) {
                    const uint8_t *src = slot_src(p.down, p.ids64, s, p.err, true, p.quiet);
                    if (!src) continue;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src + static_cast<size_t>(r0) * p.rb);
                    const uintptr_t aa = a0 & ~uintptr_t(15);
                    const uintptr_t ab = (a0 + static_cast<size_t>(n) * p.rb + 15) & ~uintptr_t(15);
                    total += static_cast<uint32_t>(ab - aa);
                }
                if (total == 0) {
                    mbar_arrive(&full[st]);
                    continue;
                }
                mbar_arrive_expect_tx(&full[st], total);
                for (int s = 0; s < p.k; s++) {
                    const uint8_t *src = slot_src(p.down, p.ids64, s, p.err, false, p.quiet);
                    if (!src) continue;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src + static_cast<size_t>(r0) * p.rb);
                    const uintptr_t aa = a0 & ~uintptr_t(15);
                    const uintptr_t ab = (a0 + static_cast<size_t>(n) * p.rb + 15) & ~uintptr_t(15);
                    bulk_g2s(dst + static_cast<size_t>(s) * p.slot_stride, reinterpret_cast<const void *>(aa),
                             static_cast<uint32_t>(ab - aa), &full[st]);
                }
            }
        }
        return;
    }

    // consumers: h -> digits (shared), weights
    const int cw = warp - 1;
    digits_vector<8, true>(p.h, kF, hd1, hd2, hd3, hsc, threadIdx.x - 32, CW * 32);
    if (cw == 0 && lane < p.k) wts[lane] = p.w[lane];
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");

    const int rpw = 32 / p.gs;
    const int ug = lane & (p.gs - 1), grp = lane / p.gs;
    const bool active = ug < p.units;
    // warp -> (slot, row phase): k <= 8 slots share the 8 warps, k > 8 loop
    const bool multi = p.k > CW;
    const int nwps = multi ? 1 : CW / p.k;
    const int slot0 = multi ? cw : cw / nwps;
    const int sub = multi ? 0 : cw % nwps;
    const int sstep = multi ? CW : 1 << 30;
    // rows of at most 32 units: a lane's unit of h stays in registers; wider
    // rows (a dense GEMV over more than 2048 columns) reload it per unit
    const bool preload = p.units <= 32;
    XUnit x;
    if (preload && !multi && slot0 < p.k && active)
        load_xunit<QT>(x, hd1 + slot0 * p.F, hd2 + slot0 * p.F, hd3 + slot0 * p.F, hsc + slot0 * (p.F >> 5), ug);

    // After a timed-out wait a warp stops computing but keeps taking part in
    // the named barriers, so the other consumer warps are never stranded.
    bool ok = true;
    int ci = 0;
    for (int r0 = rbeg; r0 < rend; r0 += p.rc, ci++) {
        const int n = min(p.rc, rend - r0);
        const int st = ci % p.nst;
        if (ok) ok = mbar_wait(&full[st], (ci / p.nst) & 1, p.err, kErrWaitFull);
        float *part = dpart + static_cast<size_t>(ci % nparts) * p.k * p.rc;
        for (int s = slot0; ok && s < p.k; s += sstep) {
            if (preload && multi && active)
                load_xunit<QT>(x, hd1 + s * p.F, hd2 + s * p.F, hd3 + s * p.F, hsc + s * (p.F >> 5), ug);
            const uint8_t *src = slot_src(p.down, p.ids64, s, p.err, false, p.quiet);
            const uint8_t *base = stages + static_cast<size_t>(st) * p.stage_bytes +
                                  static_cast<size_t>(s) * p.slot_stride +
                                  (src ? (reinterpret_cast<uintptr_t>(src + static_cast<size_t>(r0) * p.rb) & 15) : 0);
            // two rows per lane group per pass when the unit's digits stay in
            // registers: independent dot products in flight
            for (int t = sub * rpw; preload && t < n; t += 2 * nwps * rpw) {
                const int ra = t + grp, rb = t + nwps * rpw + grp;
                float va = 0.f, vb = 0.f;
                if (src && active && ra < n) va = unit_dot<QT>(base + static_cast<size_t>(ra) * p.rb, ug, x);
                if (src && active && rb < n) vb = unit_dot<QT>(base + static_cast<size_t>(rb) * p.rb, ug, x);
                __syncwarp();   // regroup the lanes after the row-bound branches
                for (int o = p.gs >> 1; o; o >>= 1) {
                    va += __shfl_xor_sync(0xffffffffu, va, o);
                    vb += __shfl_xor_sync(0xffffffffu, vb, o);
                }
                if (ug == 0 && ra < n) part[s * p.rc + ra] = va;
                if (ug == 0 && rb < n) part[s * p.rc + rb] = vb;
            }
            for (int t = sub * rpw; !preload && t < n; t += nwps * rpw) {
                const int row = t + grp;
                float v = 0.f;
                if (src && row < n) {
                    for (int u = ug; u < p.units; u += p.gs) {
                        load_xunit<QT>(x, hd1 + s * p.F, hd2 + s * p.F, hd3 + s * p.F, hsc + s * (p.F >> 5), u);
                        v += unit_dot<QT>(base + static_cast<size_t>(row) * p.rb, u, x);
                    }
                }
                __syncwarp();   // regroup the lanes after the row-bound branches
                for (int o = p.gs >> 1; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (ug == 0 && row < n) part[s * p.rc + row] = v;
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
        const int ct = threadIdx.x - 32;
        if (ok && ct < n) {
            if (p.partial) {   // per-slot contributions for a cross-device sum (expert parallelism)
                for (int s = 0; s < p.k; s++)
                    p.partial[static_cast<size_t>(s) * p.H + r0 + ct] = __fmul_rn(wts[s], part[s * p.rc + ct]);
            } else {
                float acc = 0.f;
                for (int s = 0; s < p.k; s++) acc = __fadd_rn(acc, __fmul_rn(wts[s], part[s * p.rc + ct]));
                p.x[r0 + ct] = __fadd_rn(p.x[r0 + ct], acc);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
}

template <int QT, int CW>
static cudaError_t launch_down_t(const DownArgs &a, int grid, uint32_t smem, cudaStream_t st) {
    static bool attr_done = false;   // (the attributes are the same on every device)
    if (!attr_done) {
        cudaFuncSetAttribute(k_down<QT, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        cudaFuncSetAttribute(k_down<QT, CW>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        attr_done = true;
    }
    return launch_pdl(k_down<QT, CW>, dim3(grid), dim3(32 * (CW + 1)), smem, st, a);
}

template <int CW>
static cudaError_t launch_down_w(const DownArgs &a, int qtype, int grid, uint32_t smem, cudaStream_t st) {
    switch (qtype) {
    case STYX_Q4_K: return launch_down_t<STYX_Q4_K, CW>(a, grid, smem, st);
    case STYX_Q5_K: return launch_down_t<STYX_Q5_K, CW>(a, grid, smem, st);
    case STYX_Q6_K: return launch_down_t<STYX_Q6_K, CW>(a, grid, smem, st);
    case STYX_Q8_0: return launch_down_t<STYX_Q8_0, CW>(a, grid, smem, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_down(const DownArgs &a, int qtype, int grid, uint32_t smem, cudaStream_t st, bool wide) {
    return wide ? launch_down_w<kWideConsumerWarps>(a, qtype, grid, smem, st)
                : launch_down_w<kConsumerWarps>(a, qtype, grid, smem, st);
}

// ------------------------------------------------ generic id matvec
// MatVecIdPush semantics (ops.rs:120-147, kernels.rs:124-131).  Grid
// (row tiles of rows_per_cta, slots).  Weights are read straight from global
// memory; x row (slot % ne11) becomes digits in shared memory.

template <int QT>
__global__ void __launch_bounds__(256) k_matvec_id(const MatVecIdArgs p) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t sm[];
    const int s = blockIdx.y;
    const uint8_t *a = nullptr;
    if (p.src3[0] || p.src3[1] || p.src3[2]) {   // hot, arena, full: the last source set and in range
        for (int i = 0; i < 3; i++) {
            if (!p.src3[i]) continue;
            const uint32_t e = static_cast<uint32_t>(p.ids[16 * (i + 1) + s]);
            if (e == kSkip) continue;
            if (e >= static_cast<uint32_t>(p.count3[i])) {
                if (threadIdx.x == 0 && blockIdx.x == 0 && p.err) atomicExch(p.err, kErrBadId);
                continue;
            }
            a = p.src3[i] + static_cast<uint64_t>(e) * p.stride3[i];
        }
        if (!a) return;   // the slot's output is left as it is
    } else {
        const uint32_t e = static_cast<uint32_t>(p.ids[s]);
        if (e == kSkip) return;
        if (e >= static_cast<uint32_t>(p.n_expert)) {
            if (threadIdx.x == 0 && blockIdx.x == 0 && p.err) atomicExch(p.err, kErrBadId);
            return;
        }
        a = p.a + static_cast<uint64_t>(e) * p.expert_bytes;
    }
    int8_t *d1 = reinterpret_cast<int8_t *>(sm);
    uint8_t *d2 = reinterpret_cast<uint8_t *>(sm) + p.ncols;
    uint8_t *d3 = d2 + p.ncols;
    float *sc = reinterpret_cast<float *>(d3 + p.ncols);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *xr = p.x + static_cast<size_t>(s % p.ne11) * p.stride_b;
    const DigitsView dv{d1, d2, d3, sc};
    for (int g = warp; g < (p.ncols >> 5); g += 8) digits_group_warp(xr[g * 32 + lane], lane, dv, g);
    __syncthreads();

    const int rpw = 32 / p.gs;
    const int ug = lane & (p.gs - 1), grp = lane / p.gs;
    const int r0 = blockIdx.x * p.rows_per_cta, r1 = min(p.nrows, r0 + p.rows_per_cta);
    XUnit x;
    const bool preload = p.units <= 32;
    if (preload && ug < p.units) load_xunit<QT>(x, d1, d2, d3, sc, ug);
    // four rows per lane group in flight; each row's sum (lane order, then
    // the shuffle tree) is the same whatever the grouping
    constexpr int R = 4;
    for (int t = r0 + warp * rpw * R; t < r1; t += 8 * rpw * R) {
        float v[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int row = t + j * rpw + grp;
            v[j] = 0.f;
            if (row < r1) {
                for (int u = ug; u < p.units; u += p.gs) {
                    if (!preload) load_xunit<QT>(x, d1, d2, d3, sc, u);
                    v[j] += unit_dot<QT>(a + static_cast<size_t>(row) * p.rb, u, x);
                }
            }
        }
        __syncwarp();   // regroup the lanes after the row-bound branches
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int row = t + j * rpw + grp;
            for (int o = p.gs >> 1; o; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
            if (ug == 0 && row < r1) p.y[static_cast<size_t>(s) * p.stride_d + row] = v[j];
        }
    }
}

template <int QT>
static cudaError_t launch_matvec_id_t(const MatVecIdArgs &a, cudaStream_t st) {
    const size_t smem = static_cast<size_t>(a.ncols) * 3 + static_cast<size_t>(a.ncols / 32) * 4;
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(k_matvec_id<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr_done = true;
    }
    dim3 grid((a.nrows + a.rows_per_cta - 1) / a.rows_per_cta, a.n_ids);
    return launch_pdl(k_matvec_id<QT>, grid, dim3(256), smem, st, a);
}

cudaError_t launch_matvec_id(const MatVecIdArgs &a, int qtype, cudaStream_t st) {
    switch (qtype) {
    case STYX_Q4_K: return launch_matvec_id_t<STYX_Q4_K>(a, st);
    case STYX_Q5_K: return launch_matvec_id_t<STYX_Q5_K>(a, st);
    case STYX_Q6_K: return launch_matvec_id_t<STYX_Q6_K>(a, st);
    case STYX_Q8_0: return launch_matvec_id_t<STYX_Q8_0>(a, st);
    default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------ single ops
__global__ void __launch_bounds__(256) k_rms_norm(const float *x, const float *w, float eps, int ncols,
                                                  float *out) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const float *xr = x + static_cast<size_t>(blockIdx.x) * ncols;
    float *orow = out + static_cast<size_t>(blockIdx.x) * ncols;
    float ss = 0.f;
    for (int c = threadIdx.x; c < ncols; c += 256) ss += xr[c] * xr[c];
    ss = block_sum256(ss, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(ncols) + eps);
    for (int c = threadIdx.x; c < ncols; c += 256) {
        const float v = xr[c] * scale;
        orow[c] = w ? v * w[c] : v;
    }
}

cudaError_t launch_rms_norm(const float *x, const float *w, float eps, int ncols, int nrows, float *out,
                            cudaStream_t st) {
    return launch_pdl(k_rms_norm, dim3(nrows), dim3(256), 0, st, x, w, eps, ncols, out);
}

__global__ void __launch_bounds__(256) k_matvec_f32(const float *a, int ncols, int stride_a, const float *x,
                                                    float *d) {
    __shared__ float red[32];
    const float *ar = a + static_cast<size_t>(blockIdx.x) * stride_a;
    float acc = 0.f;
    for (int c = threadIdx.x; c < ncols; c += 256) acc += ar[c] * x[c];
    acc = block_sum256(acc, red);
    if (threadIdx.x == 0) d[blockIdx.x] = acc;
}

cudaError_t launch_matvec_f32(const float *a, int nrows, int ncols, int stride_a, const float *x, float *d,
                              cudaStream_t st) {
    k_matvec_f32<<<nrows, 256, 0, st>>>(a, ncols, stride_a, x, d);
    return cudaGetLastError();
}

__global__ void __launch_bounds__(256) k_topk(const float *logits, int n, int k, int renorm,
                                              const uint32_t *remap, const uint32_t *pmap, float *weights,
                                              int32_t *ids64) {
    __shared__ float red[32];
    __shared__ float lg[STYX_MAX_EXPERTS];
    __shared__ int sel[16];
    for (int i = threadIdx.x; i < n; i += 256) lg[i] = logits[i];
    __syncthreads();
    topk_block(lg, n, k, renorm, remap, pmap, weights, ids64, red, sel);
}

cudaError_t launch_topk(const float *logits, int n, int k, int renorm, const uint32_t *remap,
                        const uint32_t *pmap, float *weights, int32_t *ids64, cudaStream_t st) {
    k_topk<<<1, 256, 0, st>>>(logits, n, k, renorm, remap, pmap, weights, ids64);
    return cudaGetLastError();
}

__global__ void k_swiglu(const float *g, const float *u, float *out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float a = g[i];
        out[i] = a / (1.0f + expf(-a)) * u[i];
    }
}

cudaError_t launch_swiglu(const float *g, const float *u, float *out, int n, cudaStream_t st) {
    k_swiglu<<<(n + 255) / 256, 256, 0, st>>>(g, u, out, n);
    return cudaGetLastError();
}

__global__ void k_moe_reduce(const float *d, const float *w, float *x, int ne, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ne) return;
    float acc = 0.f;
    for (int s = 0; s < k; s++) acc = __fadd_rn(acc, __fmul_rn(w[s], d[static_cast<size_t>(s) * ne + i]));
    x[i] = __fadd_rn(x[i], acc);
}

// x[i] += sum_s partial[s*ne + i] in slot order: moe_reduce_f32.comp with the
// weights already applied by the devices that own the slots (each slot has
// one non-zero contributor, so the cross-device sum before this is exact and
// the result equals the single-device combine bit for bit)
__global__ void k_combine_partial(const float *partial, float *x, int ne, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ne) return;
    float acc = 0.f;
    for (int s = 0; s < k; s++) acc = __fadd_rn(acc, partial[static_cast<size_t>(s) * ne + i]);
    x[i] = __fadd_rn(x[i], acc);
}

cudaError_t launch_combine_partial(const float *partial, float *x, int ne, int k, cudaStream_t st) {
    k_combine_partial<<<(ne + 255) / 256, 256, 0, st>>>(partial, x, ne, k);
    return cudaGetLastError();
}

// ------------------------------------------------ cross-rank sum + combine over peer memory
constexpr int kEpThreads = 256;

// CTA b owns columns [kEpCols b, kEpCols (b+1)) of every slot: it sends
// this rank's values of them as tagged words into row `rank` of every
// peer's inbox, then each thread waits for its columns' words of every peer
// and adds sum_s (sum_p partial_p[s][c]) into x[c], ranks then slots in
// order (ep_sync.cuh).
__global__ void __launch_bounds__(kEpThreads) k_ep_combine(const EpCombineArgs a) {
    pdl_trigger();
    pdl_wait();
    const EpPeers &ep = *a.ep;
    const int b = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
    const int c0 = b * kEpCols, nc = min(kEpCols, a.H - c0);
    const int rank = ep.rank, world = ep.world, k = ep.k;
    const unsigned long long gen = ep_generation(ep);
    const unsigned tag = static_cast<unsigned>(gen);
    // 1. send
    for (int i = tid; i < k * nc; i += kEpThreads) {
        const int s = i / nc, c = c0 + (i - s * nc);
        const float v = a.partial[static_cast<size_t>(s) * a.H + c];
        const size_t o = ep_index(ep, gen, rank, s, c);
        for (int p = 0; p < world; p++)
            if (p != rank) ep_put(ep.inbox[p] + o, tag, v);
    }
    // 2. the slot-ordered sum as the peers' words arrive (one non-zero rank
    // per slot: exact in any order)
    const unsigned long long *box = ep.inbox[rank];
    bool live = true;
    for (int j = tid; j < nc; j += kEpThreads) {
        const int c = c0 + j;
        float acc = 0.f;
        for (int s = 0; s < k; s++) {
            float v = 0.f;
            for (int p = 0; p < world; p++)
                v = __fadd_rn(v, p == rank ? a.partial[static_cast<size_t>(s) * a.H + c]
                                           : ep_get(box + ep_index(ep, gen, p, s, c), tag, live, a.err));
            acc = __fadd_rn(acc, v);
        }
        a.x[c] = __fadd_rn(a.x[c], acc);
    }
    // 3. the last CTA of the call advances the generation
    __syncthreads();
    ep_call_done(ep, gen, G);
}

cudaError_t launch_ep_combine(const EpCombineArgs &a, cudaStream_t st) {
    return launch_pdl(k_ep_combine, dim3((a.H + kEpCols - 1) / kEpCols), dim3(kEpThreads), 0, st, a);
}

cudaError_t launch_moe_reduce(const float *d, const float *w, float *x, int ne, int k, cudaStream_t st) {
    k_moe_reduce<<<(ne + 255) / 256, 256, 0, st>>>(d, w, x, ne, k);
    return cudaGetLastError();
}

// gather_slabs_f32.comp:40-85 over (piece, slot): 16-byte vector copies; the
// source may be pinned host memory mapped into the device address space.
constexpr int kGatherPieces = 32;

__global__ void __launch_bounds__(256) k_gather(const GatherArgs p) {
    const int s = blockIdx.y;
    const uint32_t e = static_cast<uint32_t>(p.ids[s]);
    if (e == kSkip) return;
    if (e >= static_cast<uint32_t>(p.n_expert)) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && p.err) atomicExch(p.err, kErrBadId);
        return;
    }
    const uint64_t slot = static_cast<uint64_t>(p.layer) * p.k + s;
#pragma unroll
    for (int t = 0; t < 3; t++) {
        const uint4 *src = reinterpret_cast<const uint4 *>(p.src[t] + e * p.src_bytes[t]);
        uint4 *dst = reinterpret_cast<uint4 *>(p.dst[t] + slot * p.dst_bytes[t]);
        const uint64_t nv = p.src_bytes[t] / 16;
        for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * 256 + threadIdx.x; i < nv;
             i += static_cast<uint64_t>(gridDim.x) * 256)
            dst[i] = src[i];
    }
}

cudaError_t launch_gather(const GatherArgs &a, cudaStream_t st) {
    dim3 grid(kGatherPieces, a.k);
    k_gather<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace styx
