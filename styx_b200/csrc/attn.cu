// attn.cu -- the attention half of a decode layer (the part of
// MoeModel::forward_token before the MoE block, crates/model/src/moe.rs:
// 1845-1972), sm_100a:
//
//   k_qk_norm_rope_kv   per-head RMSNorm of q and k (QkNorm::PerHead,
//                       moe.rs:1880-1897), NEOX RoPE at the token's position
//                       (rope_neox_f32 as RopePush::neox sets it up,
//                       crates/vk-backend/src/ops.rs:413-445; moe.rs:1914-1932)
//                       and the K / V cache rows at that position
//                       (moe.rs:1933-1945) -- six dispatches of the reference
//                       in one launch, one CTA per q or kv head
//   k_attn_split        single-token GQA attention (shaders/attn_decode_f32.comp)
//                       as split-sequence partials: CTA (kv head, split) reads
//                       its K and V rows once for all the kv head's q heads
//   k_attn_combine      merges the splits' (max, sum, acc) per head
//   k_add_f32           shaders/add_flat_f32.comp
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace styx {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kHeadsPerPass = 8;   // q heads whose V accumulators a lane holds at once

// float offset of the per-warp accumulators in k_attn_split's shared memory
// (16-byte aligned: they are stored as float4)
__host__ __device__ inline int attn_acc_offset(int gqa, int hd, int tps) {
    return (gqa * hd + tps * gqa + 2 * gqa + 3) & ~3;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------ q/k norm + RoPE + KV rows
// CTA (token t, row r): r < n_heads is q head r, normalised and rotated in
// place; r = n_heads + j is kv head j -- k normalised, rotated, written to k
// (in place) and to the K cache row pos[t]; v copied to the V cache row.
// Thread i < hd/2 owns the NEOX pair (i, i + hd/2).
__global__ void __launch_bounds__(128) k_qk_norm_rope_kv(QkRopeArgs a) {
    __shared__ float red[4];
    const int rows = a.n_heads + a.n_kv;
    const int t = blockIdx.x / rows, h = blockIdx.x - t * rows;
    const bool is_q = h < a.n_heads;
    const int head = is_q ? h : h - a.n_heads;
    float *src = is_q ? a.q + (static_cast<size_t>(t) * a.n_heads + head) * a.hd
                      : a.k + (static_cast<size_t>(t) * a.n_kv + head) * a.hd;
    const float *w = is_q ? a.q_norm : a.k_norm;
    const int half = a.hd >> 1, i = threadIdx.x;
    const bool on = i < half;
    float x0 = on ? src[i] : 0.f, x1 = on ? src[i + half] : 0.f;
    if (w) {
        // rms_norm_f32 over the head's hd elements: x * (1/sqrt(mean(x^2)+eps)) * w
        float ss = warp_sum(x0 * x0 + x1 * x1);
        if ((i & 31) == 0) red[i >> 5] = ss;
        __syncthreads();
        ss = red[0] + red[1] + red[2] + red[3];
        const float scale = 1.0f / sqrtf(ss / static_cast<float>(a.hd) + a.eps);
        if (on) {
            x0 = x0 * scale * w[i];
            x1 = x1 * scale * w[i + half];
        }
    }
    const int pos = a.pos[t];
    const bool row_ok = pos >= 0 && pos < a.n_ctx;   // a cache row outside is skipped and reported
    if (!is_q && !row_ok && threadIdx.x == 0 && (a.kcache || a.vcache)) atomicExch(a.err, kErrBadPos);
    if (on) {
        // theta_i = pos * base^(-2i/hd), evaluated in double (the reference
        // test's CPU form, crates/vk-backend/tests/ops2.rs:427-438)
        const double theta = static_cast<double>(pos) * pow(a.theta_scale, static_cast<double>(i));
        double sn, cs;
        sincos(theta, &sn, &cs);
        const double y0 = static_cast<double>(x0) * cs - static_cast<double>(x1) * sn;
        const double y1 = static_cast<double>(x0) * sn + static_cast<double>(x1) * cs;
        const float r0 = static_cast<float>(y0), r1 = static_cast<float>(y1);
        src[i] = r0;
        src[i + half] = r1;
        if (!is_q && a.kcache && row_ok) {
            float *krow = a.kcache + static_cast<size_t>(pos) * a.kv_dim + static_cast<size_t>(head) * a.hd;
            krow[i] = r0;
            krow[i + half] = r1;
        }
    }
    if (!is_q && a.vcache && row_ok) {
        const float *vh = a.v + (static_cast<size_t>(t) * a.n_kv + head) * a.hd;
        float *vrow = a.vcache + static_cast<size_t>(pos) * a.kv_dim + static_cast<size_t>(head) * a.hd;
        for (int j = i; j < a.hd; j += 128) vrow[j] = vh[j];
    }
}

// ------------------------------------------------------------ attention partials
// CTA (kv head j, split s) covers tokens [s*tps, min(n_t, (s+1)*tps)) for the
// gqa q heads j*gqa .. j*gqa+gqa-1.  Scores go to shared memory; the split's
// max and sum per head, then P.V with each lane holding float4 columns of V
// for up to 8 heads.  Writes per (head, split): m, l and acc[hd] (unnormalised).
template <int NF4>   // float4s of a row per lane: hd <= 128 * NF4
__global__ void __launch_bounds__(kAttnThreads) k_attn_split(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int gqa = a.gqa, hd = a.hd;
    float *sq = sm;                                   // [gqa][hd] the q heads
    float *ssc = sq + gqa * hd;                       // [tps][gqa] scores, then probabilities
    float *sml = ssc + a.tps * gqa;                   // [gqa][2] split max, sum
    float *sacc = sm + attn_acc_offset(gqa, hd, a.tps);   // [warps][8][hd] per-warp accumulators
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int t0 = split * a.tps, t1 = min(a.n_t, t0 + a.tps), nt = t1 - t0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *qb = a.q + static_cast<size_t>(kvh) * gqa * hd;
    for (int i = threadIdx.x; i < gqa * hd; i += kAttnThreads) sq[i] = qb[i];
    __syncthreads();
    const size_t koff = static_cast<size_t>(kvh) * hd;

    // scores: one token per warp pass, lane c holds elements 4c + 128 f
    for (int t = warp; t < nt; t += kAttnWarps) {
        const float *kr = a.kcache + static_cast<size_t>(t0 + t) * a.kv_dim + koff;
        float4 kv[NF4];
#pragma unroll
        for (int f = 0; f < NF4; f++) {
            const int c = 4 * lane + 128 * f;
            kv[f] = c < hd ? __ldg(reinterpret_cast<const float4 *>(kr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int g = 0; g < gqa; g++) {
            float d = 0.f;
#pragma unroll
            for (int f = 0; f < NF4; f++) {
                const int c = 4 * lane + 128 * f;
                if (c < hd) {
                    const float4 qv = *reinterpret_cast<const float4 *>(sq + g * hd + c);
                    d += qv.x * kv[f].x + qv.y * kv[f].y + qv.z * kv[f].z + qv.w * kv[f].w;
                }
            }
            d = warp_sum(d);
            if (lane == 0) ssc[t * gqa + g] = d * a.scale;
        }
    }
    __syncthreads();
    // per head: the split's max, the probabilities exp(s - m) and their sum
    for (int g = warp; g < gqa; g += kAttnWarps) {
        float m = -INFINITY;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, ssc[t * gqa + g]);
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < nt; t += 32) {
            const float p = expf(ssc[t * gqa + g] - m);
            ssc[t * gqa + g] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            sml[2 * g] = m;
            sml[2 * g + 1] = l;
        }
    }
    __syncthreads();
    // P.V: heads in passes of 8, tokens spread over the warps
    for (int g0 = 0; g0 < gqa; g0 += kHeadsPerPass) {
        const int ng = min(kHeadsPerPass, gqa - g0);
        float4 acc[kHeadsPerPass][NF4];
#pragma unroll
        for (int g = 0; g < kHeadsPerPass; g++)
#pragma unroll
            for (int f = 0; f < NF4; f++) acc[g][f] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t = warp; t < nt; t += kAttnWarps) {
            const float *vr = a.vcache + static_cast<size_t>(t0 + t) * a.kv_dim + koff;
            float4 vv[NF4];
#pragma unroll
            for (int f = 0; f < NF4; f++) {
                const int c = 4 * lane + 128 * f;
                vv[f] = c < hd ? __ldg(reinterpret_cast<const float4 *>(vr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int g = 0; g < kHeadsPerPass; g++) {
                if (g < ng) {
                    const float p = ssc[t * gqa + g0 + g];
#pragma unroll
                    for (int f = 0; f < NF4; f++) {
                        acc[g][f].x += p * vv[f].x;
                        acc[g][f].y += p * vv[f].y;
                        acc[g][f].z += p * vv[f].z;
                        acc[g][f].w += p * vv[f].w;
                    }
                }
            }
        }
        // the warps' accumulators through shared memory, summed in warp order
#pragma unroll
        for (int g = 0; g < kHeadsPerPass; g++)
#pragma unroll
            for (int f = 0; f < NF4; f++) {
                const int c = 4 * lane + 128 * f;
                if (g < ng && c < hd)
                    *reinterpret_cast<float4 *>(sacc + (warp * kHeadsPerPass + g) * hd + c) = acc[g][f];
            }
        __syncthreads();
        for (int i = threadIdx.x; i < ng * hd; i += kAttnThreads) {
            const int g = i / hd, c = i - g * hd;
            float s = 0.f;
            for (int w = 0; w < kAttnWarps; w++) s += sacc[(w * kHeadsPerPass + g) * hd + c];
            const int head = kvh * gqa + g0 + g;
            a.part_acc[(static_cast<size_t>(head) * a.n_splits + split) * hd + c] = s;
        }
        __syncthreads();
    }
    for (int g = threadIdx.x; g < gqa; g += kAttnThreads) {
        const size_t ix = static_cast<size_t>(kvh * gqa + g) * a.n_splits + split;
        a.part_ml[2 * ix] = sml[2 * g];
        a.part_ml[2 * ix + 1] = sml[2 * g + 1];
    }
}

// out[h][c] = sum_s e^(m_s - M) acc_s[c] / sum_s e^(m_s - M) l_s
__global__ void __launch_bounds__(128) k_attn_combine(AttnArgs a) {
    const int h = blockIdx.x;
    const float *ml = a.part_ml + static_cast<size_t>(h) * a.n_splits * 2;
    float M = -INFINITY;
    for (int s = 0; s < a.n_splits; s++) M = fmaxf(M, ml[2 * s]);
    float L = 0.f;
    for (int s = 0; s < a.n_splits; s++) L += expf(ml[2 * s] - M) * ml[2 * s + 1];
    const float inv = 1.0f / L;
    for (int c = threadIdx.x; c < a.hd; c += 128) {
        float o = 0.f;
        for (int s = 0; s < a.n_splits; s++)
            o += expf(ml[2 * s] - M) * a.part_acc[(static_cast<size_t>(h) * a.n_splits + s) * a.hd + c];
        a.out[static_cast<size_t>(h) * a.hd + c] = o * inv;
    }
}

__global__ void k_add_f32(const float *x, const float *y, float *d, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) d[i] = x[i] + y[i];
}

}  // namespace

size_t attn_smem_bytes(int gqa, int hd, int tps) {
    return (static_cast<size_t>(attn_acc_offset(gqa, hd, tps)) + static_cast<size_t>(kAttnWarps) * kHeadsPerPass * hd) *
           4;
}

cudaError_t launch_qk_norm_rope_kv(const QkRopeArgs &a, cudaStream_t st) {
    k_qk_norm_rope_kv<<<a.n_tokens * (a.n_heads + a.n_kv), 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st) {
    const size_t smem = attn_smem_bytes(a.gqa, a.hd, a.tps);
    const dim3 grid(a.n_kv, a.n_splits);
    cudaError_t e;
    if (a.hd <= 128) {
        e = cudaFuncSetAttribute(k_attn_split<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        k_attn_split<1><<<grid, kAttnThreads, smem, st>>>(a);
    } else {
        e = cudaFuncSetAttribute(k_attn_split<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        k_attn_split<2><<<grid, kAttnThreads, smem, st>>>(a);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_attn_combine<<<a.n_kv * a.gqa, 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_add_f32(const float *x, const float *y, float *d, int n, cudaStream_t st) {
    k_add_f32<<<(n + 255) / 256, 256, 0, st>>>(x, y, d, n);
    return cudaGetLastError();
}

}  // namespace styx
