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
//   k_get_rows          the token-embedding row (dequant_q4k on the host,
//                       moe.rs:1824-1836), any of the four block formats
//   k_argmax            the greedy pick over the logits
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
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
    pdl_trigger();
    pdl_wait();
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
    pdl_trigger();
    pdl_wait();
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

// out[h][c] = sum_s e^(m_s - M) acc_s[c] / sum_s e^(m_s - M) l_s: the
// split weights once per head in shared memory, then every column's sum
// with its loads in flight.
__global__ void __launch_bounds__(128) k_attn_combine(AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ float w[kAttnMaxSplits];
    __shared__ float red[8];
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ns = a.n_splits;
    const float *ml = a.part_ml + static_cast<size_t>(h) * ns * 2;
    float m = -INFINITY;
    for (int s = tid; s < ns; s += 128) m = fmaxf(m, ml[2 * s]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float l = 0.f;
    for (int s = tid; s < ns; s += 128) {
        const float ws = expf(ml[2 * s] - M);
        w[s] = ws;
        l += ws * ml[2 * s + 1];
    }
    l = warp_sum(l);
    if (lane == 0) red[4 + warp] = l;
    __syncthreads();
    const float inv = 1.0f / (red[4] + red[5] + red[6] + red[7]);
    const float *acc = a.part_acc + static_cast<size_t>(h) * ns * a.hd;
    for (int c = tid; c < a.hd; c += 128) {
        float o = 0.f;
#pragma unroll 8
        for (int s = 0; s < ns; s++) o += w[s] * acc[static_cast<size_t>(s) * a.hd + c];
        a.out[static_cast<size_t>(h) * a.hd + c] = o * inv;
    }
}

__global__ void k_add_f32(const float *x, const float *y, float *d, int n) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) d[i] = x[i] + y[i];
}

// ------------------------------------------------------------ embedding rows
// out[r][c] = deq(W)[rows[r]][c]: one thread per element, the block formats
// decoded with the reference's own expression order (moe.rs:506-533 for
// q4_K; the published GGUF layouts for q5_K / q6_K / q8_0) and no fused
// multiply-adds, so the rows are bit-identical to a CPU decode.
__device__ __forceinline__ float rd_f16(const uint8_t *p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}
__device__ __forceinline__ void kq_scale_min(const uint8_t *s, int j, float &sc, float &m) {
    if (j < 4) {
        sc = static_cast<float>(s[j] & 63);
        m = static_cast<float>(s[j + 4] & 63);
    } else {
        sc = static_cast<float>((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        m = static_cast<float>((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

__global__ void k_get_rows(GetRowsArgs a) {
    pdl_trigger();
    pdl_wait();
    const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<long long>(a.n) * a.ncols) return;
    const int r = static_cast<int>(e / a.ncols), c = static_cast<int>(e - static_cast<long long>(r) * a.ncols);
    const int row = a.rows[r];
    if (row < 0 || row >= a.nrows) {   // skipped and reported
        a.out[e] = 0.f;
        if (c == 0) atomicExch(a.err, kErrBadId);
        return;
    }
    const uint8_t *rp = a.w + static_cast<size_t>(row) * a.row_bytes;
    float v = 0.f;
    if (a.qtype == STYX_Q8_0) {
        const uint8_t *b = rp + static_cast<size_t>(c / 32) * 34;
        v = __fmul_rn(rd_f16(b), static_cast<float>(static_cast<int8_t>(b[2 + c % 32])));
    } else {
        const int blk = c / 256, i = c % 256;
        if (a.qtype == STYX_Q4_K || a.qtype == STYX_Q5_K) {
            const uint8_t *b = rp + static_cast<size_t>(blk) * (a.qtype == STYX_Q4_K ? 144 : 176);
            const int j = i / 64, w = i % 64, l = w % 32, hi = w >= 32;
            float sc, m;
            kq_scale_min(b + 4, 2 * j + hi, sc, m);
            int q;
            if (a.qtype == STYX_Q4_K) {
                q = (b[16 + 32 * j + l] >> (hi ? 4 : 0)) & 0x0F;
            } else {
                q = ((b[48 + 32 * j + l] >> (hi ? 4 : 0)) & 0x0F) + (((b[16 + l] >> (2 * j + hi)) & 1) << 4);
            }
            const float d = rd_f16(b), dmin = rd_f16(b + 2);
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, sc), static_cast<float>(q)), __fmul_rn(dmin, m));
        } else {   // q6_K
            const uint8_t *b = rp + static_cast<size_t>(blk) * 210;
            const int n = i / 128, rr = i % 128, qq = rr / 32, l = rr % 32;
            const uint8_t h = b[128 + 32 * n + l];
            const uint8_t lo = b[64 * n + l + ((qq & 1) ? 32 : 0)];
            const int q = (((qq & 2) ? (lo >> 4) : (lo & 0x0F)) | (((h >> (2 * qq)) & 3) << 4)) - 32;
            const int8_t sc = static_cast<int8_t>(b[192 + 8 * n + l / 16 + 2 * qq]);
            v = __fmul_rn(__fmul_rn(rd_f16(b + 208), static_cast<float>(sc)), static_cast<float>(q));
        }
    }
    a.out[e] = v;
}

// ------------------------------------------------------------ greedy pick
// The index of the largest value under IEEE total order (f32::total_cmp),
// the last one among equals (Iterator::max_by, the greedy pick of
// crates/model/examples/generate_moe.rs:29).  One CTA.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    int b = __float_as_int(v);
    b ^= static_cast<int>(static_cast<unsigned>(b >> 31) >> 1);   // total_cmp's key, compared as signed
    const unsigned u = static_cast<unsigned>(b) ^ 0x80000000u;      // ... as unsigned
    return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned>(i);
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
    if (threadIdx.x < 32) {
#pragma unroll
        for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;   // valid in thread 0
}

// Each CTA reduces a stride of x to one key; the last CTA to finish (a
// ticket counter that wraps back to zero, after a fence) reduces the CTAs'
// keys.  No CTA waits for another.
__global__ void __launch_bounds__(256) k_argmax(const float *x, int n, int32_t *out, unsigned long long *part,
                                                unsigned *ticket) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long red[8];
    __shared__ bool last;
    unsigned long long best = 0;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) best = max(best, argmax_key(x[i], i));
    best = block_max_u64(best, red);
    if (threadIdx.x == 0) {
        part[blockIdx.x] = best;
        __threadfence();
        last = atomicInc(ticket, gridDim.x - 1) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    best = 0;
    for (int b = threadIdx.x; b < gridDim.x; b += 256) best = max(best, __ldcg(part + b));
    __syncthreads();
    best = block_max_u64(best, red);
    if (threadIdx.x == 0) *out = static_cast<int32_t>(best & 0xffffffffu);
}

}  // namespace

cudaError_t launch_get_rows(const GetRowsArgs &a, cudaStream_t st) {
    const long long total = static_cast<long long>(a.n) * a.ncols;
    return launch_pdl(k_get_rows, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, st, a);
}

cudaError_t launch_argmax(const float *x, int n, int32_t *out, void *scratch, cudaStream_t st) {
    auto *part = static_cast<unsigned long long *>(scratch);
    auto *ticket = reinterpret_cast<unsigned *>(part + kArgmaxCtas);
    const int grid = std::min(kArgmaxCtas, std::max(1, (n + 1023) / 1024));
    return launch_pdl(k_argmax, dim3(grid), dim3(256), 0, st, x, n, out, part, ticket);
}

size_t attn_smem_bytes(int gqa, int hd, int tps) {
    return (static_cast<size_t>(attn_acc_offset(gqa, hd, tps)) + static_cast<size_t>(kAttnWarps) * kHeadsPerPass * hd) *
           4;
}

cudaError_t launch_qk_norm_rope_kv(const QkRopeArgs &a, cudaStream_t st) {
    return launch_pdl(k_qk_norm_rope_kv, dim3(a.n_tokens * (a.n_heads + a.n_kv)), dim3(128), 0, st, a);
}

cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st) {
    const size_t smem = attn_smem_bytes(a.gqa, a.hd, a.tps);
    const dim3 grid(a.n_kv, a.n_splits);
    cudaError_t e;
    if (a.hd <= 128) {
        e = cudaFuncSetAttribute(k_attn_split<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = launch_pdl(k_attn_split<1>, grid, dim3(kAttnThreads), smem, st, a);
    } else {
        e = cudaFuncSetAttribute(k_attn_split<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = launch_pdl(k_attn_split<2>, grid, dim3(kAttnThreads), smem, st, a);
    }
    if (e != cudaSuccess) return e;
    return launch_pdl(k_attn_combine, dim3(a.n_kv * a.gqa), dim3(128), 0, st, a);
}

cudaError_t launch_add_f32(const float *x, const float *y, float *d, int n, cudaStream_t st) {
    return launch_pdl(k_add_f32, dim3((n + 255) / 256), dim3(256), 0, st, x, y, d, n);
}

}  // namespace styx
