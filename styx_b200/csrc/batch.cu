// batch.cu -- the MoE block for a batch of B decode tokens (B <= 64) of one
// layer, with the expert matrices on the 5th-generation tensor cores.
//
// At batch 1 every expert byte is used once (the GEMV kernels); at batch B
// the tokens routed to one expert share its bytes, so the expert work
// becomes a small grouped GEMM: M = the expert's weight rows (128-row
// tiles), N = its tokens (padded to 16), K = the row length.  Kernels:
//   1  k_batch_logits  per (token, 8 experts): RMSNorm of x (recomputed by
//                      every CTA of the token, one fixed order), 8 router
//                      rows; x_norm as f16 rows for the GEMMs
//   2  k_batch_lists   one CTA: per token the top-k of topk_softmax_f32.comp
//                      (a warp each), the softmax weights and the id block;
//                      per used expert its (token, slot) pairs in token
//                      order and its slab sources
//   3  k_bgemm<Q, 2>   gate and up: persistent, one CTA per SM
//   4  k_bgemm<Q, 1>   down: the same kernel with one matrix
//   5  k_batch_combine x[b][r] += sum_s w[b][s] d[b][s][r], slot order
//                      (moe_reduce_f32.comp)
//
// The GEMM kernel.  A work unit is (used expert, 128-row tile, K piece):
// the K range of a tile is cut into S pieces when that spreads the units
// more evenly over the SMs (S is a function of the used-expert count only,
// the same in every CTA).  The CTA walks its units' K chunks (one quant
// super-block per row: 256 elements) through a ring of R raw
// stages filled with cp.async (the 128 rows' quant bytes of the chunk and
// the B rows of the unit's tokens, f16, in the canonical K-major layout):
// chunk q + R - 1 is requested while chunk q is consumed.  Each chunk is
// consumed in 64-wide K slices: all threads dequantise the slice's weight
// rows into one of two A slots (f16, canonical K-major layout), then thread
// 0 issues the slice's tcgen05.mma (M 128, N = the unit's tokens rounded to
// 16, K 64) into the TMEM accumulator and commits them to the slot's
// mbarrier, which the slot's next writer waits on.  At a unit's last chunk
// the accumulator goes out: h = SiLU(g) * u as f16 (gate/up) or d as f32
// (down) when S == 1, else f32 partials per piece, which the CTA that
// finishes an item's last piece sums in piece order (gate/up) or the combine
// kernel sums (down): the result does not depend on which CTA ran what.
//
// Dequantisation stays in packed f16 arithmetic: a quant byte q becomes the
// half 1024 + q by OR-ing it into the bits of 1024, then q = that - 1024
// exactly, then d * sc * q - dmin * m in one fused multiply-add.  Splitting a
// 32-bit word of four bytes into two half2 gives the element order
// (0, 2, 1, 3) in every group of four; the B rows (x_norm and h) are stored
// in the same order, so the dot products are unchanged.
//
// Precision: operands are rounded to f16 (11-bit significand), products and
// sums are f32 in TMEM; the block stays within 1e-3 of max|dx| of the f32
// oracle.  No TMA multicast anywhere; each CTA allocates and frees its own
// TMEM columns; every wait is bounded.
#include <cfloat>
#include <cstring>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "moe_common.cuh"

namespace styx {

// ------------------------------------------------------------ tcgen05 helpers
// canonical K-major layout without swizzle: 8-row x 16-byte core matrices;
// the R rows of one 8-element K chunk are contiguous (R * 16 bytes), chunks
// R * 16 bytes apart
__device__ __forceinline__ uint32_t kmaj_off(int r, int k, int R) {
    return static_cast<uint32_t>((k >> 3) * (R * 16) + (r >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
// shared-memory matrix descriptor (sm_100 format, version 1, no swizzle)
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    return d;
}
// instruction descriptor: f16 x f16 -> f32, both operands K-major
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols));
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 8 consecutive f32 columns of this thread's TMEM lane (warp w: lanes 32(w%4)..)
__device__ __forceinline__ void tmem_ld8(uint32_t addr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __uint_as_float(r[j]);
}

// ------------------------------------------------------------ cp.async
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src, uint64_t pol) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most n of this thread's groups are pending (n = 0 .. 6)
__device__ __forceinline__ void cp_async_wait(int n) {
    switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    }
}

// position of element i of a B row (x_norm, h) in memory: positions 1 and
// 2 of every group of four swapped, the order the dequantisation produces
__host__ __device__ __forceinline__ int kperm(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

// ------------------------------------------------------------ 1: logits
// One CTA (256 threads) per (token b, 8 experts).  RMSNorm with the
// reference's expression (rms_norm_f32.comp: x * 1/sqrt(mean(x^2) + eps) *
// w), then warp w takes router row 8 * blockIdx.y + w: float4 lane-strided
// partial sums, a fixed shuffle tree.
constexpr int kLogitThreads = 256;
constexpr int kLogitRows = kLogitThreads / 32;
__global__ void __launch_bounds__(kLogitThreads) k_batch_logits(BatchArgs a) {
    extern __shared__ __align__(16) float xn[];   // [H]
    __shared__ float red[kLogitThreads / 32];
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = a.H;
    const float4 *x4 = reinterpret_cast<const float4 *>(a.x + static_cast<size_t>(b) * H);
    const float4 *w4 = reinterpret_cast<const float4 *>(a.norm_w);
    float ss = 0.f;
    for (int i = tid; i < H / 4; i += kLogitThreads) {
        const float4 v = x4[i];
        reinterpret_cast<float4 *>(xn)[i] = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = lane < kLogitThreads / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 4; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    tot = __shfl_sync(0xffffffffu, tot, 0);
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(H) + a.eps);
    __half *xh = a.xh + static_cast<size_t>(b) * H;
    for (int i = tid; i < H / 4; i += kLogitThreads) {
        float4 v = reinterpret_cast<float4 *>(xn)[i];
        const float4 w = w4[i];
        v.x = v.x * scale * w.x;
        v.y = v.y * scale * w.y;
        v.z = v.z * scale * w.z;
        v.w = v.w * scale * w.w;
        reinterpret_cast<float4 *>(xn)[i] = v;
        if (blockIdx.y == 0) {   // memory order (0, 2, 1, 3)
            const __half2 p0 = __floats2half2_rn(v.x, v.z), p1 = __floats2half2_rn(v.y, v.w);
            reinterpret_cast<__half2 *>(xh)[2 * i] = p0;
            reinterpret_cast<__half2 *>(xh)[2 * i + 1] = p1;
        }
    }
    __syncthreads();
    const int e = blockIdx.y * kLogitRows + warp;
    if (e < a.E) {
        const float4 *r4 = reinterpret_cast<const float4 *>(a.router + static_cast<size_t>(e) * H);
        float acc = 0.f;
#pragma unroll 4
        for (int i = lane; i < H / 4; i += 32) {
            const float4 r = __ldg(r4 + i), v = reinterpret_cast<const float4 *>(xn)[i];
            acc = fmaf(r.x, v.x, acc);
            acc = fmaf(r.y, v.y, acc);
            acc = fmaf(r.z, v.z, acc);
            acc = fmaf(r.w, v.w, acc);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a.logits[static_cast<size_t>(b) * a.E + e] = acc;
    }
}

// ------------------------------------------------------------ 2: routing and expert lists
// One CTA of 1024 threads.  Warp w routes tokens w, w + 32: the top-k of
// the token's logits (warp_pick, moe_common.cuh), the softmax weights of
// topk_softmax_f32.comp:47-52 (renormalised when norm_topk), the id block
// (ids, hot index, arena slot, full index).  Then per expert a 64-bit mask
// of the tokens routed to it (OR is order-free: deterministic); the used
// experts in ascending id with their pair offsets (a block scan); pair
// (b, s) goes to place popc(mask[e] & ((1 << b) - 1)) of its expert, i.e.
// token order; the sources of an expert come from its first token's id row.
constexpr int kListThreads = 1024;
__global__ void __launch_bounds__(kListThreads) k_batch_lists(BatchArgs a) {
    __shared__ unsigned long long mask[STYX_MAX_EXPERTS];
    __shared__ int pos_e[STYX_MAX_EXPERTS];
    __shared__ int pe[STYX_MAX_BATCH * STYX_MAX_TOPK];
    __shared__ int warp_sum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = a.E, k = a.k, P = a.B * a.k;
    for (int e = tid; e < E; e += kListThreads) mask[e] = 0ull;
    for (int i = tid; i < a.n_item_cnt; i += kListThreads) a.item_cnt[i] = 0;
    __syncthreads();
    const int nper = (E + 31) >> 5;
    for (int b = warp; b < a.B; b += kListThreads / 32) {
        const float *lg = a.logits + static_cast<size_t>(b) * E;
        uint32_t key[kLogitRegs];
        float lv[kLogitRegs];
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) {
            lv[j] = (j < nper && lane + 32 * j < E) ? lg[lane + 32 * j] : -INFINITY;
            key[j] = lv[j] > -INFINITY ? order_key(lv[j]) : 0u;
        }
        int e = -1;
        uint32_t ke = 0;
        if (nper <= 4) warp_pick_sorted4(key, k, lane, e, ke);
        else warp_pick<kLogitRegs>(key, k, lane, e, ke);
        float mx = -INFINITY, sum = 0.f;
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) mx = fmaxf(mx, lv[j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++)
            if (j < nper && lane + 32 * j < E) sum += expf(lv[j] - mx);
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float w = (lane < k && ke) ? expf(key_value(ke) - mx) / sum : 0.f;
        float wsum = 0.f;
        for (int t = 0; t < k; t++) wsum += __shfl_sync(0xffffffffu, w, t);
        if (lane < k) {
            a.weights[b * k + lane] = a.renorm ? w / wsum : w;
            int hi = -1, ai = -1, fi = -1;
            const uint32_t hot = (e >= 0 && a.remap) ? a.remap[e] : kSkip;
            if (hot != kSkip) {
                hi = static_cast<int>(hot);
            } else {
                const uint32_t am = (e >= 0 && a.pmap) ? a.pmap[e] : kSkip;
                if (am != kSkip) ai = static_cast<int>(am);
                else fi = e;
            }
            int32_t *ids = a.ids + static_cast<size_t>(b) * kIdsPerLayer;
            ids[lane] = e;
            ids[16 + lane] = hi;
            ids[32 + lane] = ai;
            ids[48 + lane] = fi;
            bool valid = e >= 0 && e < E;
            if (valid) {
                valid = fused_slot_src(a.gate, hi, ai, fi) && fused_slot_src(a.up, hi, ai, fi) &&
                        fused_slot_src(a.down, hi, ai, fi);
                if (!valid && !a.quiet) atomicExch(a.err, kErrBadId);
            }
            pe[b * k + lane] = valid ? e : -1;
            a.pv[b * k + lane] = valid;
            if (valid) atomicOr(&mask[e], 1ull << b);
        }
    }
    __syncthreads();
    // prefix over the used experts (ascending id): one block scan of E <= 1024 flags
    const int cnt = tid < E ? __popcll(mask[tid]) : 0;
    const int used = cnt > 0 ? 1 : 0;
    int iu = used, ic = cnt;   // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u2 = __shfl_up_sync(0xffffffffu, iu, o), c2 = __shfl_up_sync(0xffffffffu, ic, o);
        if (lane >= o) {
            iu += u2;
            ic += c2;
        }
    }
    if (lane == 31) warp_sum[warp] = (iu << 16) | ic;   // used <= 1024, pairs <= 1024
    __syncthreads();
    if (warp == 0) {
        const int v = warp_sum[lane];
        int acc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, acc, o);
            if (lane >= o) acc += t;
        }
        warp_sum[lane] = acc - v;   // exclusive over warps
    }
    __syncthreads();
    const int base = warp_sum[warp];
    const int upos = (base >> 16) + iu - used;      // exclusive position among used experts
    const int poff = (base & 0xFFFF) + ic - cnt;    // first pair of this expert
    if (tid < E) pos_e[tid] = used ? upos : -1;
    if (tid < E && used) {
        a.used_e[upos] = tid;
        a.cnt[upos] = cnt;
        a.off[upos] = poff;
    }
    if (tid == E - 1) {
        *a.n_used = upos + used;
        a.off[upos + used] = poff + cnt;
    }
    __syncthreads();
    for (int p = tid; p < P; p += kListThreads) {
        const int e = pe[p];
        if (e < 0) continue;
        const int b = p / k, s = p - b * k;
        const int rank = __popcll(mask[e] & ((1ull << b) - 1ull));
        const int u = pos_e[e];
        a.pair[a.off[u] + rank] = p;
        if (rank == 0) {
            const int32_t *ids = a.ids + static_cast<size_t>(b) * kIdsPerLayer;
            a.srcs[3 * u + 0] = fused_slot_src(a.gate, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 1] = fused_slot_src(a.up, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 2] = fused_slot_src(a.down, ids[16 + s], ids[32 + s], ids[48 + s]);
        }
    }
}

// ------------------------------------------------------------ quant formats
// per format: elements of one K chunk (one super-block per row), its bytes
// per row, the stage row stride (a multiple of 16 whose quotient by 16 is
// odd: 16-byte reads of 32 consecutive rows are free of bank conflicts), the
// cp.async size (16 where every row chunk starts on a 16-byte boundary; 8
// for q6_K, whose 210-byte blocks start on 2-byte boundaries)
__host__ __device__ constexpr int q_kch(int) { return 256; }
__host__ __device__ constexpr int q_bb(int qt) { return qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : 210; }
__host__ __device__ constexpr int q_rsb(int qt) { return qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : 240; }
__host__ __device__ constexpr int q_cpb(int qt) { return qt == STYX_Q6_K ? 8 : 16; }

__device__ __forceinline__ __half2 u2h2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return h;
}
__device__ __forceinline__ uint32_t h22u(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}
constexpr uint32_t kHalf1024x2 = 0x64006400u;   // the half 1024.0, twice
// four bytes v = (b0, b1, b2, b3), each < 256, as the halves of
// (b0 + 1024 - bias, b2 + ...) and (b1 + ..., b3 + ...) scaled: fma(q, s, c)
__device__ __forceinline__ void bytes4_fma(uint32_t v, __half2 bias, __half2 s, __half2 c, uint32_t &lo,
                                           uint32_t &hi) {
    const uint32_t e02 = (v & 0x00FF00FFu) | kHalf1024x2;
    const uint32_t e13 = ((v >> 8) & 0x00FF00FFu) | kHalf1024x2;
    lo = h22u(__hfma2(__hsub2(u2h2(e02), bias), s, c));
    hi = h22u(__hfma2(__hsub2(u2h2(e13), bias), s, c));
}
// 32 bytes at byte `off` (even) of a stage row, as eight words; the row is
// read with 16-byte loads from off rounded down to 16
__device__ __forceinline__ void run32(const uint8_t *row, int off, uint32_t (&w)[8]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(row + (off & ~15));
    const uint4 A = p[0], B = p[1], C = p[2];
    const uint32_t V[12] = {A.x, A.y, A.z, A.w, B.x, B.y, B.z, B.w, C.x, C.y, C.z, C.w};
    const int bo = off & 15;
    const uint32_t s1 = static_cast<uint32_t>(bo & 4) << 3, sh = static_cast<uint32_t>(bo & 3) << 3;
    const bool two = (bo & 8) != 0;
    uint32_t T1[11];
#pragma unroll
    for (int i = 0; i < 11; i++) T1[i] = __funnelshift_rc(V[i], V[i + 1], s1);
    uint32_t T2[9];
#pragma unroll
    for (int i = 0; i < 9; i++) T2[i] = two ? T1[i + 2] : T1[i];
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = __funnelshift_r(T2[i], T2[i + 1], sh);
}
// the 6-bit scale and min of sub-block j of a q4_K / q5_K super-block
// (the packing of get_scale_min_k4, moe.rs:506-533)
__device__ __forceinline__ void scale_min_k4(const uint8_t *s, int j, float &sc, float &m) {
    if (j < 4) {
        sc = static_cast<float>(s[j] & 63);
        m = static_cast<float>(s[j + 4] & 63);
    } else {
        sc = static_cast<float>((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
        m = static_cast<float>((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}
__device__ __forceinline__ float half_at(const uint8_t *p) {   // 2-byte aligned
    return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(p)));
}

// Elements e0 .. e0 + 31 (e0 % 32 == 0) of a K chunk of one weight row, from
// its stage row (quant data at byte `o`), dequantised to f16 and written as
// four 16-byte groups of eight to `dst` (the A slot, rows 128 apart per K
// group: kmaj_off(r, k0 + 8 i, 128)); element order (0, 2, 1, 3) per four.
// The value of each element is the reference's d * sc * q - dmin * m
// (q4_K / q5_K), d * sc * (q - 32) (q6_K).
template <int QT>
__device__ __forceinline__ void deq32(const uint8_t *row, int o, int e0, uint8_t *slot, int r, int k0) {
    uint32_t out[16];
    if constexpr (QT == STYX_Q4_K || QT == STYX_Q5_K) {
        // d * sc * q - dmin * m with one systematic error removed: t = sc * q
        // is an integer below 2048, exact in f16; d is the stored half; the
        // min term c = dmin * m (exact in f32) goes in as c_hi + c_lo, so
        // the element is round(round(d * t - c_hi) - c_lo) and no rounding
        // is shared by the 32 elements of a sub-block
        const int sb = e0 >> 5, j = sb >> 1, hi = sb & 1;
        const uint32_t hd = *reinterpret_cast<const uint32_t *>(row);
        const __half dh = __ushort_as_half(static_cast<unsigned short>(hd & 0xFFFFu));
        const float dm = __half2float(__ushort_as_half(static_cast<unsigned short>(hd >> 16)));
        float sc, mn;
        scale_min_k4(row + 4, sb, sc, mn);
        const float c = dm * mn;
        const __half chi = __float2half_rn(c);
        const __half clo = __float2half_rn(c - __half2float(chi));
        const __half2 d2 = __half2half2(dh), nchi2 = __half2half2(__hneg(chi)), clo2 = __half2half2(clo);
        const __half2 sc2 = __float2half2_rn(sc), nsc1024 = __float2half2_rn(-1024.0f * sc);
        const __half2 k1024 = u2h2(kHalf1024x2);
        constexpr int QS = QT == STYX_Q4_K ? 16 : 48;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(row + QS + 32 * j);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(row + QS + 32 * j + 16);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t h5[8];
        if constexpr (QT == STYX_Q5_K) {
            const uint4 h0 = *reinterpret_cast<const uint4 *>(row + 16);
            const uint4 h1 = *reinterpret_cast<const uint4 *>(row + 32);
            const uint32_t hb[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) h5[i] = ((hb[i] >> sb) & 0x01010101u) << 4;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t v = (w[i] >> (4 * hi)) & 0x0F0F0F0Fu;
            if constexpr (QT == STYX_Q5_K) v |= h5[i];
            const uint32_t e02 = (v & 0x00FF00FFu) | kHalf1024x2, e13 = ((v >> 8) & 0x00FF00FFu) | kHalf1024x2;
            __half2 t02, t13;
            if constexpr (QT == STYX_Q4_K) {   // (1024 + q) * sc - 1024 * sc: below 65504 throughout
                t02 = __hfma2(u2h2(e02), sc2, nsc1024);
                t13 = __hfma2(u2h2(e13), sc2, nsc1024);
            } else {                           // q up to 31: subtract first
                t02 = __hmul2(__hsub2(u2h2(e02), k1024), sc2);
                t13 = __hmul2(__hsub2(u2h2(e13), k1024), sc2);
            }
            out[2 * i] = h22u(__hsub2(__hfma2(t02, d2, nchi2), clo2));
            out[2 * i + 1] = h22u(__hsub2(__hfma2(t13, d2, nchi2), clo2));
        }
    } else if constexpr (QT == STYX_Q6_K) {
        const int n = e0 >> 7, qd = (e0 & 127) >> 5;
        uint32_t ql[8], qh[8];
        run32(row, o + 64 * n + 32 * (qd & 1), ql);
        run32(row, o + 128 + 32 * n, qh);
        const float d = half_at(row + o + 208);
        const int8_t *scp = reinterpret_cast<const int8_t *>(row + o + 192 + 8 * n + 2 * qd);
        const __half2 s0 = __float2half2_rn(d * static_cast<float>(scp[0]));
        const __half2 s1 = __float2half2_rn(d * static_cast<float>(scp[1]));
        const __half2 bias = u2h2(0x64206420u);   // 1024 + 32
        const __half2 zero = u2h2(0u);
        const int s4 = 4 * (qd >> 1), sq = 2 * qd;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t v = ((ql[i] >> s4) & 0x0F0F0F0Fu) | (((qh[i] >> sq) & 0x03030303u) << 4);
            bytes4_fma(v, bias, i < 4 ? s0 : s1, zero, out[2 * i], out[2 * i + 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
        *reinterpret_cast<uint4 *>(slot + kmaj_off(r, k0 + 8 * i, 128)) =
            make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
}

// ------------------------------------------------------------ 3, 4: grouped GEMMs
// The number of K pieces S of every (expert, tile) item: the divisor of the
// chunk count (at most smax) that gives the busiest CTA the fewest chunks,
// the smallest such.  A function of the item count, so every CTA (and the
// combine kernel) computes the same S.
__host__ __device__ inline int choose_split(int n_items, int nk, int G, int smax) {
    int best = 1;
    long long best_cost = -1;
    for (int s = 1; s <= nk && s <= smax; s++) {
        if (nk % s) continue;
        const long long units = static_cast<long long>(n_items) * s;
        const long long cost = ((units + G - 1) / G) * (nk / s);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int n) { return n <= 32 ? 32u : n <= 64 ? 64u : 128u; }

// One side of the block: gate + up (NM = 2) or down (NM = 1).
struct GemmSide {
    int K, M, rb;            // row length, rows of one expert matrix, bytes of a row
    int mat0;                // srcs index of the first matrix (0: gate, up; 2: down)
    const __half *bsrc;      // B rows: x_norm [B][K] (by token) or h [P][K] (by pair)
    int by_token;
    float *part0, *part1;    // f32 partials [smax][P][M] per matrix (down: part0 piece 0 = d)
    int npm;                 // B rows a stage holds (tokens of one expert, padded to 16)
    int stages;              // R
    int smax;
    int *split_out;          // the S this launch used
};

// What a stage's chunk is: written by thread 0 when the chunk's copies are
// issued, read by every thread after the chunk-start barrier.
struct ChunkMeta {
    const uint8_t *src0, *src1;   // the unit's matrices (row 0 of the tile, chunk 0)
    int N, p0, u, tile, piece, kc, first, last;
};

template <int QT, int NM>
__global__ void __launch_bounds__(256 * NM, 1) k_bgemm(BatchArgs a, GemmSide g) {
    constexpr int T = 256 * NM;
    constexpr int KCH = q_kch(QT), BB = q_bb(QT), RSB = q_rsb(QT), CPB = q_cpb(QT);
    constexpr int NPC = CPB == 16 ? BB / 16 : (BB + 6 + 7) / 8;   // copies per stage row, at most
    constexpr int SLICES = KCH / 64;
    constexpr int JB = SLICES > 2 ? 2 : 1;                       // slice that issues the B rows
    constexpr int ASLOT = NM * 128 * 64 * 2;
    constexpr int BITEMS = (64 * (KCH / 8) + T - 1) / T;         // B copies per thread, at most
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar[2];
    __shared__ uint32_t tbase;
    __shared__ int s_fin;
    __shared__ ChunkMeta meta[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    const int n_used = *a.n_used;
    const int tiles = g.M / 128, nk = g.K / KCH, P = a.B * a.k;
    const int n_items = n_used * tiles;
    const int S = choose_split(n_items, nk, G, g.smax);
    if (cta == 0 && tid == 0) *g.split_out = S;
    const int CPU = nk / S;   // chunks of one unit
    const int n_units = n_items * S;
    const int my_units = cta < n_units ? (n_units - 1 - cta) / G + 1 : 0;
    if (my_units == 0) return;   // the whole CTA, before any barrier or TMEM use
    const int Q = my_units * CPU;
    const int Npm = g.npm, R = g.stages;
    const int stage_w = NM * 128 * RSB, stage_bytes = stage_w + Npm * KCH * 2;
    uint8_t *slots = sm, *stages = sm + 2 * ASLOT;
    const uint32_t tcols = tmem_cols_for(NM * Npm);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncwarp();   // lane 0 of warp 0 took the branch above; .sync.aligned needs the whole warp
    if (warp == 0) {
        tmem_alloc(&tbase, tcols);
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tbase;
    const uint64_t pol_w = l2_evict_first(), pol_b = l2_evict_last();

    // ---- chunk q -> its unit; the unit's tables (read-only in this kernel)
    auto meta_of = [&](int q) {
        ChunkMeta x;
        const int vi = q / CPU, cq = q - vi * CPU;
        const int v = cta + vi * G, item = v / S;
        x.piece = v - item * S;
        x.u = item / tiles;
        x.tile = item - x.u * tiles;
        x.kc = x.piece * CPU + cq;
        x.first = cq == 0;
        x.last = cq == CPU - 1;
        x.N = __ldg(a.cnt + x.u);
        x.p0 = __ldg(a.off + x.u);
        const size_t at = static_cast<size_t>(x.tile) * 128 * g.rb;
        x.src0 = a.srcs[3 * x.u + g.mat0] + at;
        x.src1 = NM == 2 ? a.srcs[3 * x.u + g.mat0 + 1] + at : x.src0;
        return x;
    };
    // the weight rows of chunk x into stage st (no loads besides the copies)
    auto issue_w = [&](const ChunkMeta &x, uint8_t *st) {
        const size_t kb = static_cast<size_t>(x.kc) * BB;
        for (int i = tid; i < NM * 128 * NPC; i += T) {
            const int m = i / (128 * NPC), rem = i - m * (128 * NPC), r = rem / NPC, pc = rem - r * NPC;
            const uint8_t *rs = (m ? x.src1 : x.src0) + static_cast<size_t>(r) * g.rb + kb;
            uint8_t *dst = st + (m * 128 + r) * RSB + pc * CPB;
            if constexpr (CPB == 16) {
                cp_async16(dst, rs + pc * 16, pol_w);
            } else {
                const int o = static_cast<int>(reinterpret_cast<uintptr_t>(rs) & 7);
                if (pc * 8 < o + BB) cp_async8(dst, rs - o + pc * 8, pol_w);
            }
        }
    };
    // this thread's B-row pairs of chunk x (loads issued early, used by issue_b)
    auto b_pairs = [&](const ChunkMeta &x, int (&pr)[BITEMS]) {
#pragma unroll
        for (int t = 0; t < BITEMS; t++) {
            const int n = (tid + t * T) / (KCH / 8);
            pr[t] = n < x.N ? __ldg(a.pair + x.p0 + n) : -1;
        }
    };
    auto issue_b = [&](const ChunkMeta &x, uint8_t *st, const int (&pr)[BITEMS]) {
        const int Np = max(16, (x.N + 15) & ~15);
        uint8_t *sb = st + stage_w;
#pragma unroll
        for (int t = 0; t < BITEMS; t++) {
            const int i = tid + t * T, n = i / (KCH / 8), kp = i - n * (KCH / 8);
            if (n >= Np) continue;
            uint8_t *dst = sb + kmaj_off(n, kp * 8, Npm);
            if (pr[t] >= 0) {
                const int row = g.by_token ? pr[t] / a.k : pr[t];
                cp_async16(dst, g.bsrc + static_cast<size_t>(row) * g.K + static_cast<size_t>(x.kc) * KCH + kp * 8,
                           pol_b);
            } else {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };

    // prologue: chunks 0 .. R - 2, one group each
    for (int q = 0; q < R - 1; q++) {
        if (q < Q) {
            const ChunkMeta x = meta_of(q);
            uint8_t *st = stages + (q % R) * stage_bytes;
            int pr[BITEMS];
            b_pairs(x, pr);
            issue_w(x, st);
            issue_b(x, st, pr);
            if (tid == 0) meta[q % R] = x;
        }
        cp_async_commit();
    }
    bool ok = true;
    int gs = 0;   // slices issued so far
    // dequantisation: thread -> (matrix, row, half of the 64-wide slice)
    const int dm = (tid >> 7) % NM, dr = tid & 127, dh = tid / (128 * NM);
    for (int q = 0; q < Q; q++) {
        cp_async_wait(R - 2);
        __syncthreads();
        const ChunkMeta x = meta[q % R];
        // the chunk R - 1 ahead: its tables now, its copies from slice 1 on
        const int qn = q + R - 1;
        const bool have_n = qn < Q;
        ChunkMeta xn{};
        if (have_n) xn = meta_of(qn);
        int prn[BITEMS];
        const int Np = max(16, (x.N + 15) & ~15);
        const uint8_t *st = stages + (q % R) * stage_bytes;
        uint8_t *stn = stages + (qn % R) * stage_bytes;
        const uint8_t *drow = st + (dm * 128 + dr) * RSB;
        int o = 0;
        if constexpr (CPB == 8)
            o = static_cast<int>((reinterpret_cast<uintptr_t>(dm ? x.src1 : x.src0) + static_cast<size_t>(dr) * g.rb +
                                  static_cast<size_t>(x.kc) * BB) & 7);
        const uint32_t sB = smem_addr(st + stage_w);
#pragma unroll 1
        for (int j = 0; j < SLICES; j++, gs++) {
            const int slot = gs & 1;
            // the slot's previous MMAs (slice gs - 2, and all before it) done
            if (gs >= 2 && ok) ok = mbar_wait(&bar[slot], static_cast<uint32_t>(((gs >> 1) - 1) & 1), a.err, kErrWaitFull);
            if (j == 1 && have_n) {   // into chunk q - 1's stage: its MMAs are done
                issue_w(xn, stn);
                b_pairs(xn, prn);
                if (tid == 0) meta[qn % R] = xn;
            }
            if (j == JB) {
                if (have_n) issue_b(xn, stn, prn);
                cp_async_commit();
            }
            deq32<QT>(drow, o, 64 * j + 32 * dh, slots + slot * ASLOT + dm * (128 * 64 * 2), dr, 32 * dh);
            fence_async_smem();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t idesc = umma_idesc_f16(128, Np);
                const uint32_t sA = smem_addr(slots + slot * ASLOT);
#pragma unroll
                for (int m = 0; m < NM; m++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t da = umma_desc(sA + m * (128 * 64 * 2) + kk * 2 * 2048, 2048, 128);
                        const uint64_t db = umma_desc(sB + (j * 8 + kk * 2) * Npm * 16, Npm * 16, 128);
                        umma_f16(tmem + m * Npm, da, db, idesc, (x.first && j == 0 && kk == 0) ? 0u : 1u);
                    }
                umma_commit(&bar[slot]);
            }
        }
        if (!x.last) continue;
        // ---- the unit's accumulator out
        {
            const int lg = gs - 1;
            if (ok) ok = mbar_wait(&bar[lg & 1], static_cast<uint32_t>((lg >> 1) & 1), a.err, kErrWaitFull);
        }
        // the lanes of a warp may leave the (suspending) wait at different
        // times: reconverge before the .sync.aligned TMEM loads
        __syncwarp();
        tc_fence_after();
        const int N = x.N, p0 = x.p0;
        const int row = x.tile * 128 + 32 * (warp & 3) + lane;   // TMEM lane = weight row
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        for (int c = (warp >> 2) * 8; c < Np; c += (T / 128) * 8) {
            float v0[8], v1[8];
            tmem_ld8(tmem + lane_base + c, v0);
            if constexpr (NM == 2) tmem_ld8(tmem + lane_base + Npm + c, v1);
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
                const int n = c + jj;
                if (n >= N) continue;
                const int p = __ldg(a.pair + p0 + n);
                if constexpr (NM == 2) {
                    if (S == 1) {
                        // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
                        const float hv = ok ? v0[jj] / (1.0f + expf(-v0[jj])) * v1[jj] : 0.f;
                        a.h[static_cast<size_t>(p) * g.M + kperm(row)] = __float2half_rn(hv);
                    } else {
                        const size_t at = (static_cast<size_t>(x.piece) * P + p) * g.M + row;
                        g.part0[at] = ok ? v0[jj] : 0.f;
                        g.part1[at] = ok ? v1[jj] : 0.f;
                    }
                } else {
                    g.part0[(static_cast<size_t>(x.piece) * P + p) * g.M + row] = ok ? v0[jj] : 0.f;
                }
            }
        }
        tc_fence_before();
        if constexpr (NM == 2) {
            if (S > 1) {   // the item's last piece sums the pieces in order
                __syncthreads();   // every partial of this piece stored
                if (tid == 0) {
                    __threadfence();
                    s_fin = atomicAdd(&a.item_cnt[x.u * tiles + x.tile], 1) == S - 1;
                    __threadfence();
                }
                __syncthreads();
                if (s_fin) {
                    for (int i = tid; i < 128 * N; i += T) {
                        const int n = i >> 7, rr = x.tile * 128 + (i & 127);
                        const int p = __ldg(a.pair + p0 + n);
                        float gsum = 0.f, usum = 0.f;
                        for (int s = 0; s < S; s++) {
                            const size_t at = (static_cast<size_t>(s) * P + p) * g.M + rr;
                            gsum += __ldcg(g.part0 + at);
                            usum += __ldcg(g.part1 + at);
                        }
                        a.h[static_cast<size_t>(p) * g.M + kperm(rr)] =
                            __float2half_rn(gsum / (1.0f + expf(-gsum)) * usum);
                    }
                }
            }
        }
    }
    __syncthreads();
    __syncwarp();
    if (warp == 0) tmem_dealloc(tmem, tcols);
}

// ------------------------------------------------------------ 5: combine
// x[b][r] += sum_s w[b][s] * d[b][s][r], the slot-ordered sum of
// moe_reduce_f32.comp:8-13 (a slot without an expert adds nothing); d of a
// pair is the sum of its down pieces in piece order
__global__ void k_batch_combine(BatchArgs a) {
    const int b = blockIdx.y, r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.H) return;
    const int S = *a.split_d, P = a.B * a.k;
    float acc = 0.f;
    for (int s = 0; s < a.k; s++) {
        const int p = b * a.k + s;
        if (!a.pv[p]) continue;
        float dv = a.d[static_cast<size_t>(p) * a.H + r];
        for (int piece = 1; piece < S; piece++) dv += a.d[(static_cast<size_t>(piece) * P + p) * a.H + r];
        acc = __fadd_rn(acc, __fmul_rn(a.weights[p], dv));
    }
    float *x = a.x + static_cast<size_t>(b) * a.H + r;
    *x = __fadd_rn(*x, acc);
}

// ------------------------------------------------------------ launchers
// q8_0 is not taken: its instantiation raised an illegal-instruction fault
// at the smallest shape tried (hidden 512, FFN 256, 32 experts, top-4,
// batch 1) whose cause is not known; it stays off the GPU.
bool batch_supported(int qg, int qd) {
    auto ok = [](int q) { return q == STYX_Q4_K || q == STYX_Q5_K || q == STYX_Q6_K; };
    return ok(qg) && ok(qd);
}

int batch_split_max(int K) { return K / 128 < 8 ? K / 128 : 8; }

constexpr int kSmemCap = 232448 - 1024;   // 227 KB per CTA, less the static barriers

template <int QT, int NM>
static cudaError_t launch_bgemm(const BatchArgs &a, GemmSide g, cudaStream_t st) {
    constexpr int KCH = q_kch(QT), RSB = q_rsb(QT);
    const int stage_bytes = NM * 128 * RSB + g.npm * KCH * 2;
    const int slots = 2 * NM * 128 * 64 * 2;
    int R = (kSmemCap - slots) / stage_bytes;
    if (R > 4) R = 4;
    if (R < 2) return cudaErrorInvalidValue;
    g.stages = R;
    const int smem = slots + R * stage_bytes;
    cudaError_t e = cudaFuncSetAttribute(k_bgemm<QT, NM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_bgemm<QT, NM><<<a.sms, 256 * NM, smem, st>>>(a, g);
    return cudaGetLastError();
}

template <int NM>
static cudaError_t launch_bgemm_q(int qt, const BatchArgs &a, const GemmSide &g, cudaStream_t st) {
    switch (qt) {
    case STYX_Q4_K: return launch_bgemm<STYX_Q4_K, NM>(a, g, st);
    case STYX_Q5_K: return launch_bgemm<STYX_Q5_K, NM>(a, g, st);
    case STYX_Q6_K: return launch_bgemm<STYX_Q6_K, NM>(a, g, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_batch(const BatchArgs &a, int qg, int qd, cudaStream_t st) {
    k_batch_logits<<<dim3(a.B, (a.E + kLogitRows - 1) / kLogitRows), kLogitThreads, static_cast<size_t>(a.H) * 4, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_batch_lists<<<1, kListThreads, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int npm = a.B >= 64 ? 64 : ((a.B + 15) & ~15);
    GemmSide gu{};
    gu.K = a.H;
    gu.M = a.F;
    gu.rb = a.rb_g;
    gu.mat0 = 0;
    gu.bsrc = a.xh;
    gu.by_token = 1;
    gu.part0 = a.gpart;
    gu.part1 = a.upart;
    gu.npm = npm;
    gu.smax = batch_split_max(a.H);
    gu.split_out = a.split_d + 1;
    if ((e = launch_bgemm_q<2>(qg, a, gu, st)) != cudaSuccess) return e;
    GemmSide dn{};
    dn.K = a.F;
    dn.M = a.H;
    dn.rb = a.rb_d;
    dn.mat0 = 2;
    dn.bsrc = a.h;
    dn.by_token = 0;
    dn.part0 = a.d;
    dn.part1 = nullptr;
    dn.npm = npm;
    dn.smax = batch_split_max(a.F);
    dn.split_out = a.split_d;
    if ((e = launch_bgemm_q<1>(qd, a, dn, st)) != cudaSuccess) return e;
    k_batch_combine<<<dim3((a.H + 255) / 256, a.B), 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace styx
