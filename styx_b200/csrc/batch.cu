// batch.cu -- the MoE block for a batch of B decode tokens (B <= 64) of one
// layer, with the expert matrices on the 5th-generation tensor cores.
//
// At batch 1 every expert byte is used once (the GEMV kernels); at batch B
// the tokens routed to one expert share its bytes, so the expert work
// becomes a small grouped GEMM: M = the expert's weight rows (128-row
// tiles), N = its tokens (padded to 16), K = the row length.  Kernels:
//   1  k_batch_route   one CTA per token: RMSNorm, router logits, the
//                      top-k of topk_softmax_f32.comp (warp reductions),
//                      softmax weights, the id block; x_norm as f16 rows
//   2  k_batch_lists   one warp: per used expert its (token, slot) pairs,
//                      in token-major order, and its slab sources
//   3  k_batch_gateup  per (used expert, 128-row tile of F): gate and up
//                      rows of the tile dequantised to f16 in shared memory
//                      (the canonical K-major layout), x_norm rows of the
//                      expert's tokens as the B operand, tcgen05.mma into
//                      two TMEM accumulators, epilogue SiLU(g) * u -> h (f16)
//   4  k_batch_down    per (used expert, 128-row tile of H): down rows as
//                      f16, the pairs' h rows as the B operand, -> d (f32)
//   5  k_batch_combine x[b][r] += sum_s w[b][s] d[b][s][r], slot order
//                      (moe_reduce_f32.comp)
// Precision: operands are rounded to f16 (11-bit significand), products and
// sums are f32 in TMEM; the block stays within 1e-3 of max|dx| of the f32
// oracle.  No TMA multicast anywhere; each CTA allocates and frees its own
// TMEM columns; every wait is bounded.
#include <cfloat>
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

// ------------------------------------------------------------ 1: routing
// One CTA (256 threads) per token.  Logits: warp w takes rows e = w, w + 8,
// ...: lane-strided partial sums over the row, then a fixed shuffle tree
// (one fixed order, the same in every run).  The top-k is warp 0's
// selection (moe_common.cuh), the weights the softmax of
// topk_softmax_f32.comp:47-52.
constexpr int kRouteThreads = 256;
__global__ void __launch_bounds__(kRouteThreads) k_batch_route(BatchArgs a) {
    extern __shared__ __align__(16) float rsm[];
    float *xn = rsm;                 // [H]
    float *lg = xn + a.H;            // [E]
    __shared__ float red[32];
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = a.H, E = a.E, k = a.k;
    const float *x = a.x + static_cast<size_t>(b) * H;
    float ss = 0.f;
    for (int i = tid; i < H; i += kRouteThreads) {
        const float v = x[i];
        xn[i] = v;
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = lane < kRouteThreads / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 4; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    tot = __shfl_sync(0xffffffffu, tot, 0);
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(H) + a.eps);
    __half *xh = a.xh + static_cast<size_t>(b) * H;
    for (int i = tid; i < H; i += kRouteThreads) {
        const float v = xn[i] * scale * a.norm_w[i];
        xn[i] = v;
        xh[i] = __float2half_rn(v);
    }
    __syncthreads();
    for (int e = warp; e < E; e += kRouteThreads / 32) {
        const float *r = a.router + static_cast<size_t>(e) * H;
        float acc = 0.f;
        for (int i = lane; i < H; i += 32) acc = fmaf(r[i], xn[i], acc);
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) lg[e] = acc;
    }
    __syncthreads();
    if (warp == 0) {
        const int nper = (E + 31) >> 5;
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
        int32_t *ids = a.ids + static_cast<size_t>(b) * kIdsPerLayer;
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
            ids[lane] = e;
            ids[16 + lane] = hi;
            ids[32 + lane] = ai;
            ids[48 + lane] = fi;
        }
    }
}
// ------------------------------------------------------------ 2: expert lists
// One CTA of 1024 threads.  Pair p = b * k + s (token-major).  Per expert:
// how many pairs route to it (shared atomics on integers: deterministic),
// the used experts in ascending id with their pair offsets (a prefix sum),
// each pair's place = the number of earlier pairs of the same expert (a
// scan over p' < p, so the order inside an expert is token-major), and the
// expert's slab sources (resolved from a pair's id rows: hot, arena, full).
constexpr int kListThreads = 1024;
__global__ void __launch_bounds__(kListThreads) k_batch_lists(BatchArgs a) {
    __shared__ int cnt_e[STYX_MAX_EXPERTS];
    __shared__ int pos_e[STYX_MAX_EXPERTS];   // list position of expert e (or -1)
    __shared__ int warp_sum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = a.E, k = a.k, P = a.B * a.k;
    for (int e = tid; e < E; e += kListThreads) cnt_e[e] = 0;
    __syncthreads();
    auto pair_expert = [&](int p) -> int {
        const int b = p / k, s = p - b * k;
        const int32_t *ids = a.ids + static_cast<size_t>(b) * kIdsPerLayer;
        const int e = ids[s];
        if (e < 0 || e >= E) return -1;
        const uint8_t *sg = fused_slot_src(a.gate, ids[16 + s], ids[32 + s], ids[48 + s]);
        const uint8_t *su = fused_slot_src(a.up, ids[16 + s], ids[32 + s], ids[48 + s]);
        const uint8_t *sd = fused_slot_src(a.down, ids[16 + s], ids[32 + s], ids[48 + s]);
        if (!sg || !su || !sd) {
            if (!a.quiet) atomicExch(a.err, kErrBadId);
            return -1;
        }
        return e;
    };
    for (int p = tid; p < P; p += kListThreads) {
        const int e = pair_expert(p);
        a.pv[p] = e >= 0;
        if (e >= 0) atomicAdd(&cnt_e[e], 1);
    }
    __syncthreads();
    // prefix over the used experts (ascending id): one block scan of E <= 1024 flags
    const int used = (tid < E && cnt_e[tid] > 0) ? 1 : 0;
    const int cnt = tid < E ? cnt_e[tid] : 0;
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
        int v = warp_sum[lane], acc = v;
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
    if (tid == E - 1 || (E > kListThreads && tid == kListThreads - 1)) {
        *a.n_used = upos + used;
        a.off[upos + used] = poff + cnt;
    }
    __syncthreads();
    for (int p = tid; p < P; p += kListThreads) {
        if (!a.pv[p]) continue;
        const int b = p / k, s = p - b * k;
        const int e = a.ids[static_cast<size_t>(b) * kIdsPerLayer + s];
        int before = 0;
        for (int q = 0; q < p; q++) {
            const int bq = q / k, sq = q - bq * k;
            before += (a.pv[q] && a.ids[static_cast<size_t>(bq) * kIdsPerLayer + sq] == e) ? 1 : 0;
        }
        const int u = pos_e[e];
        a.pair[a.off[u] + before] = p;
        if (before == 0) {   // the expert's sources, from this pair's id rows
            const int32_t *ids = a.ids + static_cast<size_t>(b) * kIdsPerLayer;
            a.srcs[3 * u + 0] = fused_slot_src(a.gate, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 1] = fused_slot_src(a.up, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 2] = fused_slot_src(a.down, ids[16 + s], ids[32 + s], ids[48 + s]);
        }
    }
}

// ------------------------------------------------------------ dequantisation
// eight consecutive elements k0..k0+7 (k0 % 8 == 0) of a quantised row, as
// f32, in the reference's expression d*sc*q - dmin*m (moe.rs:506-533) and the
// public block layouts of q5_K / q6_K / q8_0; read with byte loads (q6_K and
// q8_0 blocks are only 2-byte aligned)
__device__ __forceinline__ void scale_min_k4(const uint8_t *s, int j, float &sc, float &m) {
    if (j < 4) {
        sc = static_cast<float>(s[j] & 63);
        m = static_cast<float>(s[j + 4] & 63);
    } else {
        sc = static_cast<float>((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
        m = static_cast<float>((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}
template <int QT>
__device__ __forceinline__ void deq8(const uint8_t *row, int k0, float (&o)[8]) {
    if constexpr (QT == STYX_Q4_K || QT == STYX_Q5_K) {
        constexpr int BB = QT == STYX_Q4_K ? 144 : 176;
        const uint8_t *blk = row + (k0 >> 8) * BB;
        const int kb = k0 & 255, j = kb >> 6, hi = (kb >> 5) & 1, l = kb & 31;
        const float d = __half2float(*reinterpret_cast<const __half *>(blk));
        const float dm = __half2float(*reinterpret_cast<const __half *>(blk + 2));
        float sc, mn;
        scale_min_k4(blk + 4, 2 * j + hi, sc, mn);
        const float a = d * sc, c = dm * mn;
        const uint8_t *qs = blk + (QT == STYX_Q4_K ? 16 : 48) + 32 * j + l;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int q = hi ? (qs[i] >> 4) : (qs[i] & 0xF);
            if constexpr (QT == STYX_Q5_K) q += ((blk[16 + l + i] >> (2 * j + hi)) & 1) << 4;
            o[i] = a * static_cast<float>(q) - c;
        }
    } else if constexpr (QT == STYX_Q6_K) {
        const uint8_t *blk = row + (k0 >> 8) * 210;
        const int kb = k0 & 255, n = kb >> 7, r = kb & 127, q = r >> 5, l = r & 31;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[208] | (blk[209] << 8))));
        const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + 8 * n + (l >> 4) + 2 * q]));
        const uint8_t *ql = blk + 64 * n + 32 * (q & 1) + l;
        const uint8_t *qh = blk + 128 + 32 * n + l;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int lo = (q >> 1) ? (ql[i] >> 4) : (ql[i] & 0xF);
            const int v = (lo | (((qh[i] >> (2 * q)) & 3) << 4)) - 32;
            o[i] = d * sc * static_cast<float>(v);
        }
    } else {   // q8_0
        const uint8_t *blk = row + (k0 >> 5) * 34;
        const int l = k0 & 31;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = d * static_cast<float>(static_cast<int8_t>(blk[2 + l + i]));
    }
}
__device__ __forceinline__ uint4 pack8_f16(const float (&v)[8]) {
    uint4 r;
    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
    __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
    r.x = *reinterpret_cast<uint32_t *>(&h0);
    r.y = *reinterpret_cast<uint32_t *>(&h1);
    r.z = *reinterpret_cast<uint32_t *>(&h2);
    r.w = *reinterpret_cast<uint32_t *>(&h3);
    return r;
}
// ------------------------------------------------------------ 3, 4: grouped GEMMs
// One CTA (256 threads) per (used expert, 128-row weight tile).  Per K chunk
// of 256 the CTA dequantises its 128 weight rows to f16 into shared memory
// (thread t: row t / 2, half of the chunk t % 2, eight elements per 16-byte
// store), copies the B rows (one per pair of the expert, zero rows up to Np),
// and thread 0 issues the K / 16 UMMAs of the chunk and commits them to an
// mbarrier that every thread waits on before the buffers are refilled.  The
// accumulators (TMEM lane = weight row, column = pair) are read by warps 0-3
// with tcgen05.ld.
constexpr int kGemmThreads = 256;
constexpr int kKC = 256;          // K per chunk
constexpr int kMaxPairs = 64;     // pairs of one expert (N), = the largest batch

__device__ __forceinline__ bool batch_wait(uint64_t *bar, uint32_t parity, int *err) {
    return mbar_wait(bar, parity, err, kErrWaitFull);
}

template <int QG>
__global__ void __launch_bounds__(kGemmThreads, 1) k_batch_gateup(BatchArgs a) {
    extern __shared__ __align__(1024) uint8_t gsm[];
    uint8_t *sAg = gsm, *sAu = gsm + 128 * kKC * 2, *sB = sAu + 128 * kKC * 2;
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int tiles = a.F / 128;
    const int u = blockIdx.x / tiles, tile = blockIdx.x - u * tiles;
    if (u >= *a.n_used) return;   // the same for the whole CTA, before any TMEM use
    const int N = a.cnt[u], Np = max(16, (N + 15) & ~15), p0 = a.off[u];
    const uint8_t *sg = a.srcs[3 * u], *su = a.srcs[3 * u + 1];
    const int tid = threadIdx.x, warp = tid >> 5, row0 = tile * 128;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tbase, 128);   // gate columns [0, 64), up [64, 128)
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tbase;
    bool ok = true;
    for (int kc = 0; kc < a.H / kKC; kc++) {
        {
            const int r = tid >> 1, half = tid & 1;
            const uint8_t *grow = sg + static_cast<size_t>(row0 + r) * a.rb_g;
            const uint8_t *urow = su + static_cast<size_t>(row0 + r) * a.rb_g;
#pragma unroll 2
            for (int pc = 0; pc < 16; pc++) {
                const int kk = half * 128 + pc * 8;
                float v[8];
                deq8<QG>(grow, kc * kKC + kk, v);
                *reinterpret_cast<uint4 *>(sAg + kmaj_off(r, kk, 128)) = pack8_f16(v);
                deq8<QG>(urow, kc * kKC + kk, v);
                *reinterpret_cast<uint4 *>(sAu + kmaj_off(r, kk, 128)) = pack8_f16(v);
            }
        }
        for (int i = tid; i < Np * (kKC / 8); i += kGemmThreads) {
            const int n = i / (kKC / 8), kk = (i % (kKC / 8)) * 8;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (n < N) {
                const int b = a.pair[p0 + n] / a.k;
                v = *reinterpret_cast<const uint4 *>(a.xh + static_cast<size_t>(b) * a.H + kc * kKC + kk);
            }
            *reinterpret_cast<uint4 *>(sB + kmaj_off(n, kk, Np)) = v;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0) {
            const uint32_t idesc = umma_idesc_f16(128, Np);
            for (int ks = 0; ks < kKC / 16; ks++) {
                const uint64_t dg = umma_desc(smem_addr(sAg) + ks * 2 * 128 * 16, 128 * 16, 128);
                const uint64_t du = umma_desc(smem_addr(sAu) + ks * 2 * 128 * 16, 128 * 16, 128);
                const uint64_t db = umma_desc(smem_addr(sB) + ks * 2 * Np * 16, Np * 16, 128);
                const uint32_t acc = (kc | ks) != 0;
                umma_f16(tmem, dg, db, idesc, acc);
                umma_f16(tmem + 64, du, db, idesc, acc);
            }
            umma_commit(&bar);
        }
        if (ok) ok = batch_wait(&bar, static_cast<uint32_t>(kc & 1), a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    if (tid < 128) {   // warps 0-3: TMEM lane = row tid
        const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
        for (int c = 0; c < Np; c += 8) {
            float g[8], up[8];
            tmem_ld8(tmem + lane_base + c, g);
            tmem_ld8(tmem + lane_base + 64 + c, up);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int n = c + j;
                if (n < N) {
                    // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
                    const float hv = ok ? g[j] / (1.0f + expf(-g[j])) * up[j] : 0.f;
                    a.h[static_cast<size_t>(a.pair[p0 + n]) * a.F + row0 + tid] = __float2half_rn(hv);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 128);
}

template <int QD>
__global__ void __launch_bounds__(kGemmThreads) k_batch_down(BatchArgs a) {
    extern __shared__ __align__(1024) uint8_t dsm[];
    uint8_t *sA = dsm, *sB = dsm + 128 * kKC * 2;
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int tiles = a.H / 128;
    const int u = blockIdx.x / tiles, tile = blockIdx.x - u * tiles;
    if (u >= *a.n_used) return;
    const int N = a.cnt[u], Np = max(16, (N + 15) & ~15), p0 = a.off[u];
    const uint8_t *sd = a.srcs[3 * u + 2];
    const int tid = threadIdx.x, warp = tid >> 5, row0 = tile * 128;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tbase, 64);
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tbase;
    bool ok = true;
    for (int kc = 0; kc < a.F / kKC; kc++) {
        {
            const int r = tid >> 1, half = tid & 1;
            const uint8_t *drow = sd + static_cast<size_t>(row0 + r) * a.rb_d;
#pragma unroll 2
            for (int pc = 0; pc < 16; pc++) {
                const int kk = half * 128 + pc * 8;
                float v[8];
                deq8<QD>(drow, kc * kKC + kk, v);
                *reinterpret_cast<uint4 *>(sA + kmaj_off(r, kk, 128)) = pack8_f16(v);
            }
        }
        for (int i = tid; i < Np * (kKC / 8); i += kGemmThreads) {
            const int n = i / (kKC / 8), kk = (i % (kKC / 8)) * 8;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (n < N)
                v = *reinterpret_cast<const uint4 *>(a.h + static_cast<size_t>(a.pair[p0 + n]) * a.F + kc * kKC + kk);
            *reinterpret_cast<uint4 *>(sB + kmaj_off(n, kk, Np)) = v;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0) {
            const uint32_t idesc = umma_idesc_f16(128, Np);
            for (int ks = 0; ks < kKC / 16; ks++) {
                const uint64_t da = umma_desc(smem_addr(sA) + ks * 2 * 128 * 16, 128 * 16, 128);
                const uint64_t db = umma_desc(smem_addr(sB) + ks * 2 * Np * 16, Np * 16, 128);
                umma_f16(tmem, da, db, idesc, (kc | ks) != 0);
            }
            umma_commit(&bar);
        }
        if (ok) ok = batch_wait(&bar, static_cast<uint32_t>(kc & 1), a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    if (tid < 128) {
        const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
        for (int c = 0; c < Np; c += 8) {
            float dv[8];
            tmem_ld8(tmem + lane_base + c, dv);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int n = c + j;
                if (n < N) a.d[static_cast<size_t>(a.pair[p0 + n]) * a.H + row0 + tid] = ok ? dv[j] : 0.f;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------ 5: combine
// x[b][r] += sum_s w[b][s] * d[b][s][r], the slot-ordered sum of
// moe_reduce_f32.comp:8-13 (a slot without an expert adds nothing)
__global__ void k_batch_combine(BatchArgs a) {
    const int b = blockIdx.y, r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.H) return;
    float acc = 0.f;
    for (int s = 0; s < a.k; s++) {
        const int p = b * a.k + s;
        if (a.pv[p]) acc = __fadd_rn(acc, __fmul_rn(a.weights[p], a.d[static_cast<size_t>(p) * a.H + r]));
    }
    float *x = a.x + static_cast<size_t>(b) * a.H + r;
    *x = __fadd_rn(*x, acc);
}

// ------------------------------------------------------------ launchers
bool batch_supported(int qg, int qd) {
    auto ok = [](int q) { return q == STYX_Q4_K || q == STYX_Q5_K || q == STYX_Q6_K || q == STYX_Q8_0; };
    return ok(qg) && ok(qd);
}

template <int QG>
static cudaError_t launch_gateup_q(const BatchArgs &a, cudaStream_t st) {
    const uint32_t smem = 2 * 128 * kKC * 2 + kMaxPairs * kKC * 2;
    cudaError_t e = cudaFuncSetAttribute(k_batch_gateup<QG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_batch_gateup<QG><<<a.E * (a.F / 128), kGemmThreads, smem, st>>>(a);
    return cudaGetLastError();
}
template <int QD>
static cudaError_t launch_down_q(const BatchArgs &a, cudaStream_t st) {
    const uint32_t smem = 128 * kKC * 2 + kMaxPairs * kKC * 2;
    cudaError_t e = cudaFuncSetAttribute(k_batch_down<QD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_batch_down<QD><<<a.E * (a.H / 128), kGemmThreads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_batch(const BatchArgs &a, int qg, int qd, cudaStream_t st) {
    const uint32_t rsmem = static_cast<uint32_t>(a.H + a.E) * 4;
    k_batch_route<<<a.B, kRouteThreads, rsmem, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_batch_lists<<<1, kListThreads, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    switch (qg) {
    case STYX_Q4_K: e = launch_gateup_q<STYX_Q4_K>(a, st); break;
    case STYX_Q5_K: e = launch_gateup_q<STYX_Q5_K>(a, st); break;
    case STYX_Q6_K: e = launch_gateup_q<STYX_Q6_K>(a, st); break;
    default: e = launch_gateup_q<STYX_Q8_0>(a, st); break;
    }
    if (e != cudaSuccess) return e;
    switch (qd) {
    case STYX_Q4_K: e = launch_down_q<STYX_Q4_K>(a, st); break;
    case STYX_Q5_K: e = launch_down_q<STYX_Q5_K>(a, st); break;
    case STYX_Q6_K: e = launch_down_q<STYX_Q6_K>(a, st); break;
    default: e = launch_down_q<STYX_Q8_0>(a, st); break;
    }
    if (e != cudaSuccess) return e;
    k_batch_combine<<<dim3((a.H + 255) / 256, a.B), 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace styx
