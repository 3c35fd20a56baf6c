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
//   2b k_batch_panels  per used expert its tokens' x_norm rows as B panels
//   3  k_bgemm<Q, 2>   gate and up: persistent, one CTA per SM; h goes
//                      straight into the down kernel's B panels
//   4  k_bgemm<Q, 1>   down: the same kernel with one matrix
//   5  k_batch_combine x[b][r] += sum_s w[b][s] d[b][s][r], slot order
//                      (moe_reduce_f32.comp)
//
// The GEMM kernel.  A work unit is (used expert, 128-row tile, K piece):
// the K range of a tile is cut into S pieces when that spreads the units
// more evenly over the SMs (S is a function of the used-expert count only,
// the same in every CTA).  Warp roles, linked by mbarriers (no block barrier
// in the loop):
//   copies      the unit's K chunks (one quant super-block per row, 256
//               elements) into a ring of R stages: one TMA tensor copy per
//               matrix (a 128-row x chunk box of a 3-D map over the source
//               buffer) for q4_K / q5_K, cp.async from 16-byte aligned row
//               windows for q6_K; plus the unit's B panel chunk (bulk copy)
//   dequant     two groups taking alternate 64-wide K slices; a thread
//               turns one row's slice into f16 in an A slot (2 or 4 slots,
//               canonical K-major layout)
//   MMA         one thread: tcgen05.mma (M 128, N = the unit's tokens
//               rounded to 16, K 16) into a TMEM accumulator, commits to the
//               slot, stage and accumulator barriers
//   epilogue    four warps: TMEM -> h = SiLU(g) * u as f16 straight into the
//               down kernel's B panel (gate/up) or d as f32 (down) when
//               S == 1, else f32 partials per piece, which the CTA that
//               finishes an item's last piece sums in piece order (gate/up)
//               or the combine kernel sums (down); two accumulator buffers
// The result does not depend on which CTA ran what.
//
// Dequantisation stays in packed f16 arithmetic: a quant byte q becomes the
// half 1024 + q by OR-ing it into the bits of 1024, t = sc * q exactly by one
// fused multiply-add, then round(round(d * t - c_hi) - c_lo) with the min
// term split in two halves.  Splitting a 32-bit word of four bytes into two
// half2 gives the element order (0, 2, 1, 3) in every group of four; the B
// rows (x_norm and h) are stored in the same order, so the dot products are
// unchanged.
//
// Precision: operands are rounded to f16 (11-bit significand), products and
// sums are f32 in TMEM; the block stays within 1e-3 of max|dx| of the f32
// oracle.  No TMA multicast anywhere; each CTA allocates and frees its own
// TMEM columns; every wait is bounded.
#include <cfloat>
#include <cstring>
#include <type_traits>
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
            const int hi = ids[16 + s], ai = ids[32 + s], fi = ids[48 + s];
            a.src_sel[u] = hi >= 0 ? static_cast<uint32_t>(hi)
                                   : ai >= 0 ? (1u << 28) | static_cast<uint32_t>(ai) : (2u << 28) | static_cast<uint32_t>(fi);
            a.srcs[3 * u + 0] = fused_slot_src(a.gate, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 1] = fused_slot_src(a.up, ids[16 + s], ids[32 + s], ids[48 + s]);
            a.srcs[3 * u + 2] = fused_slot_src(a.down, ids[16 + s], ids[32 + s], ids[48 + s]);
        }
    }
}

// ------------------------------------------------------------ 2b: x_norm panels
// Per used expert u and K chunk kc: the f16 x_norm rows of u's tokens (list
// order), Np = its token count rounded up to 16 rows (zero rows past it), in
// the canonical K-major core-matrix layout the MMA reads; one contiguous
// Np x 512-byte block, so the GEMM brings it with a single bulk copy.
__global__ void __launch_bounds__(256) k_batch_panels(BatchArgs a) {
    const int u = blockIdx.x, kc = blockIdx.y;
    if (u >= *a.n_used) return;
    const int N = a.cnt[u], p0 = a.off[u], Np = max(16, (N + 15) & ~15);
    __half *dst = a.panel_x + static_cast<size_t>(u) * a.npm * a.H + static_cast<size_t>(kc) * Np * 256;
    for (int i = threadIdx.x; i < Np * 32; i += blockDim.x) {
        const int n = i >> 5, kp = i & 31;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (n < N) {
            const int b = a.pair[p0 + n] / a.k;
            v = *reinterpret_cast<const uint4 *>(a.xh + static_cast<size_t>(b) * a.H + kc * 256 + kp * 8);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(dst) + kmaj_off(n, kp * 8, Np)) = v;
    }
}

// ------------------------------------------------------------ quant formats
// Per format: bytes of one K chunk of a row (one 256-element super-block),
// the bulk copy that brings it (a 16-byte aligned window: q4_K / q5_K row
// chunks start on 16-byte boundaries; q6_K's 210-byte blocks on 2-byte ones,
// so its window is the chunk rounded down to 16, 224 bytes, never past the
// 16-byte block that holds the chunk's last byte), and the stage row stride
// (a multiple of 16 whose quotient by 16 is odd: 16-byte reads of 32
// consecutive rows are free of bank conflicts).
__host__ __device__ constexpr int q_bb(int qt) { return qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : 210; }
__host__ __device__ constexpr int q_win(int qt) { return qt == STYX_Q6_K ? 224 : q_bb(qt); }
__host__ __device__ constexpr int q_rsb(int qt) { return qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : 240; }

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
__device__ __forceinline__ uint32_t lop_or(uint32_t v, uint32_t mask) { return (v & mask) | kHalf1024x2; }
// the 6-bit scale and min of sub-block j (0..7) of a q4_K / q5_K super-block
// from its 12 packed bytes in three words (get_scale_min_k4, moe.rs:506-533)
template <int J>
__device__ __forceinline__ void scale_min_k4(uint32_t s0, uint32_t s1, uint32_t s2, float &sc, float &m) {
    auto byte = [&](int i) -> uint32_t { return ((i < 4 ? s0 : i < 8 ? s1 : s2) >> (8 * (i & 3))) & 0xFFu; };
    if constexpr (J < 4) {
        sc = static_cast<float>(byte(J) & 63);
        m = static_cast<float>(byte(J + 4) & 63);
    } else {
        sc = static_cast<float>((byte(J + 4) & 0xF) | ((byte(J - 4) >> 6) << 4));
        m = static_cast<float>((byte(J + 4) >> 4) | ((byte(J) >> 6) << 4));
    }
}

// the 32 bytes at base + o (base 16-byte aligned, o even, 0..14) as eight
// words: three 16-byte reads, then a shift by o in 8-, 4- and 2-byte steps
__device__ __forceinline__ void run32_at(const uint8_t *base, int o, uint32_t (&w)[8]) {
    const uint4 A = *reinterpret_cast<const uint4 *>(base);
    const uint4 B = *reinterpret_cast<const uint4 *>(base + 16);
    const uint4 C = *reinterpret_cast<const uint4 *>(base + 32);
    const uint32_t V[12] = {A.x, A.y, A.z, A.w, B.x, B.y, B.z, B.w, C.x, C.y, C.z, C.w};
    const bool s8 = (o & 8) != 0, s4 = (o & 4) != 0;
    const uint32_t sh = static_cast<uint32_t>(o & 2) << 3;
    uint32_t T1[10], T2[9];
#pragma unroll
    for (int i = 0; i < 10; i++) T1[i] = s8 ? V[i + 2] : V[i];
#pragma unroll
    for (int i = 0; i < 9; i++) T2[i] = s4 ? T1[i + 1] : T1[i];
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = __funnelshift_r(T2[i], T2[i + 1], sh);
}

// 32 elements of K slice J (64 wide) of one weight row, half H: elements
// 64 J + 32 H .. + 31 of the row's 256-element chunk, from its stage row
// (quant data at byte `o`: 0 but for q6_K), as f16 in sixteen words, element order
// (0, 2, 1, 3) in every four.  Values: the reference's d * sc * q - dmin * m
// (q4_K / q5_K), d * sc * (q - 32) (q6_K).
//
// q4_K / q5_K keep the error per element: t = sc * q is an integer below
// 2048, exact in f16, from one fused multiply-add on the half 1024 + q (the
// quant bits OR-ed into 1024's, exact); high nibbles are taken in place, as
// 1024 + 16 q, with sc / 16 and 64 sc (exact too); d is the stored half; the
// min term c = dmin * m (exact in f32) goes in as c_hi + c_lo.  So an element
// is round(round(d * t - c_hi) - c_lo), and no rounding is shared by the 32
// elements of a sub-block.
template <int QT, int J, int H>
__device__ __forceinline__ void deq_run(const uint8_t *row, int o, uint32_t (&out)[16]) {
    if constexpr (QT == STYX_Q4_K || QT == STYX_Q5_K) {
        constexpr int SB = 2 * J + H;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(row);   // d, dmin, 12 scale bytes
        const __half dh = __ushort_as_half(static_cast<unsigned short>(hdr.x & 0xFFFFu));
        const float dm = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr.x >> 16)));
        float sc, mn;
        scale_min_k4<SB>(hdr.y, hdr.z, hdr.w, sc, mn);
        const float c = dm * mn;
        const __half chi = __float2half_rn(c);
        const __half clo = __float2half_rn(c - __half2float(chi));
        const __half2 d2 = __half2half2(dh), nchi2 = __half2half2(__hneg(chi)), clo2 = __half2half2(clo);
        constexpr int QS = QT == STYX_Q4_K ? 16 : 48;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(row + QS + 32 * J);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(row + QS + 32 * J + 16);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        if constexpr (QT == STYX_Q4_K) {
            // H = 0: 1024 + q, t = e sc - 1024 sc; H = 1: 1024 + 16 q, t = e sc/16 - 64 sc
            const __half2 sc2 = __float2half2_rn(H ? sc * 0.0625f : sc);
            const __half2 nb2 = __float2half2_rn(H ? -64.0f * sc : -1024.0f * sc);
            constexpr uint32_t M = H ? 0x00F000F0u : 0x000F000Fu;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const __half2 t02 = __hfma2(u2h2(lop_or(w[i], M)), sc2, nb2);
                const __half2 t13 = __hfma2(u2h2(lop_or(w[i] >> 8, M)), sc2, nb2);
                out[2 * i] = h22u(__hsub2(__hfma2(t02, d2, nchi2), clo2));
                out[2 * i + 1] = h22u(__hsub2(__hfma2(t13, d2, nchi2), clo2));
            }
        } else {   // q5_K: the fifth bit from qh (bit SB of each byte); q up to 31
            const uint4 h0 = *reinterpret_cast<const uint4 *>(row + 16);
            const uint4 h1 = *reinterpret_cast<const uint4 *>(row + 32);
            const uint32_t hb[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            const __half2 sc2 = __float2half2_rn(sc), k1024 = u2h2(kHalf1024x2);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t v = ((w[i] >> (4 * H)) & 0x0F0F0F0Fu) | (((hb[i] >> SB) & 0x01010101u) << 4);
                const __half2 t02 = __hmul2(__hsub2(u2h2(lop_or(v, 0x00FF00FFu)), k1024), sc2);
                const __half2 t13 = __hmul2(__hsub2(u2h2(lop_or(v >> 8, 0x00FF00FFu)), k1024), sc2);
                out[2 * i] = h22u(__hsub2(__hfma2(t02, d2, nchi2), clo2));
                out[2 * i + 1] = h22u(__hsub2(__hfma2(t13, d2, nchi2), clo2));
            }
        }
    } else {   // q6_K: quadrant QD = 2 (J & 1) + H of the 128-element half N = J / 2; data at byte o (0..14)
        constexpr int N = J >> 1, QD = 2 * (J & 1) + H;
        uint32_t ql[8], qh[8];
        run32_at(row + 64 * N + 32 * (QD & 1), o, ql);
        run32_at(row + 128 + 32 * N, o, qh);
        // the quadrant's two int8 scales (l < 16, l >= 16) and d: 2-byte aligned pairs
        const uint32_t sc_pair = *reinterpret_cast<const unsigned short *>(row + o + 192 + 8 * N + 2 * QD);
        const float d = __half2float(*reinterpret_cast<const __half *>(row + o + 208));
        const __half2 s0 = __float2half2_rn(d * static_cast<float>(static_cast<int8_t>(sc_pair & 0xFFu)));
        const __half2 s1 = __float2half2_rn(d * static_cast<float>(static_cast<int8_t>(sc_pair >> 8)));
        const __half2 bias = u2h2(0x64206420u);   // 1024 + 32
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t v = ((ql[i] >> (4 * (QD >> 1))) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * QD)) & 0x03030303u) << 4);
            const __half2 sc = i < 4 ? s0 : s1;
            out[2 * i] = h22u(__hmul2(__hsub2(u2h2(lop_or(v, 0x00FF00FFu)), bias), sc));
            out[2 * i + 1] = h22u(__hmul2(__hsub2(u2h2(lop_or(v >> 8, 0x00FF00FFu)), bias), sc));
        }
    }
}
// the sixteen words of a run into the A slot (row r, K offset k0 of the slice)
__device__ __forceinline__ void store_run(uint8_t *slot, int r, int k0, const uint32_t (&out)[16]) {
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

__host__ __device__ constexpr uint32_t tmem_cols_for(int n) {
    return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : 256u;
}

// One side of the block: gate + up (NM = 2) or down (NM = 1).
struct GemmSide {
    int K, M, rb;            // row length, rows of one expert matrix, bytes of a row
    int mat0;                // srcs index of the first matrix (0: gate, up; 2: down)
    const __half *panel;     // B panels: per used expert npm * K halves, chunk kc at kc * Np * 256
    float *part0, *part1;    // f32 partials [smax][P][M] per matrix (down: part0 piece 0 = d)
    int npm;                 // largest Np (tokens of one expert, padded to 16)
    int stages;              // R
    int nslot;               // A slots: 2 or 4
    int smax;
    int *split_out;          // the S this launch used
};

// Warp roles of a GEMM CTA: copies (one warp issuing TMA tensor copies for
// q4_K / q5_K; four warps of cp.async for q6_K, whose rows are not 16-byte
// multiples), dequantisation (two groups of 4 warps per matrix taking
// alternate 64-wide slices, a whole row's slice per thread), the MMA thread
// (one warp), the epilogue (four consecutive warps, whose ids mod 4 cover the
// four TMEM lane quarters).
constexpr int kEpiWarps = 4;
constexpr int kMaxStages = 4;
template <int QT, int NM>
struct GemmRoles {
    static constexpr bool kTma = QT != STYX_Q6_K;
    static constexpr int kProd = kTma ? 1 : 4;
    static constexpr int kDeq = 8 * NM;
    static constexpr int kMma = kProd + kDeq;
    static constexpr int kEpi0 = kMma + 1;
    static constexpr int kThreads = 32 * (kEpi0 + kEpiWarps);
};
bool batch_uses_tma(int qt) { return qt == STYX_Q4_K || qt == STYX_Q5_K; }

struct GemmBars {
    uint64_t full[kMaxStages];    // a stage's copies landed (expect_tx arrival, or one cp.async arrival per copy thread)
    uint64_t empty[kMaxStages];   // a stage's MMAs done (tcgen05.commit)
    uint64_t afull[4];            // an A slot dequantised (one arrival per warp of its dequant group)
    uint64_t aempty[4];           // an A slot's MMAs done
    uint64_t accf[2];             // an accumulator buffer complete
    uint64_t acce[2];             // an accumulator buffer read out (one arrival per epilogue warp)
    uint64_t drain;               // the MMA thread's last commit
};

__device__ __forceinline__ void tma_load3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar,
                                           uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}
// the mbarrier counts one arrival when all of this thread's earlier cp.async are done
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }
// every epilogue thread arrives (whatever its wait returned), so this barrier
// always completes; true when all of them passed their wait
__device__ __forceinline__ bool epi_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "barrier.cta.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(ok)), "n"(32 * kEpiWarps)
        : "memory");
    return r != 0;
}

template <int QT, int NM>
__global__ void __launch_bounds__(GemmRoles<QT, NM>::kThreads, 1)
    k_bgemm(BatchArgs a, GemmSide g, const __grid_constant__ TmaSet tm) {
    using RL = GemmRoles<QT, NM>;
    constexpr int BB = q_bb(QT), RSB = q_rsb(QT);
    constexpr int ASLOT = NM * 128 * 64 * 2;
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ GemmBars bars;
    __shared__ uint32_t tbase;
    __shared__ int s_abort, s_fin;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    const int n_used = *a.n_used;
    const int tiles = g.M / 128, nk = g.K / 256, P = a.B * a.k;
    const int n_items = n_used * tiles;
    const int S = choose_split(n_items, nk, G, g.smax);
    if (cta == 0 && tid == 0) *g.split_out = S;
    const int CPU = nk / S;   // chunks of one unit
    const int n_units = n_items * S;
    const int my_units = cta < n_units ? (n_units - 1 - cta) / G + 1 : 0;
    if (my_units == 0) return;   // the whole CTA, before any barrier or TMEM use
    const int Q = my_units * CPU;
    const int Npm = g.npm, R = g.stages, NS = g.nslot;
    const int stage_w = NM * 128 * RSB, stage_bytes = stage_w + Npm * 512;
    uint8_t *slots = sm, *stages = sm + NS * ASLOT;
    const int acc_cols = NM * Npm;   // one accumulator buffer; two of them
    const uint32_t tcols = tmem_cols_for(2 * acc_cols);
    if (tid == 0) {
        for (int i = 0; i < R; i++) {
            mbar_init(&bars.full[i], RL::kTma ? 1 : 32 * RL::kProd);
            mbar_init(&bars.empty[i], 1);
        }
        for (int i = 0; i < NS; i++) {
            mbar_init(&bars.afull[i], RL::kDeq / 2);
            mbar_init(&bars.aempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars.accf[i], 1);
            mbar_init(&bars.acce[i], kEpiWarps);
        }
        mbar_init(&bars.drain, 1);
        s_abort = 0;
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

    // unit i of this CTA: v = cta + i G -> (item, piece) -> (used expert, tile)
    auto unit_of = [&](int i, int &u, int &tile, int &piece) {
        const int v = cta + i * G, item = v / S;
        piece = v - item * S;
        u = item / tiles;
        tile = item - u * tiles;
    };
    // bounded wait; false once any role of the CTA gave up
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        const long long t0 = clock64();
        while (true) {
            if (mbar_try_wait_suspend(bar, parity)) return true;
            if (*reinterpret_cast<volatile int *>(&s_abort)) return false;
            if (clock64() - t0 > kSpinCycles) {
                atomicExch(a.err, kErrWaitFull);
                *reinterpret_cast<volatile int *>(&s_abort) = 1;
                return false;
            }
        }
    };

    if (warp < RL::kProd) {
        // ---------------- copies: chunk q into stage q % R once its MMAs are done
        const uint64_t pol_w = l2_evict_first(), pol_b = l2_evict_last();
        int cu, ct, cpc;
        unit_of(0, cu, ct, cpc);
        int N = __ldg(a.cnt + cu);
        uint32_t sel = __ldg(a.src_sel + cu);
        const uint8_t *s0 = a.srcs[3 * cu + g.mat0], *s1 = a.srcs[3 * cu + g.mat0 + (NM - 1)];
        for (int q = 0; q < Q; q++) {
            const int ui = q / CPU, kc = cpc * CPU + (q - ui * CPU);
            const bool unit_end = q - ui * CPU == CPU - 1;
            int u = cu, tile = ct, piece = cpc, nN = N;
            uint32_t nsel = sel;
            const uint8_t *ns0 = s0, *ns1 = s1;
            if (unit_end && ui + 1 < my_units) {   // the next unit's tables, loaded early
                unit_of(ui + 1, u, tile, piece);
                nN = __ldg(a.cnt + u);
                nsel = __ldg(a.src_sel + u);
                ns0 = a.srcs[3 * u + g.mat0];
                ns1 = a.srcs[3 * u + g.mat0 + (NM - 1)];
            }
            const int st_i = q % R, use = q / R;
            const int Np = max(16, (N + 15) & ~15);
            if (use > 0 && !wait(&bars.empty[st_i], static_cast<uint32_t>((use - 1) & 1))) break;
            uint8_t *st = stages + st_i * stage_bytes;
            const __half *pan = g.panel + static_cast<size_t>(cu) * Npm * g.K + static_cast<size_t>(kc) * Np * 256;
            if constexpr (RL::kTma) {
                // one tensor copy per matrix: the chunk's 128 rows x BB bytes; one bulk copy for the panel
                if (lane == 0) {
                    mbar_arrive_expect_tx(&bars.full[st_i], static_cast<uint32_t>(NM * 128 * BB + Np * 512));
                    const int kind = static_cast<int>(sel >> 28), slot = static_cast<int>(sel & 0x0FFFFFFFu);
#pragma unroll
                    for (int mm = 0; mm < NM; mm++)
                        tma_load3d(st + mm * 128 * RSB, &tm.m[mm][kind], kc * BB, ct * 128, slot, &bars.full[st_i], pol_w);
                    bulk_g2s_hint(st + stage_w, pan, static_cast<uint32_t>(Np * 512), &bars.full[st_i], pol_b);
                }
            } else {
                // cp.async from each row's 16-byte aligned window of the chunk, then the panel
                const int pt = tid;   // 0 .. 32 * kProd - 1
                const size_t at = static_cast<size_t>(ct) * 128 * g.rb + static_cast<size_t>(kc) * BB;
                constexpr int PCS = q_win(QT) / 16;
                for (int i = pt; i < NM * 128 * PCS; i += 32 * RL::kProd) {
                    const int rr = i / PCS, pc = i - rr * PCS;
                    const uint8_t *rs = ((rr >> 7) ? s1 : s0) + at + static_cast<size_t>(rr & 127) * g.rb;
                    cp_async16(st + rr * RSB + pc * 16, rs - (reinterpret_cast<uintptr_t>(rs) & 15) + pc * 16, pol_w);
                }
                for (int i = pt; i < Np * 32; i += 32 * RL::kProd)
                    cp_async16(st + stage_w + i * 16, reinterpret_cast<const uint8_t *>(pan) + i * 16, pol_b);
                cp_async_arrive(&bars.full[st_i]);
            }
            if (unit_end && ui + 1 < my_units) {
                N = nN;
                sel = nsel;
                s0 = ns0;
                s1 = ns1;
                cu = u;
                ct = tile;
                cpc = piece;
            }
        }
        if constexpr (!RL::kTma) asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp < RL::kMma) {
        // ---------------- dequantisation: group grp takes the slices of its parity;
        // thread -> (matrix, row): the row's whole 64-wide slice
        const int dt = tid - 32 * RL::kProd;
        const int grp = dt / (128 * NM), idx = dt - grp * 128 * NM;
        const int m = idx >> 7, r = idx & 127;
        bool live = true;
        for (int q = 0; q < Q && live; q++) {
            const int st_i = q % R;
            if (!wait(&bars.full[st_i], static_cast<uint32_t>((q / R) & 1))) break;
            __syncwarp();
            const uint8_t *row = stages + st_i * stage_bytes + (m * 128 + r) * RSB;
            int o = 0;
            if constexpr (!RL::kTma) {   // where the chunk starts in its 16-byte window (slabs are 16-byte aligned)
                int u, tile, piece;
                const int ui = q / CPU;
                unit_of(ui, u, tile, piece);
                const int kc = piece * CPU + (q - ui * CPU);
                o = static_cast<int>((static_cast<size_t>(tile * 128 + r) * g.rb + static_cast<size_t>(kc) * BB) & 15);
            }
            auto slice = [&](auto jc) {
                constexpr int J = decltype(jc)::value;
                const int gsl = 4 * q + J, slot = gsl % NS, use = gsl / NS;
                if (use > 0 && !wait(&bars.aempty[slot], static_cast<uint32_t>((use - 1) & 1))) {
                    live = false;
                    return;
                }
                __syncwarp();
                uint32_t o0[16], o1[16];
                deq_run<QT, J, 0>(row, o, o0);
                deq_run<QT, J, 1>(row, o, o1);
                uint8_t *sA = slots + slot * ASLOT + m * (128 * 64 * 2);
                store_run(sA, r, 0, o0);
                store_run(sA, r, 32, o1);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars.afull[slot]);
            };
            if (grp == 0) {
                slice(std::integral_constant<int, 0>{});
                if (live) slice(std::integral_constant<int, 2>{});
            } else {
                slice(std::integral_constant<int, 1>{});
                if (live) slice(std::integral_constant<int, 3>{});
            }
        }
    } else if (warp == RL::kMma) {
        // ---------------- one thread issues the MMAs
        if (lane == 0) {
            int gsl = 0;
            bool live = true;
            for (int ui = 0; ui < my_units && live; ui++) {
                int u, tile, piece;
                unit_of(ui, u, tile, piece);
                const int N = __ldg(a.cnt + u), Np = max(16, (N + 15) & ~15);
                const int ab = ui & 1;
                if (ui >= 2 && !wait(&bars.acce[ab], static_cast<uint32_t>(((ui >> 1) - 1) & 1))) break;
                tc_fence_after();
                const uint32_t dacc = tmem + static_cast<uint32_t>(ab * acc_cols);
                const uint32_t idesc = umma_idesc_f16(128, Np);
                for (int c = 0; c < CPU && live; c++) {
                    const int q = ui * CPU + c, st_i = q % R;
                    if (!wait(&bars.full[st_i], static_cast<uint32_t>((q / R) & 1))) {
                        live = false;
                        break;
                    }
                    fence_async_smem();   // the copied B rows, seen by the tensor core
                    const uint32_t sB = smem_addr(stages + st_i * stage_bytes + stage_w);
                    for (int j = 0; j < 4; j++, gsl++) {
                        const int slot = gsl % NS;
                        if (!wait(&bars.afull[slot], static_cast<uint32_t>((gsl / NS) & 1))) {
                            live = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sA = smem_addr(slots + slot * ASLOT);
#pragma unroll
                        for (int mm = 0; mm < NM; mm++)
#pragma unroll
                            for (int kk = 0; kk < 4; kk++) {
                                const uint64_t da = umma_desc(sA + mm * (128 * 64 * 2) + kk * 2 * 2048, 2048, 128);
                                const uint64_t db = umma_desc(sB + (j * 8 + kk * 2) * Np * 16, Np * 16, 128);
                                umma_f16(dacc + mm * Npm, da, db, idesc, (c == 0 && j == 0 && kk == 0) ? 0u : 1u);
                            }
                        umma_commit(&bars.aempty[slot]);
                    }
                    if (live) umma_commit(&bars.empty[st_i]);
                }
                if (live) umma_commit(&bars.accf[ab]);
            }
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(&bars.drain);
            const long long t0 = clock64();
            while (!mbar_try_wait(&bars.drain, 0u) && clock64() - t0 < kSpinCycles) {
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: TMEM lane quarter ew = warp mod 4, row = 32 ew + lane
        const int ew = warp & 3, et = tid - 32 * RL::kEpi0;
        const uint32_t lane_base = static_cast<uint32_t>(32 * ew) << 16;
        for (int ui = 0; ui < my_units; ui++) {
            int u, tile, piece;
            unit_of(ui, u, tile, piece);
            const int N = __ldg(a.cnt + u), p0 = __ldg(a.off + u), Np = max(16, (N + 15) & ~15);
            const int pr0 = lane < N ? __ldg(a.pair + p0 + lane) : 0;
            const int pr1 = lane + 32 < N ? __ldg(a.pair + p0 + 32 + lane) : 0;
            const int ab = ui & 1;
            const bool ok = epi_all(wait(&bars.accf[ab], static_cast<uint32_t>((ui >> 1) & 1)));
            if (!ok) break;
            tc_fence_after();
            const uint32_t dacc = tmem + static_cast<uint32_t>(ab * acc_cols) + lane_base;
            const int row = tile * 128 + 32 * ew + lane;
            const size_t hpan = static_cast<size_t>(u) * Npm * g.M;   // gate/up: this expert's down panel
            for (int c = 0; c < Np; c += 8) {
                float v0[8], v1[8];
                tmem_ld8(dacc + c, v0);
                if constexpr (NM == 2) tmem_ld8(dacc + Npm + c, v1);
#pragma unroll
                for (int jj = 0; jj < 8; jj++) {
                    const int n = c + jj;
                    const int p = __shfl_sync(0xffffffffu, n < 32 ? pr0 : pr1, n & 31);
                    if (n >= N) continue;
                    if constexpr (NM == 2) {
                        if (S == 1) {
                            // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
                            const float hv = v0[jj] / (1.0f + expf(-v0[jj])) * v1[jj];
                            a.panel_h[hpan + static_cast<size_t>(row >> 8) * Np * 256 +
                                      kmaj_off(n, kperm(row & 255), Np) / 2] = __float2half_rn(hv);
                        } else {
                            const size_t at = (static_cast<size_t>(piece) * P + p) * g.M + row;
                            g.part0[at] = v0[jj];
                            g.part1[at] = v1[jj];
                        }
                    } else {
                        g.part0[(static_cast<size_t>(piece) * P + p) * g.M + row] = v0[jj];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.acce[ab]);
            if constexpr (NM == 2) {
                if (S > 1) {   // the item's last piece sums the pieces in piece order
                    epi_bar_sync();   // every partial of this piece stored
                    if (et == 0) {
                        __threadfence();
                        s_fin = atomicAdd(&a.item_cnt[u * tiles + tile], 1) == S - 1;
                        __threadfence();
                    }
                    epi_bar_sync();
                    if (s_fin) {
                        for (int i = et; i < 128 * N; i += 32 * kEpiWarps) {
                            const int n = i >> 7, rr = tile * 128 + (i & 127);
                            const int p = __ldg(a.pair + p0 + n);
                            const size_t hat = hpan + static_cast<size_t>(rr >> 8) * Np * 256 + kmaj_off(n, kperm(rr & 255), Np) / 2;
                            float gsum = 0.f, usum = 0.f;
                            for (int sp = 0; sp < S; sp++) {
                                const size_t at = (static_cast<size_t>(sp) * P + p) * g.M + rr;
                                gsum += __ldcg(g.part0 + at);
                                usum += __ldcg(g.part1 + at);
                            }
                            a.panel_h[hat] = __float2half_rn(gsum / (1.0f + expf(-gsum)) * usum);
                        }
                    }
                    epi_bar_sync();   // s_fin read by all before the next unit writes it
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
static cudaError_t launch_bgemm(const BatchArgs &a, GemmSide g, const TmaSet &tm, cudaStream_t st) {
    // four A slots when two stages still fit beside them, else two
    const int stage_bytes = NM * 128 * q_rsb(QT) + g.npm * 512;
    const int slot_bytes = NM * 128 * 64 * 2;
    g.nslot = (kSmemCap - 4 * slot_bytes) / stage_bytes >= 2 ? 4 : 2;
    int R = (kSmemCap - g.nslot * slot_bytes) / stage_bytes;
    if (R > kMaxStages) R = kMaxStages;
    if (R < 2) return cudaErrorInvalidValue;
    g.stages = R;
    const int smem = g.nslot * slot_bytes + R * stage_bytes;
    cudaError_t e = cudaFuncSetAttribute(k_bgemm<QT, NM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_bgemm<QT, NM><<<a.sms, GemmRoles<QT, NM>::kThreads, smem, st>>>(a, g, tm);
    return cudaGetLastError();
}

template <int NM>
static cudaError_t launch_bgemm_q(int qt, const BatchArgs &a, const GemmSide &g, const TmaSet &tm, cudaStream_t st) {
    switch (qt) {
    case STYX_Q4_K: return launch_bgemm<STYX_Q4_K, NM>(a, g, tm, st);
    case STYX_Q5_K: return launch_bgemm<STYX_Q5_K, NM>(a, g, tm, st);
    case STYX_Q6_K: return launch_bgemm<STYX_Q6_K, NM>(a, g, tm, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_batch(const BatchArgs &a, int qg, int qd, const TmaSet &tgu, const TmaSet &tdn, cudaStream_t st) {
    k_batch_logits<<<dim3(a.B, (a.E + kLogitRows - 1) / kLogitRows), kLogitThreads, static_cast<size_t>(a.H) * 4, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_batch_lists<<<1, kListThreads, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_batch_panels<<<dim3(a.E, a.H / 256), 256, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int npm = a.npm;
    GemmSide gu{};
    gu.K = a.H;
    gu.M = a.F;
    gu.rb = a.rb_g;
    gu.mat0 = 0;
    gu.panel = a.panel_x;
    gu.part0 = a.gpart;
    gu.part1 = a.upart;
    gu.npm = npm;
    gu.smax = batch_split_max(a.H);
    gu.split_out = a.split_d + 1;
    if ((e = launch_bgemm_q<2>(qg, a, gu, tgu, st)) != cudaSuccess) return e;
    GemmSide dn{};
    dn.K = a.F;
    dn.M = a.H;
    dn.rb = a.rb_d;
    dn.mat0 = 2;
    dn.panel = a.panel_h;
    dn.part0 = a.d;
    dn.part1 = nullptr;
    dn.npm = npm;
    dn.smax = batch_split_max(a.F);
    dn.split_out = a.split_d;
    if ((e = launch_bgemm_q<1>(qd, a, dn, tdn, st)) != cudaSuccess) return e;
    k_batch_combine<<<dim3((a.H + 255) / 256, a.B), 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace styx
