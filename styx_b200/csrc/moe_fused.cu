// moe_fused.cu -- the whole MoE block of one layer as ONE cooperative kernel.
//
// Grid = one CTA per SM (cooperative launch: all CTAs co-resident), 16 warps.
// A CTA's share of the layer's expert bytes (its gate/up rows and its down
// rows for all k slots) fits in shared memory at the shapes this kernel is
// planned for (the host checks), so every bulk copy is issued up front and
// the whole layer streams from HBM at once.  Phases of CTA b of G:
//   0  barrier init; L2 prefetch of this CTA's router rows (e = b, b+G, ...)
//      and ffn_norm; the next kernel in the stream may launch (PDL); wait
//      for the previous grid;
//   1  RMSNorm of x (every CTA, same fixed order -> identical x_norm), the
//      router dot products of its rows -> tagged logit slots;
//   2  all warps turn x_norm into dp4a digits; warp 0 reads all E logit
//      slots (polling until each carries this launch's tag, bounded) and
//      picks the top-k in registers with warp reductions (the selection of
//      topk_softmax_f32.comp): every CTA computes the same ids;
//   3  warp 0 resolves the k slots (id rows, slab sources; CTA 0 publishes
//      the ids) and issues the CTA's gate/up chunks (one lane per chunk) and
//      down rows (one lane per slot); all warps then run the gate/up dot
//      products as chunks land (the chunk's mbarrier also publishes the slot
//      sources), SiLU(g)*u -> h (global);
//   4  each CTA counts its h rows into per-slot arrival counters (one fence);
//      warp 1 computes the softmax weights; the warps of slot s wait for
//      slot s alone, turn h[s] into digits in shared memory and run the
//      CTA's down rows for slot s from the prefetched rows; slot-ordered
//      combine x[r] += sum_s w[s] d[s][r] (moe_reduce_f32.comp).
// Logits go through tagged exchange words: one 64-bit {value bits, tag}
// word written and read with single 64-bit relaxed accesses, so a reader
// that sees this launch's tag also sees its value, with no fence or counter.
// The tag is the launch number + 1 (the workspace's launch counter, bumped
// once by every CTA, divided by the grid size); the h arrival counts are never
// reset either: nothing in the workspace needs clearing between launches.
// Every wait is bounded (~1 s) and reports through the device error word.
#include <cfloat>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "ep_sync.cuh"
#include "kernels.h"
#include "moe_common.cuh"
#include "qdot.cuh"

namespace styx {

// shared-memory header: 32 mbarriers, reduction scratch, weights, ids,
// flags, per-slot source pointers; region A starts at kFusedHeader
constexpr int kHdrRed = 512;
constexpr int kHdrSrc = 896;
constexpr int kHdrArgs = 1280;   // a copy of the launch's FusedArgs
constexpr int kFusedHeaderBytes = 1792;
static_assert(kHdrSrc + 3 * 16 * 8 <= kHdrArgs, "fused header overflow");
static_assert(sizeof(FusedArgs) <= kFusedHeaderBytes - kHdrArgs && sizeof(FusedArgs) % 8 == 0,
              "FusedArgs does not fit its header slot");
static_assert(kFusedHeaderBytes == static_cast<int>(kFusedHeader), "host and device header sizes differ");
static_assert(32 * 8 <= kHdrRed, "mbarriers overlap the reduction scratch");

// Named barriers: 0 is __syncthreads, 1 + s the warps of slot s in the down
// phase (s < 8 when a slot has more than one warp), kBarWarp0 warp 0 alone.
constexpr int kBarWarp0 = 15;

// barrier among the nthreads threads (whole warps) that work on slot s:
// named barrier 1 + s (0 is __syncthreads), or the warp itself
__device__ __forceinline__ void slot_group_sync(int s, int nthreads) {
    if (nthreads == 32) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + s), "r"(nthreads) : "memory");
}

// Gate/up chunk c of a CTA: CTA rows [c*ch, c*ch + n) of the flattened
// (slot, row) range starting at gbeg.  A chunk holds at most two segments:
// rows rrA.. of slot sA (nA rows), then rows 0.. of slot sA + 1.
struct GuChunk {
    int sA, rrA, n, nA;
};
__device__ __forceinline__ GuChunk gu_chunk(int c, int ch, int gbeg, int nrows, int F) {
    GuChunk g;
    const int r0 = gbeg + c * ch;
    g.sA = r0 / F;
    g.rrA = r0 - g.sA * F;
    g.n = min(ch, nrows - c * ch);
    g.nA = min(g.n, F - g.rrA);
    return g;
}
// shared-memory offset of segment B inside a gate (or up) area
__device__ __forceinline__ uint32_t seg_b_off(int nA, int rb) {
    return static_cast<uint32_t>((static_cast<size_t>(nA) * rb + 32 + 15) & ~size_t(15));
}

// How a layer connects to its neighbours.  A layer that starts a chain reads
// x from global memory after the grid dependency resolves (wait_grid); a
// later one reads the x its predecessor published as tagged words (one per
// row, tag = the predecessor's tag = this layer's tag - 1), whether the
// predecessor ran earlier in the same launch or in the previous launch on
// the workspace.  A layer with a successor publishes its output rows the
// same way and warms L2 with the successor's router rows.
//
// Chained launches skip the grid dependency: the next layer's CTAs start as
// soon as their SM is free and overlap their prologue with the previous
// layer's tail.  That is safe because before any CTA of a layer exits, every
// CTA of that layer has started (each waits for all the layer's logits), so
// at most two consecutive layers are resident, neither waits for the later
// one, and the words they could both touch are kept apart: the logit words
// alternate between two banks by tag parity, the h rows and counts of the
// later layer are written only after every CTA of the earlier one has exited,
// and the residual add uses the x rows read from the tagged words.
// (LayerLink itself is declared in kernels.h, for the host.)

// the link sits in shared memory after the arguments, read where it is used
// (kept in registers across the layer it would push the kernel into spills)
constexpr int kHdrLink = kHdrArgs + ((static_cast<int>(sizeof(FusedArgs)) + 15) & ~15);
static_assert(kHdrLink + static_cast<int>(sizeof(LayerLink)) <= kFusedHeaderBytes, "layer link overflows the header");

// The launch parameters, read once in parallel into shared memory: reading
// them field by field from the parameter bank costs a constant-cache miss on
// each first touch in every phase.  Thread 0 also stores the layer link.
__device__ __forceinline__ void load_args(uint8_t *smem, const FusedArgs &a, const LayerLink &lk) {
    if (threadIdx.x < sizeof(FusedArgs) / 8)
        reinterpret_cast<uint64_t *>(smem + kHdrArgs)[threadIdx.x] = reinterpret_cast<const uint64_t *>(&a)[threadIdx.x];
    if (threadIdx.x == 0) *reinterpret_cast<LayerLink *>(smem + kHdrLink) = lk;
}

template <int QG, int QD>
__device__ __forceinline__ void fused_layer(uint8_t *smem) {
    const FusedArgs &p = *reinterpret_cast<const FusedArgs *>(smem + kHdrArgs);
    const LayerLink &lk = *reinterpret_cast<const LayerLink *>(smem + kHdrLink);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    uint64_t *full_gu = bar, *full_d = bar + 16;
    float *red = reinterpret_cast<float *>(smem + kHdrRed);  // 32 floats
    float *wts = red + 32;                                    // 16 floats
    int *s_flag = reinterpret_cast<int *>(wts + 32);          // 16 ints (after 16 spare)
    const uint8_t **src_g = reinterpret_cast<const uint8_t **>(smem + kHdrSrc);   // 16 pointers each
    const uint8_t **src_u = src_g + 16;
    const uint8_t **src_d = src_u + 16;
    const int H = p.H, F = p.F, k = p.k, E = p.E;
    uint8_t *region_a = smem + p.off_a;                       // x_norm and its digits
    float *xn = reinterpret_cast<float *>(region_a);
    int8_t *xd1 = reinterpret_cast<int8_t *>(xn + H);
    uint8_t *xd2 = reinterpret_cast<uint8_t *>(xd1) + H;
    uint8_t *xd3 = xd2 + H;
    float *xsc = reinterpret_cast<float *>(xd3 + H);
    const int kF = k * F;                                     // phase 4: h digits in region A
    int8_t *hd1 = reinterpret_cast<int8_t *>(region_a);
    uint8_t *hd2 = reinterpret_cast<uint8_t *>(hd1) + kF;
    uint8_t *hd3 = hd2 + kF;
    float *hsc = reinterpret_cast<float *>(hd3 + kF);
    float *dpart = reinterpret_cast<float *>(smem + p.off_part);
    float *lgs = dpart - ((E + 31) & ~31);                    // the logits, at the end of region A
    uint32_t *smap = reinterpret_cast<uint32_t *>(lgs) - 2 * ((E + 31) & ~31);   // remap, pmap (before the logits)
    const int Ep = (E + 31) & ~31;
    uint8_t *gubuf = smem + p.off_ring;
    uint8_t *dbuf = smem + p.off_down;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const long long T = static_cast<long long>(k) * F;
    const int gbeg = static_cast<int>(T * b / G), gend = static_cast<int>(T * (b + 1) / G);
    const int nrows = gend - gbeg;
    const int n_chunks = (nrows + p.ch - 1) / p.ch;
    const int dbeg = static_cast<int>(static_cast<long long>(H) * b / G);
    const int dend = static_cast<int>(static_cast<long long>(H) * (b + 1) / G);
    const int n_rows_mine = b < E ? (E - 1 - b) / G + 1 : 0;   // router rows e = b + G*j

#define STYX_STAMP_T(t_, i_)                                               \
    do {                                                                   \
        if (tid == (t_) && p.trace) p.trace[b * kTraceStamps + (i_)] = clock64(); \
    } while (0)
#define STYX_STAMP(i_) STYX_STAMP_T(0, i_)
    STYX_STAMP(0);
    // ------------------------------------------------ phase 0
    if (tid < 16) {   // one thread per barrier: the gate/up chunks', and the down rows'
        if (lk.index) {   // the previous layer's barriers: every phase complete, every copy landed
            mbar_inval(&full_gu[tid]);
            if (tid == 0) mbar_inval(&full_d[0]);
        }
        mbar_init(&full_gu[tid], 1);
        if (tid == 0) mbar_init(&full_d[0], 1);
        fence_mbar_init();
    }
    if (lk.index == 0) {
        pdl_trigger();
        // router rows and norms are read every token: kept in L2 (evict
        // last) while the expert slabs stream through it (evict first)
        const uint64_t keep = l2_evict_last();
        for (int j = tid; j < n_rows_mine; j += kFusedBlock)
            prefetch_l2_hint(p.router + static_cast<size_t>(b + G * j) * H, static_cast<uint32_t>(H) * 4u, keep);
        if (tid == kFusedBlock - 1) prefetch_l2_hint(p.norm_w, static_cast<uint32_t>(H) * 4u, keep);
    }
    // this launch's tag (published to the block by the barriers in phase 1).
    // Safe before the grid dependency resolves: every CTA of the previous
    // launch on this workspace took its number before any of them could exit
    // (each waits in phase 2 for all of that launch's logits), and a CTA of
    // this launch cannot be resident before one of the previous launch exits
    // (one CTA fills an SM's registers, and the grid covers every SM).
    uint32_t *s_tag = reinterpret_cast<uint32_t *>(s_flag + 2);
    // (A later layer of the same launch: every CTA took its number for the
    // previous layer before any CTA could finish that layer, so the layers
    // of a launch are numbered consecutively, as separate launches would be.
    // Its tag is then the previous one + 1, known without waiting for the
    // counter's reply.)
    if (tid == 0) {
        if (lk.index == 0) {
            *s_tag = static_cast<uint32_t>(atomicAdd(p.gen, 1ull) / static_cast<unsigned long long>(G)) + 1u;
        } else {
            atomicAdd(p.gen, 1ull);
            *s_tag += 1u;
        }
    }
    if (lk.wait_grid) pdl_wait();
    if (lk.x_from_slot) __syncthreads();   // the tag, for the poll on x below
    STYX_STAMP(1);

    // ------------------------------------------------ phase 1: RMSNorm + router
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    const float4 *n4 = reinterpret_cast<const float4 *>(p.norm_w);
    float4 *xn4 = reinterpret_cast<float4 *>(xn);
    const int H4 = H >> 2;
    // at most one float4 of each vector per thread (H <= 2048): the norm
    // weights and the first router row are loaded together with x
    const bool one = H4 <= kFusedBlock;
    float4 npre = make_float4(0.f, 0.f, 0.f, 0.f), rpre = npre;
    if (one && tid < H4) {
        npre = __ldg(n4 + tid);
        if (n_rows_mine > 0) rpre = __ldg(reinterpret_cast<const float4 *>(p.router + static_cast<size_t>(b) * H) + tid);
    }
    // one block reduction for both sum(x^2) and the first router row's
    // sum(r * w * x): logit = scale * sum(r * w * x) with scale the RMSNorm
    // factor (the same value as sum(r * x_norm) up to rounding order).  Every
    // router row goes through the same roundings, so equal rows give equal
    // logits and the top-k's index order decides between them.
    float ss = 0.f, rd = 0.f;
    float4 xr = npre;   // this thread's float4 of raw x (one-float4 case)
    float4 xin = npre;  // a later layer: the same float4 from the tagged words
    if (lk.x_from_slot) {
        // the previous layer's output rows, published with its tag (= this
        // layer's tag - 1); every warp polls in step, bounded, then regroups
        const uint32_t want = *s_tag - 1u;
        const bool on = one && tid < H4;
        const uint64_t *src = lk.xslot + 4 * static_cast<size_t>(on ? tid : 0);
        const long long t0 = clock64();
        for (;;) {
            uint64_t w0, w1, w2, w3;
            ld_slot2(src, w0, w1);
            ld_slot2(src + 2, w2, w3);
            const bool got = slot_tag(w0) == want && slot_tag(w1) == want && slot_tag(w2) == want &&
                             slot_tag(w3) == want;
            xin = make_float4(slot_val(w0), slot_val(w1), slot_val(w2), slot_val(w3));
            if (__all_sync(0xffffffffu, got || !on)) break;
            const long long dt = __shfl_sync(0xffffffffu, clock64() - t0, 0);
            if (dt > kSpinCycles) {
                if (lane == 0) atomicExch(p.err, kErrWaitRoute);
                break;
            }
            if (dt > kPollFreeCycles) __nanosleep(256);
        }
        __syncwarp();
    }
    // the id tables in shared memory, read while x travels: the slab
    // sources of the picked experts then cost no global round trip
    for (int i = tid; i < E; i += kFusedBlock) {
        smap[i] = p.remap ? __ldg(p.remap + i) : kSkip;
        smap[Ep + i] = p.pmap ? __ldg(p.pmap + i) : kSkip;
    }
    float *xown = wts + 16;   // this CTA's own rows of the raw x (<= 16), for the residual add
    for (int i = tid; i < H4; i += kFusedBlock) {
        const float4 v = lk.x_from_slot ? xin : __ldcg(x4 + i);
        if (lk.x_from_slot) {
            const float c[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++)
                if (4 * i + q >= dbeg && 4 * i + q < dend && 4 * i + q - dbeg < 16) xown[4 * i + q - dbeg] = c[q];
        }
        xn4[i] = v;   // raw x for now
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (one) {
            xr = v;
            rd = rwx4(rpre, npre, v);
        }
    }
    const float2 red2 = fblock_sum2(make_float2(ss, rd), red);   // (its barriers also publish the mbarrier inits)
    ss = red2.x;
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(H) + p.eps);
    if (one && n_rows_mine > 0 && tid == 0) {
        const float acc = scale * red2.y;
        st_slot(p.lgslot + (*s_tag & 1u) * E + b, acc, *s_tag);
        p.logits[b] = acc;   // debug view
    }
    for (int i = tid; i < H4; i += kFusedBlock) {   // same i -> thread mapping: no barrier needed
        float4 v = xn4[i];
        const float4 w = one ? npre : __ldg(n4 + i);
        v.x = v.x * scale * w.x;
        v.y = v.y * scale * w.y;
        v.z = v.z * scale * w.z;
        v.w = v.w * scale * w.w;
        xn4[i] = v;
    }
    STYX_STAMP(2);
    for (int j = one ? 1 : 0; j < n_rows_mine; j++) {   // further router rows (E > grid, or H > 2048)
        float acc = 0.f;
        const float4 *r4 = reinterpret_cast<const float4 *>(p.router + static_cast<size_t>(b + G * j) * H);
        if (one) {   // the first row's form and reduction tree
            if (tid < H4) acc = rwx4(__ldg(r4 + tid), npre, xr);
            acc = scale * fblock_sum(acc, red);
        } else {
            for (int i = tid; i < H4; i += kFusedBlock) {
                const float4 r = __ldg(r4 + i), v = xn4[i];
                acc += r.x * v.x + r.y * v.y + r.z * v.z + r.w * v.w;
            }
            acc = fblock_sum(acc, red);
        }
        if (tid == 0) {
            st_slot(p.lgslot + (*s_tag & 1u) * E + b + G * j, acc, *s_tag);
            p.logits[b + G * j] = acc;   // debug view
        }
    }
    __syncthreads();   // x_norm complete in shared memory, tag visible
    const uint32_t tag = *s_tag;
    STYX_STAMP(3);
    STYX_STAMP(4);

    // ------------------------------------------------ phase 2: x_norm digits
    // Every CTA keeps its own digits of x_norm for the gate/up dots; all
    // warps build them while the logits travel between CTAs.  (Warp 0 runs
    // the top-k alone afterwards: with other warps still busy on the SM its
    // shuffles and reductions were several times slower.)
    {
        const DigitsView dv{xd1, xd2, xd3, xsc};
        for (int g0 = warp; g0 < (H >> 5); g0 += 4 * kFusedWarps) {   // four groups' shuffle chains together
            float v[4];
            int gi[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int g = g0 + j * kFusedWarps;
                gi[j] = g < (H >> 5) ? g : -1;
                v[j] = g < (H >> 5) ? xn[g * 32 + lane] : 0.f;
            }
            digits_groups_warp<4>(v, gi, lane, dv);
        }
        if (b == 0)   // test / debug view of x_norm
            for (int i = tid; i < H; i += kFusedBlock) p.xnorm[i] = xn[i];
    }
    __syncthreads();
    STYX_STAMP(22);

    // ------------------------------------------------ phase 3: top-k (warp 0)
    // Warp 0 gathers the E logits into registers (element i on lane i % 32,
    // register i / 32), picks the k winners with warp reductions, resolves
    // their slabs and issues the copies; the softmax weights are computed
    // once the copies are in flight.
    if (warp == 0) {
        const int nper = (E + 31) >> 5;
        float lv[kLogitRegs];
        // The whole warp polls in step (no lane ever waits alone, so the
        // warp stays converged for the reductions that follow): each pass
        // re-reads the words still missing their tag; bounded (~1 s).
        uint32_t need = 0;   // bit j: word lane + 32 j not yet read with this launch's tag
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) {
            lv[j] = -INFINITY;
            if (j < nper && lane + 32 * j < E) need |= 1u << j;
        }
        const long long t0 = clock64();
        for (;;) {
            // every word of the lane is re-read each pass, all reads in
            // flight at once, with no lane-dependent branch
            uint64_t w[kLogitRegs];
#pragma unroll
            for (int j = 0; j < kLogitRegs; j++)
                if (j < nper) w[j] = ld_slot(p.lgslot + (tag & 1u) * E + min(lane + 32 * j, E - 1));
#pragma unroll
            for (int j = 0; j < kLogitRegs; j++)
                if (j < nper) {
                    const bool got = (need >> j & 1u) && slot_tag(w[j]) == tag;
                    lv[j] = got ? slot_val(w[j]) : lv[j];
                    need = got ? need & ~(1u << j) : need;
                }
            if (!__any_sync(0xffffffffu, need != 0)) break;
            // lane 0's clock decides for the warp: lanes need not read the
            // clock together, and a lane leaving alone would leave the others
            // in a warp-wide vote it never joins
            const long long dt = __shfl_sync(0xffffffffu, clock64() - t0, 0);
            if (dt > kSpinCycles) {
                if (lane == 0) atomicExch(p.err, kErrWaitRoute);
                break;
            }
            if (dt > kPollFreeCycles) __nanosleep(256);
        }
        // bring the warp back together before the reductions: after the
        // poll the lanes can run as separate groups, and every full-warp
        // shuffle or reduction then pays for regrouping them (measured at
        // several times its cost); a 32-thread named barrier reconverges it
        warp_converge(kBarWarp0);
        STYX_STAMP(5);
        uint32_t key[kLogitRegs];
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) key[j] = lv[j] > -INFINITY ? order_key(lv[j]) : 0u;
        int e = -1;            // lane s < k: the expert of slot s
        uint32_t ke = 0;       // and its key
        if (nper <= 4) warp_pick_sorted4(key, k, lane, e, ke);
        else warp_pick<kLogitRegs>(key, k, lane, e, ke);
        STYX_STAMP(17);
        // lane s < k: slot s's slab sources and id rows
        int hi = -1, ai = -1, fi = -1;
        if (lane < k) {
            const uint32_t hot = e >= 0 ? smap[e] : kSkip;
            if (hot != kSkip) {
                hi = static_cast<int>(hot);
            } else {
                const uint32_t am = e >= 0 ? smap[Ep + e] : kSkip;
                if (am != kSkip) ai = static_cast<int>(am);
                else fi = e;
            }
            src_g[lane] = fused_slot_src(p.gate, hi, ai, fi);
            src_u[lane] = fused_slot_src(p.up, hi, ai, fi);
            src_d[lane] = fused_slot_src(p.down, hi, ai, fi);
            if (b == 0) {
                if (e >= 0 && !p.quiet && (!src_g[lane] || !src_u[lane] || !src_d[lane])) atomicExch(p.err, kErrBadId);
                p.ids64[lane] = e;
                p.ids64[16 + lane] = hi;
                p.ids64[32 + lane] = ai;
                p.ids64[48 + lane] = fi;
            }
        }
        const int s = lane;
        __syncwarp();   // sources visible to every lane before the arrives that publish them
        STYX_STAMP(19);
        // ---- every expert byte this CTA needs: gate/up chunk c on lane c
        // (gate segments, then up segments, each with room for its 16-byte
        // cover), then the down rows of slot s on lane s
        if (lane < n_chunks) {
            const GuChunk c = gu_chunk(lane, p.ch, gbeg, nrows, F);
            uint8_t *cb = gubuf + static_cast<size_t>(lane) * p.gu_stride;
            const uint8_t *segs[4] = {nullptr, nullptr, nullptr, nullptr};
            uint32_t lens[4] = {0, 0, 0, 0};
            uintptr_t addr[4] = {0, 0, 0, 0};
            uint8_t *dst[4] = {cb, cb + seg_b_off(c.nA, p.rb_g), cb + p.gu_up_off,
                               cb + p.gu_up_off + seg_b_off(c.nA, p.rb_u)};
            const int nB = c.n - c.nA;
            if (src_g[c.sA]) segs[0] = src_g[c.sA] + static_cast<size_t>(c.rrA) * p.rb_g;
            if (src_u[c.sA]) segs[2] = src_u[c.sA] + static_cast<size_t>(c.rrA) * p.rb_u;
            if (nB > 0) {
                segs[1] = src_g[c.sA + 1];
                segs[3] = src_u[c.sA + 1];
            }
            uint32_t total = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (!segs[i]) continue;
                const int rows = (i & 1) ? nB : c.nA;
                const int rb = i < 2 ? p.rb_g : p.rb_u;
                cover16(segs[i], static_cast<size_t>(rows) * rb, addr[i], lens[i]);
                total += lens[i];
            }
            if (total == 0) {
                mbar_arrive(&full_gu[lane]);
            } else {
                mbar_arrive_expect_tx(&full_gu[lane], total);
                const uint64_t once = l2_evict_first();   // expert bytes are read once per token
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (lens[i])
                        bulk_g2s_hint(dst[i], reinterpret_cast<const void *>(addr[i]), lens[i], &full_gu[lane], once);
            }
        }
        STYX_STAMP(20);
        {   // the CTA's down rows of every slot, one chunk (rc >= dend - dbeg)
            const int n = dend - dbeg;
            uintptr_t a = 0;
            uint32_t len = 0;
            if (s < k && src_d[s] && n > 0)
                cover16(src_d[s] + static_cast<size_t>(dbeg) * p.rb_d, static_cast<size_t>(n) * p.rb_d, a, len);
            uint32_t total = len;
            warp_converge(kBarWarp0);   // after the per-chunk issue branches
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) {
                if (total == 0) mbar_arrive(&full_d[0]);
                else mbar_arrive_expect_tx(&full_d[0], total);
            }
            __syncwarp();
            if (len)
                bulk_g2s_hint(dbuf + static_cast<size_t>(s) * p.dslot_stride, reinterpret_cast<const void *>(a), len,
                              &full_d[0], l2_evict_first());
        }
        STYX_STAMP(21);
        // the logits and the picked ones stay in shared memory for the
        // softmax weights, computed after the gate/up phase (off this path)
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++)
            if (j < nper && lane + 32 * j < E) lgs[lane + 32 * j] = lv[j];
        if (lane < k) wts[lane] = ke ? key_value(ke) : -INFINITY;
    }
    __syncthreads();
    STYX_STAMP(7);
    {
        const int units = p.units_g, gs = p.gs_g, rpw = 32 / gs, stride = kFusedWarps * rpw;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        XUnit x;
        if (active) load_xunit<QG>(x, xd1, xd2, xd3, xsc, ug);
        bool ok = true;
        int waited = -1;
        bool first = true;
        // CTA row q = qb + grp; rows are dealt to the warps in arrival order
        for (int qb = warp * rpw; qb < nrows; qb += stride) {
            const int q = qb + grp;
            float g = 0.f, u = 0.f;
            int r = -1;
            if (q < nrows) {
                const int ci = q / p.ch;   // ch % rpw == 0: the whole lane group is in one chunk
                if (ci != waited) {
                    if (ok) ok = mbar_wait(&full_gu[ci], 0, p.err, kErrWaitFull);
                    waited = ci;
                }
                const GuChunk c = gu_chunk(ci, p.ch, gbeg, nrows, F);
                const int t = q - ci * p.ch;
                const bool inA = t < c.nA;
                const int s = inA ? c.sA : c.sA + 1;
                const int rr = inA ? c.rrA + t : t - c.nA;
                const int tt = inA ? t : t - c.nA;   // row inside its segment
                r = s * F + rr;
                const uint8_t *gsrc = src_g[s], *usrc = src_u[s];
                if (ok && gsrc && usrc && active) {
                    const uint8_t *cb = gubuf + static_cast<size_t>(ci) * p.gu_stride;
                    const uint8_t *gseg = inA ? gsrc + static_cast<size_t>(c.rrA) * p.rb_g : gsrc;
                    const uint8_t *useg = inA ? usrc + static_cast<size_t>(c.rrA) * p.rb_u : usrc;
                    const uint8_t *gb = cb + (inA ? 0u : seg_b_off(c.nA, p.rb_g)) +
                                        (reinterpret_cast<uintptr_t>(gseg) & 15) + static_cast<size_t>(tt) * p.rb_g;
                    const uint8_t *ub = cb + p.gu_up_off + (inA ? 0u : seg_b_off(c.nA, p.rb_u)) +
                                        (reinterpret_cast<uintptr_t>(useg) & 15) + static_cast<size_t>(tt) * p.rb_u;
                    g = unit_dot<QG>(gb, ug, x);
                    u = unit_dot<QG>(ub, ug, x);
                }
            }
            if (first) {
                STYX_STAMP_T(32, 8);
                first = false;
            }
            __syncwarp();   // regroup the lanes after the waits and branches above
            for (int o = gs >> 1; o; o >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, o);
                u += __shfl_xor_sync(0xffffffffu, u, o);
            }
            // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
            if (ug == 0 && r >= 0) __stcg(p.h + r, g / (1.0f + expf(-g)) * u);
        }
    }
    __syncthreads();   // the CTA's h rows are stored; region A is reused below
    STYX_STAMP(9);
    // Per-slot arrival counts of h (never reset): each CTA adds the number of
    // rows it stored for each slot it covers, so slot s of launch n is
    // complete at (n + 1) * F.  Thread 0 fences first, ordering the CTA's h
    // stores, which the barrier above made its own.
    if (tid == 0) {
        __threadfence();
        for (int r = gbeg; r < gend;) {
            const int s = r / F, e = min(gend, (s + 1) * F);
            atomicAdd(p.hcount + s * kHcStride, static_cast<unsigned long long>(e - r));
            r = e;
        }
    }
    if (warp == 1) {
        // softmax statistics over all E logits (lane-strided partials, fixed
        // shuffle tree) and the weights in slot order
        // (topk_softmax_f32.comp:47-52); wts[s] holds slot s's logit until here
        float mx = -INFINITY, sum = 0.f;
        for (int i = lane; i < E; i += 32) mx = fmaxf(mx, lgs[i]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (int i = lane; i < E; i += 32) sum += expf(lgs[i] - mx);
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float w = lane < k ? expf(wts[lane] - mx) / sum : 0.f;
        float wsum = 0.f;
        for (int t = 0; t < k; t++) wsum += __shfl_sync(0xffffffffu, w, t);
        if (lane < k) {
            const float wr = p.renorm ? w / wsum : w;
            wts[lane] = wr;
            if (b == 0) p.weights[lane] = wr;
        }
    }
    STYX_STAMP(10);

    if (lk.next_router) {   // warm L2 with the next layer's router rows and norm while h travels
        const uint64_t keep = l2_evict_last();
        for (int j = tid; j < n_rows_mine; j += kFusedBlock)
            prefetch_l2_hint(lk.next_router + static_cast<size_t>(b + G * j) * H, static_cast<uint32_t>(H) * 4u, keep);
        if (tid == kFusedBlock - 1) prefetch_l2_hint(lk.next_norm, static_cast<uint32_t>(H) * 4u, keep);
    }

    // ------------------------------------------------ phase 4: down + combine
    // The warps of slot s wait for slot s's h only, turn it into digits in
    // shared memory themselves and run the CTA's down rows for slot s; the
    // slots proceed independently until the combine.
    {
        const int units = p.units_d, gs = p.gs_d, rpw = 32 / gs;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const bool active = ug < units;
        const bool multi = k > kFusedWarps;
        const int nwps = multi ? 1 : kFusedWarps / k;
        const int slot0 = multi ? warp : warp / nwps;
        const int sub = multi ? 0 : warp % nwps;
        const int sstep = multi ? kFusedWarps : 1 << 30;
        const int gthreads = nwps * 32, gt = sub * 32 + lane;   // thread index inside the slot's warps
        const int n = dend - dbeg;                              // the CTA's down rows (one chunk)
        const unsigned long long htarget = static_cast<unsigned long long>(tag) * static_cast<unsigned long long>(F);
        bool ok = true;
        bool have_rows = false;
        for (int s = slot0; s < k; s += sstep) {
            if (gt == 0) {
                const long long t0 = clock64();
                while (ld_acquire_u64(p.hcount + s * kHcStride) < htarget) {
                    const long long dt = clock64() - t0;
                    if (dt > kSpinCycles) {
                        atomicExch(p.err, kErrWaitRoute);
                        break;
                    }
                    if (dt > kPollFreeCycles) __nanosleep(256);
                }
            }
            slot_group_sync(s, gthreads);
            if (s == slot0) STYX_STAMP(11);
            {   // h[s] -> digits: 16 elements per thread, two threads per 32-element group
                int8_t *d1 = hd1 + s * F;
                uint8_t *d2 = hd2 + s * F, *d3 = hd3 + s * F;
                float *sc = hsc + s * (F >> 5);
                const float4 *hv = reinterpret_cast<const float4 *>(p.h + static_cast<size_t>(s) * F);
                const int nparts = F >> 4, lim = ((nparts + 31) >> 5) << 5;
                for (int pidx = gt; pidx < lim; pidx += gthreads) {
                    const bool on = pidx < nparts;
                    float xv[16];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 q = on ? __ldcg(hv + pidx * 4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                        xv[4 * i] = q.x;
                        xv[4 * i + 1] = q.y;
                        xv[4 * i + 2] = q.z;
                        xv[4 * i + 3] = q.w;
                    }
                    digits_part<16>(xv, on, pidx, d1, d2, d3, sc);
                }
            }
            slot_group_sync(s, gthreads);
            XUnit x;
            if (active) load_xunit<QD>(x, hd1 + s * F, hd2 + s * F, hd3 + s * F, hsc + s * (F >> 5), ug);
            if (!have_rows) {
                if (ok) ok = mbar_wait(&full_d[0], 0, p.err, kErrWaitFull);
                have_rows = true;
                if (s == slot0) STYX_STAMP(12);
            }
            const uint8_t *src = src_d[s];
            const uint8_t *base = dbuf + static_cast<size_t>(s) * p.dslot_stride +
                                  (src ? (reinterpret_cast<uintptr_t>(src + static_cast<size_t>(dbeg) * p.rb_d) & 15) : 0);
            // two rows per lane group per pass: independent dot products in flight
            for (int t = sub * 2 * rpw; t < n; t += nwps * 2 * rpw) {
                const int ra = t + grp, rb = t + rpw + grp;
                float va = 0.f, vb = 0.f;
                if (ok && src && active && ra < n) va = unit_dot<QD>(base + static_cast<size_t>(ra) * p.rb_d, ug, x);
                if (ok && src && active && rb < n) vb = unit_dot<QD>(base + static_cast<size_t>(rb) * p.rb_d, ug, x);
                __syncwarp();   // regroup the lanes after the branches above
                for (int o = gs >> 1; o; o >>= 1) {
                    va += __shfl_xor_sync(0xffffffffu, va, o);
                    vb += __shfl_xor_sync(0xffffffffu, vb, o);
                }
                if (ug == 0 && ra < n) dpart[s * p.rc + ra] = va;
                if (ug == 0 && rb < n) dpart[s * p.rc + rb] = vb;
            }
        }
        __syncthreads();
        STYX_STAMP(13);
        if (p.ep) {
            // expert parallelism over peer memory (ep_sync.cuh): this CTA's
            // weighted rows of every slot to every peer as tagged words, then
            // the ranks' sum of the same rows, as the peers' words arrive,
            // added into x here
            const EpPeers &ep = *p.ep;
            const unsigned long long gen = ep_generation(ep);
            const unsigned tag = static_cast<unsigned>(gen);
            if (tid < n) {
                const int c = dbeg + tid;
                for (int s = 0; s < k; s++) {
                    const float v = ok ? __fmul_rn(wts[s], dpart[s * p.rc + tid]) : 0.f;
                    dpart[s * p.rc + tid] = v;
                    const size_t o = ep_index(ep, gen, ep.rank, s, c);
                    for (int q = 0; q < ep.world; q++)
                        if (q != ep.rank) ep_put(ep.inbox[q] + o, tag, v);
                }
                const unsigned long long *box = ep.inbox[ep.rank];
                bool live = true;
                float acc = 0.f;
                for (int s = 0; s < k; s++) {
                    float v = 0.f;
                    for (int q = 0; q < ep.world; q++)
                        v = __fadd_rn(v, q == ep.rank ? dpart[s * p.rc + tid]
                                                      : ep_get(box + ep_index(ep, gen, q, s, c), tag, live, p.err));
                    acc = __fadd_rn(acc, v);
                }
                p.x[c] = __fadd_rn(p.x[c], acc);
            }
            __syncthreads();
            ep_call_done(ep, gen, G);
        } else if (tid < n && p.partial) {
            // expert parallelism: each slot's weighted rows; the ranks' sum
            // (one non-zero contributor per slot) then goes through the combine
            for (int s = 0; s < k; s++)
                p.partial[static_cast<size_t>(s) * H + dbeg + tid] =
                    ok ? __fmul_rn(wts[s], dpart[s * p.rc + tid]) : 0.f;
        } else if (tid < n) {
            // the residual: the row as read from the tagged words when x came
            // that way (written by another CTA, perhaps still draining)
            float xv = lk.x_from_slot ? wts[16 + tid] : p.x[dbeg + tid];
            if (ok) {
                float acc = 0.f;
                for (int s = 0; s < k; s++) acc = __fadd_rn(acc, __fmul_rn(wts[s], dpart[s * p.rc + tid]));
                xv = __fadd_rn(xv, acc);
                // a layer with a successor hands x on only through the tagged
                // words; the last layer of the chain writes the caller's x
                if (!lk.x_to_slot) p.x[dbeg + tid] = xv;
            }
            // the next layer of the launch reads the row from here (also after
            // a wait gave up, so that it does not wait for the row as well)
            if (lk.x_to_slot) st_slot(lk.xslot + dbeg + tid, xv, tag);
        }
    }
    STYX_STAMP(14);
    // No CTA leaves with copies in flight into its shared memory, even after
    // a wait above gave up: thread 0 waits (bounded) for every barrier its
    // copies complete on (already complete on the normal path).
    if (tid == 0) {
        bool fine = true;
        for (int c = 0; c < n_chunks && fine; c++) fine = mbar_wait(&full_gu[c], 0, p.err, kErrWaitFull);
        if (fine) mbar_wait(&full_d[0], 0, p.err, kErrWaitFull);
    }
    // A chained launch that never waited on the grid dependency waits for it
    // before it ends (long resolved by now: every CTA of the previous launch
    // had written its x rows), so that the end of this grid still implies the
    // end of every earlier one on the stream.
    if (lk.index == 0 && !lk.wait_grid) pdl_wait();
#undef STYX_STAMP
#undef STYX_STAMP_T
}

template <int QG, int QD>
__global__ void __launch_bounds__(kFusedBlock, 1) k_moe_fused(const __grid_constant__ FusedArgs pa,
                                                                const __grid_constant__ LayerLink lk) {
    extern __shared__ __align__(128) uint8_t smem[];
    load_args(smem, pa, lk);
    __syncthreads();
    fused_layer<QG, QD>(smem);
}

// Several consecutive layers in one launch: the grid stays resident, and the
// boundary between layers is the exchange of x through tagged words instead
// of the end of one grid and the start of the next.
template <int QG, int QD>
__global__ void __launch_bounds__(kFusedBlock, 1) k_moe_fused_layers(const __grid_constant__ FusedLaunch la) {
    extern __shared__ __align__(128) uint8_t smem[];
    for (int li = 0; li < la.n; li++) {
        if (li) __syncthreads();   // every thread is done with the previous layer's shared memory
        const bool more = li + 1 < la.n;
        load_args(smem, la.layer[li],
                  LayerLink{li, li > 0, more, li == 0, la.xslot, more ? la.layer[li + 1].router : nullptr,
                            more ? la.layer[li + 1].norm_w : nullptr});
        __syncthreads();
        fused_layer<QG, QD>(smem);
    }
}

cudaError_t resident_fit(const void *kern, int threads, uint32_t smem, int grid) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    struct Fit {
        const void *kern;
        int dev;
        uint32_t smem;
        int threads, grid_max;
    };
    static std::mutex mu;
    static std::vector<Fit> fits;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Fit &f : fits)
            if (f.kern == kern && f.dev == dev && f.smem == smem && f.threads == threads)
                return grid <= f.grid_max ? cudaSuccess : cudaErrorCooperativeLaunchTooLarge;
    }
    // the attribute goes to the largest opt-in size (the launch's own smem
    // is what counts for residency), so a later, larger launch of the same
    // kernel never finds it set lower
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    // every large kernel asks for the same (largest) shared-memory carveout,
    // so consecutive launches of different kernels need no reconfiguration
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    int occ = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int grid_max = occ * sms;
    {
        std::lock_guard<std::mutex> lock(mu);
        fits.push_back(Fit{kern, dev, smem, threads, grid_max});
    }
    return grid <= grid_max ? cudaSuccess : cudaErrorCooperativeLaunchTooLarge;
}

// Launch with programmatic stream serialisation: the kernel lets the next
// one launch at entry and waits for the previous grid before it touches the
// workspace or x.  Every CTA must be resident at once (the tagged-slot reads
// are grid-wide waits): `coop` asks the driver for that (a cooperative
// launch); without it, co-residency follows from the grid being one CTA per
// SM on a device nothing else is using (the caller's promise,
// STYX_OPT_EXCLUSIVE), which lets each CTA start as soon as its SM is free
// instead of when the whole grid fits -- about 0.7 us per launch on B200.
// Either way a wait that cannot finish gives up after about a second.
template <class Kern, class... Args>
static cudaError_t launch_coop_pdl(Kern kern, bool coop, int grid, uint32_t smem, cudaStream_t st,
                                   const Args &...a) {
    cudaError_t e = resident_fit(reinterpret_cast<const void *>(kern), kFusedBlock, smem, grid);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kFusedBlock);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = coop ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a...);
}

cudaError_t launch_fused(const FusedArgs &a, const LayerLink &lk, int qg, int qd, int grid, uint32_t smem,
                         bool coop, cudaStream_t st) {
#define STYX_FUSED_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return launch_coop_pdl(k_moe_fused<G_, D_>, coop, grid, smem, st, a, lk);
    STYX_FUSED_CASE(STYX_Q4_K, STYX_Q6_K)
    STYX_FUSED_CASE(STYX_Q4_K, STYX_Q4_K)
    STYX_FUSED_CASE(STYX_Q5_K, STYX_Q6_K)
    STYX_FUSED_CASE(STYX_Q5_K, STYX_Q5_K)
    STYX_FUSED_CASE(STYX_Q8_0, STYX_Q8_0)
    STYX_FUSED_CASE(STYX_Q6_K, STYX_Q6_K)
#undef STYX_FUSED_CASE
    return cudaErrorNotSupported;
}

cudaError_t launch_fused_layers(const FusedLaunch &a, int qg, int qd, int grid, uint32_t smem, bool coop,
                                cudaStream_t st) {
#define STYX_FUSED_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return launch_coop_pdl(k_moe_fused_layers<G_, D_>, coop, grid, smem, st, a);
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
