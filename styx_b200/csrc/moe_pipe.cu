// moe_pipe.cu -- the MoE block of one layer as ONE kernel, with the down
// projection pipelined behind the gate/up projection slot by slot.
//
// Grid = one CTA per SM (every CTA resident: cooperative launch, or a plain
// launch on a device the caller owns), 16 warps.  CTA b of G covers, for
// EVERY slot s, gate/up rows [F*b/G, F*(b+1)/G) of slot s and down rows
// [H*b/G, H*(b+1)/G); all of those bytes fit in shared memory together and
// are requested at once.  Phases:
//   0  (before the grid dependency) barrier init; bulk copies of the CTA's
//      router rows and ffn_norm into shared memory -- weights, which the
//      previous kernel does not write; the next kernel may launch (PDL);
//   1  wait for the previous grid; the launch number; remap / pmap copied in
//      the background; RMSNorm of x and the router dot products of the
//      CTA's rows, each logit published as one tagged word;
//   2  warps 0-2 each gather the E logits and pick the top-k (the selection
//      of topk_softmax_f32.comp, identical in every warp and every CTA) and
//      resolve each slot's slab (hot / arena / full); warp 0 issues the gate
//      rows, warp 1 the up rows, warp 2 the down rows; warps 3-15 turn
//      x_norm into dp4a digits meanwhile;
//   3  gate/up warps (0-7): the CTA's row pairs slot by slot as their bytes
//      land; h = SiLU(g) * u is published per row as a tagged word, and the
//      CTA's last row of a slot adds the CTA's rows to the slot's counter;
//   4  slot groups of 16 / k warps: warps 8-15 (idle during phase 3) take
//      the first slots, whose h completes first, warps 0-7 the later ones
//      after their gate/up rows; a group waits for its slot's counter, reads
//      the slot's h words (tags checked), turns them into digits and runs
//      the CTA's down rows of the slot from shared memory -- the first slots'
//      down work overlaps the later slots' gate/up work.  Then the
//      slot-ordered combine x[r] += sum_s w[s] d[s][r] (moe_reduce_f32.comp),
//      or, for expert parallelism, partial[s][r] = w[s] d[s][r].
// Tags: launch number + 1, from the workspace's never-reset launch counter
// (bumped once by every CTA after the grid dependency resolved, so launches
// never interleave their numbers).  Logit and h words carry the tag and the
// h counters grow by F per slot per launch, so nothing in the workspace needs
// clearing between launches.  Every wait is bounded (~1 s) and reports
// through the device error word; no CTA exits with a bulk copy still landing
// in its shared memory.
#include <cfloat>

#include "common.cuh"
#include "kernels.h"
#include "moe_common.cuh"
#include "qdot.cuh"

namespace styx {

// shared-memory header
constexpr int kPBarGU = 0;        // 16 mbarriers: slot s's gate + up rows
constexpr int kPBarD = 128;       // 16 mbarriers: slot s's down rows
constexpr int kPBarPre = 256;     // router rows + ffn_norm
constexpr int kPBarMaps = 264;    // remap / pmap
constexpr int kPRed = 320;        // 32 floats of block-reduction scratch
constexpr int kPWts = 448;        // 16 floats: slot logits, then weights
constexpr int kPMisc = 512;       // ints: [0] tag, [1] active-slot mask, [2] a down wait gave up
constexpr int kPGcnt = 592;       // 16 ints: h rows of slot s this CTA has stored
constexpr int kPSrc = 656;        // 3 x 16 slab pointers
constexpr int kPXown = 1040;      // the CTA's raw x rows (<= 128 floats)
constexpr int kPArgs = 1552;      // a copy of PipeArgs
constexpr int kPHeader = static_cast<int>(kPipeHeader);
static_assert(kPSrc + 3 * 16 * 8 <= kPXown, "pipe header overflow");
static_assert(kPXown + 128 * 4 <= kPArgs, "pipe header overflow");
static_assert(kPArgs + static_cast<int>(sizeof(PipeArgs)) <= kPHeader, "PipeArgs does not fit its header slot");
static_assert(sizeof(PipeArgs) % 8 == 0, "PipeArgs size");

constexpr int kGuWarps = 8;                 // warps 0-7: gate/up; 8-15: down
constexpr int kBarW0 = 15;                  // 32-thread barriers 15, 14, 13 of warps 0-2 (phase 2)
constexpr int kHGroups = 12;                // 32-element groups of h[s] a warp converts: F / 32 / (16 / k)

// slot s's h digits (planes d1, d2, d3 of F bytes, then F / 32 scales)
__device__ __forceinline__ DigitsView hd_view_of(uint8_t *smem, const PipeArgs &p, int s, int F) {
    int8_t *d1 = reinterpret_cast<int8_t *>(smem + p.off_hd + static_cast<size_t>(s) * p.hd_stride);
    uint8_t *d2 = reinterpret_cast<uint8_t *>(d1) + F;
    uint8_t *d3 = d2 + F;
    return DigitsView{d1, d2, d3, reinterpret_cast<float *>(d3 + F)};
}

template <int QG, int QD>
__global__ void __launch_bounds__(kFusedBlock, 1) k_moe_pipe(const __grid_constant__ PipeArgs pa) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < static_cast<int>(sizeof(PipeArgs) / 8))
        reinterpret_cast<uint64_t *>(smem + kPArgs)[tid] = reinterpret_cast<const uint64_t *>(&pa)[tid];
    const PipeArgs &p = *reinterpret_cast<const PipeArgs *>(smem + kPArgs);
    uint64_t *bar_gu = reinterpret_cast<uint64_t *>(smem + kPBarGU);
    uint64_t *bar_d = reinterpret_cast<uint64_t *>(smem + kPBarD);
    uint64_t *bar_pre = reinterpret_cast<uint64_t *>(smem + kPBarPre);
    uint64_t *bar_maps = reinterpret_cast<uint64_t *>(smem + kPBarMaps);
    float *red = reinterpret_cast<float *>(smem + kPRed);
    float *wts = reinterpret_cast<float *>(smem + kPWts);
    int *misc = reinterpret_cast<int *>(smem + kPMisc);
    int *gcnt = reinterpret_cast<int *>(smem + kPGcnt);
    const uint8_t **src_g = reinterpret_cast<const uint8_t **>(smem + kPSrc);
    const uint8_t **src_u = src_g + 16;
    const uint8_t **src_d = src_u + 16;
    float *xown = reinterpret_cast<float *>(smem + kPXown);

    const int G = gridDim.x, b = blockIdx.x;
    const int H = pa.H, F = pa.F, E = pa.E, k = pa.k;
    const int gbeg = static_cast<int>(static_cast<long long>(F) * b / G);
    const int n_g = static_cast<int>(static_cast<long long>(F) * (b + 1) / G) - gbeg;   // rows of each slot
    const int dbeg = static_cast<int>(static_cast<long long>(H) * b / G);
    const int n_d = static_cast<int>(static_cast<long long>(H) * (b + 1) / G) - dbeg;
    const int n_rows_mine = b < E ? (E - 1 - b) / G + 1 : 0;   // router rows e = b + G*j

#define STYX_PSTAMP_T(t_, i_)                                                          \
    do {                                                                               \
        if (tid == (t_) && p.trace) p.trace[b * kTraceStamps + (i_)] = clock64();      \
    } while (0)
#define STYX_PSTAMP(i_) STYX_PSTAMP_T(0, i_)

    // ------------------------------------------------ phase 0
    if (tid < 16) {
        mbar_init(&bar_gu[tid], 1);
        mbar_init(&bar_d[tid], 1);
    } else if (tid == 16) {
        mbar_init(bar_pre, 1);
        mbar_init(bar_maps, 1);
    } else if (tid >= 32 && tid < 48) {
        gcnt[tid - 32] = 0;
    } else if (tid == 48) {
        misc[2] = 0;
    }
    fence_mbar_init();
    __syncthreads();
    STYX_PSTAMP(0);
    float *nrm = reinterpret_cast<float *>(smem + p.off_norm);
    float *rrows = reinterpret_cast<float *>(smem + p.off_router);
    if (tid == 0) {
        const uint32_t rb = static_cast<uint32_t>(H) * 4u;
        const uint64_t keep = l2_evict_last();
        mbar_arrive_expect_tx(bar_pre, rb * static_cast<uint32_t>(1 + n_rows_mine));
        bulk_g2s_hint(nrm, p.norm_w, rb, bar_pre, keep);
        for (int j = 0; j < n_rows_mine; j++)
            bulk_g2s_hint(rrows + static_cast<size_t>(j) * H, p.router + static_cast<size_t>(b + G * j) * H, rb, bar_pre,
                          keep);
    }
    pdl_trigger();
    pdl_wait();
    STYX_PSTAMP(1);

    // ------------------------------------------------ phase 1: launch number, RMSNorm, router
    uint8_t *maps = smem + p.off_maps;   // remap cover, then pmap cover
    if (tid == 0) {
        misc[0] = static_cast<int>(static_cast<uint32_t>(atomicAdd(p.gen, 1ull) / static_cast<unsigned long long>(G)) +
                                   1u);
        uintptr_t ra = 0, pa_ = 0;
        uint32_t rl = 0, pl = 0;
        if (p.remap) cover16(reinterpret_cast<const uint8_t *>(p.remap), static_cast<size_t>(E) * 4, ra, rl);
        if (p.pmap) cover16(reinterpret_cast<const uint8_t *>(p.pmap), static_cast<size_t>(E) * 4, pa_, pl);
        if (rl + pl == 0) {
            mbar_arrive(bar_maps);
        } else {
            const uint64_t keep = l2_evict_last();
            mbar_arrive_expect_tx(bar_maps, rl + pl);
            if (rl) bulk_g2s_hint(maps, reinterpret_cast<const void *>(ra), rl, bar_maps, keep);
            if (pl) bulk_g2s_hint(maps + p.maps_half, reinterpret_cast<const void *>(pa_), pl, bar_maps, keep);
        }
    }
    float *xn = reinterpret_cast<float *>(smem + p.off_x);
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    float4 *xn4 = reinterpret_cast<float4 *>(xn);
    const int H4 = H >> 2;
    float ss = 0.f;
    for (int i = tid; i < H4; i += kFusedBlock) {
        const float4 v = __ldcg(x4 + i);
        xn4[i] = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    // the router rows and ffn_norm (staged before the grid dependency)
    const bool ok_pre = mbar_wait(bar_pre, 0, p.err, kErrWaitFull);
    const float4 *n4 = reinterpret_cast<const float4 *>(nrm);
    // one block reduction for sum(x^2) and the first router row's
    // sum(r * w * x): logit = scale * sum(r * w * x), as the other single
    // kernel computes it (every router row through the same roundings)
    float rd = 0.f;
    if (n_rows_mine > 0 && ok_pre)
        for (int i = tid; i < H4; i += kFusedBlock)
            rd += rwx4(reinterpret_cast<const float4 *>(rrows)[i], n4[i], xn4[i]);
    const float2 red2 = fblock_sum2(make_float2(ss, rd), red);   // its barriers also publish misc[0]
    const uint32_t tag = static_cast<uint32_t>(misc[0]);
    const float scale = 1.0f / sqrtf(red2.x / static_cast<float>(H) + p.eps);
    if (n_rows_mine > 0 && tid == 0) {
        const float acc = scale * red2.y;
        st_slot(p.lgslot + (tag & 1u) * E + b, acc, tag);
        p.logits[b] = acc;   // debug view
    }
    for (int j = 1; j < n_rows_mine; j++) {   // further router rows (E > grid)
        float acc = 0.f;
        if (ok_pre)
            for (int i = tid; i < H4; i += kFusedBlock)
                acc += rwx4(reinterpret_cast<const float4 *>(rrows + static_cast<size_t>(j) * H)[i], n4[i], xn4[i]);
        acc = scale * fblock_sum(acc, red);
        if (tid == 0) {
            st_slot(p.lgslot + (tag & 1u) * E + b + G * j, acc, tag);
            p.logits[b + G * j] = acc;
        }
    }
    // the CTA's own raw rows (the residual of the combine), then x_norm
    for (int i = tid; i < n_d; i += kFusedBlock) xown[i] = xn[dbeg + i];
    __syncthreads();
    for (int i = tid; i < H4; i += kFusedBlock) {
        float4 v = xn4[i];
        const float4 w = n4[i];
        v.x = v.x * scale * w.x;
        v.y = v.y * scale * w.y;
        v.z = v.z * scale * w.z;
        v.w = v.w * scale * w.w;
        xn4[i] = v;
    }
    __syncthreads();
    STYX_PSTAMP(2);
    int8_t *xd1 = reinterpret_cast<int8_t *>(smem + p.off_xd);
    uint8_t *xd2 = reinterpret_cast<uint8_t *>(xd1) + H;
    uint8_t *xd3 = xd2 + H;
    float *xsc = reinterpret_cast<float *>(xd3 + H);
    // ------------------------------------------------ phase 2: top-k, sources, copies
    // Warps 0-2 each gather the logits and pick the top-k (the same ids in
    // every warp, as in every CTA); then warp 0 arms each slot's gate/up
    // barrier and issues its gate rows, warp 1 issues the up rows, warp 2
    // arms the down barrier and issues the down rows -- three issuing warps,
    // no barrier between the pick and the copies.  (A barrier's tx-count may
    // go below zero while a copy lands before its arming.)  Warps 3-15 turn
    // x_norm into digits meanwhile.
    float *lgs = reinterpret_cast<float *>(smem + p.off_lgs);
    uint8_t *gubuf = smem + p.off_gu;
    uint8_t *dbuf = smem + p.off_d;
    if (warp < 3) {
        const int nper = (E + 31) >> 5;
        float lv[kLogitRegs];
        uint32_t need = 0;
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) {
            lv[j] = -INFINITY;
            if (j < nper && lane + 32 * j < E) need |= 1u << j;
        }
        const long long t0 = clock64();
        for (;;) {
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
            const long long el = __shfl_sync(0xffffffffu, clock64() - t0, 0);
            if (el > kSpinCycles) {
                if (lane == 0 && warp == 0) atomicExch(p.err, kErrWaitRoute);
                break;
            }
            if (el > kPollFreeCycles) __nanosleep(256);
        }
        warp_converge(kBarW0 - warp);
        STYX_PSTAMP(4);
        uint32_t key[kLogitRegs];
#pragma unroll
        for (int j = 0; j < kLogitRegs; j++) key[j] = lv[j] > -INFINITY ? order_key(lv[j]) : 0u;
        int e = -1;
        uint32_t ke = 0;
        if (nper <= 4) warp_pick_sorted4(key, k, lane, e, ke);
        else warp_pick<kLogitRegs>(key, k, lane, e, ke);
        STYX_PSTAMP(5);
        if (warp == 0) {   // the logits and the picked ones stay for the softmax weights
#pragma unroll
            for (int j = 0; j < kLogitRegs; j++)
                if (j < nper && lane + 32 * j < E) lgs[lane + 32 * j] = lv[j];
            if (lane < k) wts[lane] = ke ? key_value(ke) : -INFINITY;
        }
        // lane s < k: slot s's slab sources
        const bool maps_ok = mbar_wait(bar_maps, 0, p.err, kErrWaitFull);
        const uint32_t *remap_s = reinterpret_cast<const uint32_t *>(maps + (reinterpret_cast<uintptr_t>(p.remap) & 15));
        const uint32_t *pmap_s =
            reinterpret_cast<const uint32_t *>(maps + p.maps_half + (reinterpret_cast<uintptr_t>(p.pmap) & 15));
        bool active = false;
        if (lane < k) {
            int hi = -1, ai = -1, fi = -1;
            const uint32_t hot = (e >= 0 && p.remap && maps_ok) ? remap_s[e] : kSkip;
            if (hot != kSkip) {
                hi = static_cast<int>(hot);
            } else {
                const uint32_t am = (e >= 0 && p.pmap && maps_ok) ? pmap_s[e] : kSkip;
                if (am != kSkip) ai = static_cast<int>(am);
                else fi = e;
            }
            const uint8_t *sg = fused_slot_src(p.gate, hi, ai, fi);
            const uint8_t *su = fused_slot_src(p.up, hi, ai, fi);
            const uint8_t *sd = fused_slot_src(p.down, hi, ai, fi);
            active = e >= 0 && sg && su && sd;
            const int s = lane;
            const uint64_t stream = l2_evict_first();
            uintptr_t ga = 0, ua = 0, da = 0;
            uint32_t gl = 0, ul = 0, dl = 0;
            if (active && n_g > 0) {
                cover16(sg + static_cast<size_t>(gbeg) * p.rb_g, static_cast<size_t>(n_g) * p.rb_g, ga, gl);
                cover16(su + static_cast<size_t>(gbeg) * p.rb_g, static_cast<size_t>(n_g) * p.rb_g, ua, ul);
            }
            if (active && n_d > 0)
                cover16(sd + static_cast<size_t>(dbeg) * p.rb_d, static_cast<size_t>(n_d) * p.rb_d, da, dl);
            uint8_t *gslot = gubuf + static_cast<size_t>(s) * p.gu_slot;
            if (warp == 0) {
                if (gl + ul) mbar_arrive_expect_tx(&bar_gu[s], gl + ul);
                else mbar_arrive(&bar_gu[s]);
                if (gl) bulk_g2s_hint(gslot, reinterpret_cast<const void *>(ga), gl, &bar_gu[s], stream);
                src_g[s] = active ? sg : nullptr;
                src_u[s] = active ? su : nullptr;
                if (b == 0) {
                    if (e >= 0 && !active && !p.quiet) atomicExch(p.err, kErrBadId);
                    p.ids64[s] = e;
                    p.ids64[16 + s] = hi;
                    p.ids64[32 + s] = ai;
                    p.ids64[48 + s] = fi;
                }
            } else if (warp == 1) {
                if (ul) bulk_g2s_hint(gslot + p.gu_up_off, reinterpret_cast<const void *>(ua), ul, &bar_gu[s], stream);
            } else {
                if (dl) mbar_arrive_expect_tx(&bar_d[s], dl);
                else mbar_arrive(&bar_d[s]);
                if (dl)
                    bulk_g2s_hint(dbuf + static_cast<size_t>(s) * p.d_slot, reinterpret_cast<const void *>(da), dl,
                                  &bar_d[s], stream);
                src_d[s] = active ? sd : nullptr;
            }
        }
        const uint32_t mask = __ballot_sync(0xffffffffu, active);
        if (warp == 0 && lane == 0) misc[1] = static_cast<int>(mask);
        __syncwarp();
        STYX_PSTAMP(7);
    } else {
        const DigitsView dv{xd1, xd2, xd3, xsc};
        for (int g0 = warp - 3; g0 < (H >> 5); g0 += 4 * (kFusedWarps - 3)) {
            float v[4];
            int gi[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int g = g0 + j * (kFusedWarps - 3);
                gi[j] = g < (H >> 5) ? g : -1;
                v[j] = g < (H >> 5) ? xn[g * 32 + lane] : 0.f;
            }
            digits_groups_warp<4>(v, gi, lane, dv);
        }
        if (b == 0)
            for (int i = tid - 96; i < H; i += kFusedBlock - 96) p.xnorm[i] = xn[i];   // debug view
    }
    __syncthreads();   // x digits, slab sources, slot mask, slot logits
    STYX_PSTAMP(6);
    const uint32_t amask = static_cast<uint32_t>(misc[1]);
    // The gate/up warps take their x_norm units into registers.  The down
    // warps later put the h digits of every slot over the route-phase
    // regions (norm, router rows, x_norm), never over these digits.
    XUnit xg;
    const bool gu_on = warp < kGuWarps && (lane & (p.gs_g - 1)) < p.units_g;
    if (gu_on) load_xunit<QG>(xg, xd1, xd2, xd3, xsc, lane & (p.gs_g - 1));
    if (warp < kGuWarps) {
        // ------------------------------------------------ phase 3: gate/up
        const int gs = p.gs_g, rpw = 32 / gs;
        const int ug = lane & (gs - 1), grp = lane / gs;
        const int n_items = k * n_g;
        // every slot's counter grows by F per launch: the CTA's rows of an
        // empty slot are counted here at once
        if (warp == 0 && lane < k && !(amask >> lane & 1u) && n_g > 0)
            red_add_u64(p.hcount + lane * kHcStride, static_cast<unsigned long long>(n_g));
        int waited = -1;
        bool ok = true;
        bool first = true;
        for (int qb = warp * rpw; qb < n_items; qb += kGuWarps * rpw) {
            const int q = qb + grp;
            float g = 0.f, u = 0.f;
            int s = -1, i = 0;
            if (q < n_items) {
                s = q / n_g;
                i = q - s * n_g;
                if (amask >> s & 1u) {
                    if (s != waited) {
                        if (ok) ok = mbar_wait(&bar_gu[s], 0, p.err, kErrWaitFull);
                        waited = s;
                    }
                    if (ok && gu_on) {
                        const uint8_t *gslot = gubuf + static_cast<size_t>(s) * p.gu_slot;
                        const size_t off = static_cast<size_t>(i) * p.rb_g;
                        const uint8_t *gr =
                            gslot + (reinterpret_cast<uintptr_t>(src_g[s] + static_cast<size_t>(gbeg) * p.rb_g) & 15) + off;
                        const uint8_t *ur = gslot + p.gu_up_off +
                                            (reinterpret_cast<uintptr_t>(src_u[s] + static_cast<size_t>(gbeg) * p.rb_g) & 15) +
                                            off;
                        g = unit_dot<QG>(gr, ug, xg);
                        u = unit_dot<QG>(ur, ug, xg);
                    }
                } else {
                    s = -1;   // an empty slot: no h rows
                }
            }
            if (first) {
                STYX_PSTAMP_T(0, 8);
                first = false;
            }
            __syncwarp();
            for (int o = gs >> 1; o; o >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, o);
                u += __shfl_xor_sync(0xffffffffu, u, o);
            }
            // swiglu split (ops2.rs:305-308): g / (1 + exp(-g)) * u
            if (ug == 0 && s >= 0) {
                const float hv = g / (1.0f + expf(-g)) * u;
                st_slot_plain(p.hslot + static_cast<size_t>(s) * F + gbeg + i, hv, tag);
                __stcg(p.h + static_cast<size_t>(s) * F + gbeg + i, hv);   // debug view
                // the CTA's last row of slot s counts all n_g of them at once: a
                // hint for the readers, which check the tags
                if (atomicAdd(gcnt + s, 1) == n_g - 1)
                    red_add_u64(p.hcount + s * kHcStride, static_cast<unsigned long long>(n_g));
            }
        }
        STYX_PSTAMP(9);
    }
    // ------------------------------------------------ phase 4: down, by slot groups
    // Every warp joins a slot group of nw = 16 / k warps (slot s: group s,
    // then s + 16 / nw, ...).  Warps 8-15, free while the gate/up warps work,
    // form the groups of the first slots, whose h is complete first; warps
    // 0-7 take the later slots once their gate/up rows are done.  A group
    // polls its slot's counter, reads the slot's h words (tags checked, a
    // missing word read again), turns them into digits (warp `sub` of the
    // group holds 32-element groups sub, sub + nw, ...), then runs the CTA's
    // down rows of the slot, two rows per lane group in flight.
    {
        const int nw = k >= kFusedWarps ? 1 : kFusedWarps / k;     // warps per slot group
        const int ngroups = kFusedWarps / nw;
        const int wr = (warp + kGuWarps) % kFusedWarps;             // warps 8-15 first
        const int grp_id = wr / nw, sub = wr % nw;
        const int gthreads = nw * 32;
        float *dpart = reinterpret_cast<float *>(smem + p.off_dpart);
        if (wr == 0) {
            // softmax statistics over all E logits and the slot weights
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
                const float wv = p.renorm ? w / wsum : w;
                wts[lane] = wv;
                if (b == 0) p.weights[lane] = wv;
            }
        }
        const int gs = p.gs_d, rpw = 32 / gs;
        const int ug = lane & (gs - 1), lgrp = lane / gs;
        const bool on = ug < p.units_d;
        const unsigned long long target = static_cast<unsigned long long>(tag) * static_cast<unsigned long long>(F);
        const int ngrp32 = F >> 5;   // 32-element groups of h[s]
        bool ok = true;              // one value per warp
        for (int s = grp_id; s < k; s += ngroups) {
            if (!(amask >> s & 1u)) {
                for (int r = sub * 32 + lane; r < n_d; r += gthreads) dpart[s * p.rows_d + r] = 0.f;
                continue;
            }
            const long long t0 = clock64();
            // the slot's counter: every CTA has stored its rows of h[s]
            if (ok) {
                for (;;) {
                    const unsigned long long c = lane == 0 ? ld_relaxed_u64(p.hcount + s * kHcStride) : 0ull;
                    if (__shfl_sync(0xffffffffu, c >= target ? 1 : 0, 0)) break;
                    const long long el = __shfl_sync(0xffffffffu, clock64() - t0, 0);
                    if (el > kSpinCycles) {
                        if (lane == 0) {
                            atomicExch(p.err, kErrWaitRoute);
                            atomicOr(misc + 2, 1);
                        }
                        ok = false;
                        break;
                    }
                    if (el > kPollFreeCycles) __nanosleep(256);
                }
            }
            if (p.trace && sub == 0 && lane == 0 && s < 8) p.trace[b * kTraceStamps + 14 + s] = clock64();
            // every word of this warp's 32-element groups (sub, sub + nw, ...:
            // at most kHGroups) read in one pass, then their digits in one
            // interleaved batch
            const DigitsView hv = hd_view_of(smem, p, s, F);
            {
                float v[kHGroups];
                int gi[kHGroups];
                uint32_t need = 0;
#pragma unroll
                for (int j = 0; j < kHGroups; j++) {
                    const int g = sub + j * nw;
                    gi[j] = g < ngrp32 ? g : -1;
                    v[j] = 0.f;
                    if (g < ngrp32) need |= 1u << j;
                }
                while (ok) {
                    uint64_t w[kHGroups];
#pragma unroll
                    for (int j = 0; j < kHGroups; j++)
                        w[j] = (need >> j & 1u) ? ld_slot(p.hslot + static_cast<size_t>(s) * F + gi[j] * 32 + lane) : 0ull;
#pragma unroll
                    for (int j = 0; j < kHGroups; j++) {
                        const bool hit = (need >> j & 1u) && slot_tag(w[j]) == tag;
                        v[j] = hit ? slot_val(w[j]) : v[j];
                        need = hit ? need & ~(1u << j) : need;
                    }
                    if (!__any_sync(0xffffffffu, need != 0)) break;
                    const long long el = __shfl_sync(0xffffffffu, clock64() - t0, 0);
                    if (el > kSpinCycles) {
                        if (lane == 0) {
                            atomicExch(p.err, kErrWaitRoute);
                            atomicOr(misc + 2, 1);
                        }
                        ok = false;
                    }
                }
                __syncwarp();   // regroup after the poll before the digits' shuffles
                digits_groups_warp<kHGroups>(v, gi, lane, hv);
            }
            if (nw > 1) asm volatile("bar.sync %0, %1;" ::"r"(1 + grp_id), "r"(gthreads) : "memory");
            else __syncwarp();
            if (s == 0) STYX_PSTAMP_T(32 * kGuWarps, 10);
            XUnit x;
            if (on) load_xunit<QD>(x, hv.d1, hv.d2, hv.d3, hv.scale, ug);
            const bool got_rows = ok && mbar_wait(&bar_d[s], 0, p.err, kErrWaitFull);
            const uint8_t *base = dbuf + static_cast<size_t>(s) * p.d_slot +
                                  (reinterpret_cast<uintptr_t>(src_d[s] + static_cast<size_t>(dbeg) * p.rb_d) & 15);
            // four rows per lane group per pass: independent dot products in flight
            for (int t = sub * 4 * rpw; t < n_d; t += nw * 4 * rpw) {
                float vr[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int r = t + q * rpw + lgrp;
                    vr[q] = (got_rows && on && r < n_d) ? unit_dot<QD>(base + static_cast<size_t>(r) * p.rb_d, ug, x)
                                                         : 0.f;
                }
                __syncwarp();
                for (int o = gs >> 1; o; o >>= 1)
#pragma unroll
                    for (int q = 0; q < 4; q++) vr[q] += __shfl_xor_sync(0xffffffffu, vr[q], o);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int r = t + q * rpw + lgrp;
                    if (ug == 0 && r < n_d) dpart[s * p.rows_d + r] = vr[q];
                }
            }
            if (p.trace && sub == 0 && lane == 0 && s < 8) p.trace[b * kTraceStamps + 22 + s] = clock64();
        }
        __syncthreads();   // every slot's rows and the weights
        STYX_PSTAMP(11);
        const bool fine = misc[2] == 0;
        for (int r = tid; r < n_d; r += kFusedBlock) {
            if (p.partial) {
                for (int s = 0; s < k; s++)
                    p.partial[static_cast<size_t>(s) * H + dbeg + r] =
                        fine ? __fmul_rn(wts[s], dpart[s * p.rows_d + r]) : 0.f;
            } else if (fine) {
                float acc = 0.f;
                for (int s = 0; s < k; s++) acc = __fadd_rn(acc, __fmul_rn(wts[s], dpart[s * p.rows_d + r]));
                p.x[dbeg + r] = __fadd_rn(xown[r], acc);
            }
        }
        STYX_PSTAMP(12);
    }
    // No CTA leaves with copies in flight into its shared memory, even after
    // a wait above gave up: thread 0 waits (bounded) on every armed barrier.
    __syncthreads();
    if (tid == 0) {
        bool fine = true;
        for (int s = 0; s < k && fine; s++) {
            fine = mbar_wait(&bar_gu[s], 0, p.err, kErrWaitFull);
            if (fine) fine = mbar_wait(&bar_d[s], 0, p.err, kErrWaitFull);
        }
        if (fine) fine = mbar_wait(bar_pre, 0, p.err, kErrWaitFull);
        if (fine) mbar_wait(bar_maps, 0, p.err, kErrWaitFull);
        STYX_PSTAMP(13);
    }
#undef STYX_PSTAMP
#undef STYX_PSTAMP_T
}

template <class Kern>
static cudaError_t launch_pipe_kernel(Kern kern, const PipeArgs &a, bool coop, int grid, uint32_t smem,
                                      cudaStream_t st) {
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
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_pipe(const PipeArgs &a, int qg, int qd, int grid, uint32_t smem, bool coop, cudaStream_t st) {
#define STYX_PIPE_CASE(G_, D_) \
    if (qg == G_ && qd == D_) return launch_pipe_kernel(k_moe_pipe<G_, D_>, a, coop, grid, smem, st);
    STYX_PIPE_CASE(STYX_Q4_K, STYX_Q6_K)
    STYX_PIPE_CASE(STYX_Q4_K, STYX_Q4_K)
    STYX_PIPE_CASE(STYX_Q5_K, STYX_Q6_K)
    STYX_PIPE_CASE(STYX_Q5_K, STYX_Q5_K)
    STYX_PIPE_CASE(STYX_Q8_0, STYX_Q8_0)
    STYX_PIPE_CASE(STYX_Q6_K, STYX_Q6_K)
#undef STYX_PIPE_CASE
    return cudaErrorNotSupported;
}

}  // namespace styx
