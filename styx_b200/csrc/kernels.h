// kernels.h -- host-side launch interface of the styx B200 kernels
// (internal to libstyx_moe.so; the public surface is include/styx_moe.h).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace styx {

// One expert tensor with its placement (see styx_expert_tensor).
struct ExpSrc {
    const uint8_t *full;
    const uint8_t *hot;
    const uint8_t *arena;
    uint64_t slab;
    uint64_t aslab;
    uint32_t nfull, nhot, narena;   // id bounds of each source
};

struct RouteArgs {
    const float *x;          // residual f32[H]
    const float *norm_w;     // ffn_norm f32[H] or null
    float eps;
    const float *router;     // f32[E][H]
    int E, H, k, renorm;
    const uint32_t *remap, *pmap;
    float *xnorm;            // out f32[H]
    int8_t *xd1;             // out digit planes of xnorm
    uint8_t *xd2, *xd3;
    float *xscale;           // out f32[H/32]
    float *logits;           // out f32[E]
    float *weights;          // out f32[k]
    int32_t *ids64;          // out: the layer's 64-int id block
    unsigned *counter;       // zero on entry, zero on exit
    int *err;
};

struct GateUpArgs {
    ExpSrc gate, up;
    const int32_t *ids64;
    const int8_t *xd1;
    const uint8_t *xd2, *xd3;
    const float *xscale;
    float *h;                // out f32[k][F]
    int H, F, k;
    int rb_g, rb_u;          // row bytes
    int units, gs;           // 64-element units per row, lane group size
    int ch, nst;             // rows per chunk, pipeline stages
    uint32_t stage_bytes, up_off;
    int quiet;               // a slot whose fallback full tensor is null is not this device's: no error
    int *err;
};

struct DownArgs {
    ExpSrc down;
    const int32_t *ids64;
    const float *h;          // f32[k][F]
    const float *w;          // f32[k]
    float *x;                // residual f32[H], += combine
    float *partial;          // optional f32[k][H]: w[s]*d[s][r] per slot, written instead of the combine into x
    int quiet;               // as GateUpArgs::quiet
    int H, F, k, rb;
    int units, gs;
    int rc, nst;             // rows per chunk, stages
    uint32_t stage_bytes, slot_stride;
    uint32_t dig_off, part_off, stage_off;
    int *err;
};

// the single-kernel MoE block (moe_fused.cu)
// Expert parallelism over NVLink peer memory (styx_ep): every rank's inbox
// ([2][world][k][H] tagged words: f32 bits | call generation << 32; a half
// per call parity, a row per sending rank), this rank's call counter (calls
// completed) and the CTAs of the current call that have finished.  Lives in
// device memory (one copy per rank, written once when the ranks connect).
constexpr int kEpMaxRanks = 8;
struct EpPeers {
    unsigned long long *inbox[kEpMaxRanks];
    unsigned long long *calls;
    unsigned *done;
    int rank, world, k, H;
};

struct FusedArgs {
    float *x;
    const float *norm_w;
    float eps;
    const float *router;
    int E, H, F, k, renorm;
    const uint32_t *remap, *pmap;
    ExpSrc gate, up, down;
    int32_t *ids64;
    float *weights;
    float *logits;           // workspace f32[E] (debug view)
    float *xnorm;            // workspace f32[H] (debug view, written by CTA 0)
    float *h;                // workspace f32[k][F] (debug view)
    // grid-wide exchange of the logits: {value bits, tag} words; a launch's
    // tag is (launch number) + 1, the launch number read from *gen (old / grid)
    uint64_t *lgslot;        // workspace u64[E]
    unsigned long long *gen; // workspace, incremented once per CTA per launch, never reset
    unsigned long long *hcount; // workspace: rows of h stored per slot (slot s at s * kHcStride), never reset
    int *err;
    long long *trace;        // optional: kTraceStamps clock64 stamps per CTA (phase boundaries)
    // expert parallelism (single-layer launches only): when set, the block
    // writes partial[s][r] = w[s] * d[s][r] instead of adding into x, and a
    // slot whose expert has no source here is another rank's (contributes 0)
    float *partial;
    // expert parallelism over peer memory (single-layer launches, partial
    // unset): each slot's weighted rows go to every peer's inbox, and the
    // ranks' sum is added into x by the CTA that owns the rows
    const EpPeers *ep;
    int quiet;
    // shared-memory plan (every chunk of a CTA is resident at once)
    uint32_t off_a, off_part, off_ring, off_down;
    int ch;                  // gate/up rows per chunk (<= 16 chunks per CTA, a multiple of 32 / gs_g)
    uint32_t gu_up_off;      // offset of the up rows inside a chunk
    uint32_t gu_stride;      // bytes per gate/up chunk
    int rb_g, rb_u, rb_d;
    int rc;                  // down output rows per chunk (<= 16 chunks per CTA)
    uint32_t dstage_bytes, dslot_stride;
    int units_g, gs_g, units_d, gs_d;
};

// the per-slot h counters sit one 128-byte line apart (u64 stride), so the
// adds of different slots do not queue at one L2 slice
constexpr int kHcStride = 16;

// the MoE block of a batch of tokens on the tensor cores (batch.cu)
struct BatchArgs {
    float *x;                    // [B][H] residuals, += the block
    const float *norm_w;
    float eps;
    const float *router;         // f32[E][H]
    int E, H, F, k, renorm, B;
    int rb_g, rb_d;              // row bytes of gate/up and of down
    const uint32_t *remap, *pmap;
    ExpSrc gate, up, down;
    int32_t *ids;                // [B][64] id blocks
    float *weights;              // [B][k]
    __half *xh;                  // workspace [B][H]: x_norm as f16
    int *n_used;                 // workspace: used experts
    int *used_e, *cnt, *off;     // workspace [E], [E], [E + 1]: per used expert its id, pairs, first pair
    int *pair;                   // workspace [B * k]: pairs b * k + s grouped by expert
    int *pv;                     // workspace [B * k]: the pair has an expert here
    const uint8_t **srcs;        // workspace [E][3]: gate, up, down slab of each used expert
    __half *panel_x;             // workspace [E][npm][H]: per used expert its tokens' x_norm, B-panel layout
    __half *panel_h;             // workspace [E][npm][F]: per used expert its pairs' SiLU(g) * u, B-panel layout
    int npm;                     // rows of a panel at most: n_tokens rounded up to 16
    float *d;                    // workspace [smax_d][B * k][H]: down output per pair, per K piece
    float *logits;               // workspace [B][E]
    float *gpart, *upart;        // workspace [smax_g][B * k][F]: gate / up per K piece
    int *item_cnt;               // workspace [n_item_cnt]: pieces done per (expert, tile)
    int n_item_cnt;
    int *split_d;                // workspace [2]: the K pieces of down (0) and gate/up (1)
    int sms;                     // CTAs of a GEMM launch: the SM count
    uint32_t *src_sel;           // workspace [E]: per used expert its source (kind << 28 | slot; 0 hot, 1 arena, 2 full)
    int quiet;                   // a slot with no source here is not an error
    int *err;
};
// TMA descriptors of the expert matrices of one GEMM side (q4_K / q5_K: row
// chunks on 16-byte boundaries): per matrix and source (hot, arena, full) a
// 3-D map {row bytes, rows, slabs} with a box of one chunk x 128 rows
struct TmaSet {
    CUtensorMap m[2][3];
};
int batch_split_max(int K);
bool batch_supported(int qg, int qd);
bool batch_uses_tma(int qt);
cudaError_t launch_batch(const BatchArgs &a, int qg, int qd, const TmaSet &gu, const TmaSet &dn, cudaStream_t st);

// How a single-kernel layer connects to the layers before and after it (see
// moe_fused.cu): chain flags and the x exchange words.
struct LayerLink {
    int index;                   // position of the layer in the launch
    bool x_from_slot, x_to_slot;
    bool wait_grid;              // griddepcontrol.wait before touching x / the workspace
    uint64_t *xslot;             // workspace u64[H]
    const float *next_router, *next_norm;
};

// Several consecutive layers in one launch (k_moe_fused_layers): their
// arguments travel by value as one kernel parameter, under the 32 KiB limit.
constexpr int kMaxFusedLayers = 80;
struct FusedLaunch {
    int n;                   // layers in this launch, 1..kMaxFusedLayers
    uint64_t *xslot;         // workspace u64[H]: x rows passed between layers as tagged words
    FusedArgs layer[kMaxFusedLayers];
};
static_assert(sizeof(FusedLaunch) <= 32764, "FusedLaunch exceeds the kernel parameter limit");

struct MatVecIdArgs {
    const uint8_t *a;
    uint64_t expert_bytes;
    int n_expert;
    int *err;
    int nrows, ncols, rb;
    const int32_t *ids;
    int n_ids;
    const float *x;
    int stride_b, ne11;
    float *y;
    int stride_d;
    int units, gs;
    int rows_per_cta;              // a multiple of kMvRowStep(gs)
    // three-source form (src3[0] non-null): ids is a 64-int id block and slot
    // s reads from the last of hot (row 16), arena (32), full (48) whose id is
    // set and in range -- what one launch per source, in that order, leaves
    const uint8_t *src3[3];
    uint64_t stride3[3];
    int count3[3];
};
// rows a CTA of k_matvec_id covers per pass: 8 warps x (32 / gs) rows x 4 in flight
constexpr int kMvRowStep(int gs) { return 8 * (32 / gs) * 4; }

struct GatherArgs {
    const uint8_t *src[3];
    uint64_t src_bytes[3];
    uint8_t *dst[3];
    uint64_t dst_bytes[3];
    const int32_t *ids;
    int n_expert;
    int *err;
    int layer, k;
};

// launchers (return the launch error)
cudaError_t launch_route(const RouteArgs &a, cudaStream_t st);
cudaError_t launch_gate_up(const GateUpArgs &a, int qtype, int grid, cudaStream_t st);
// wide: 16 consumer warps (a dense GEMV) instead of 8
cudaError_t launch_down(const DownArgs &a, int qtype, int grid, uint32_t smem, cudaStream_t st, bool wide = false);
cudaError_t launch_matvec_id(const MatVecIdArgs &a, int qtype, cudaStream_t st);
cudaError_t launch_rms_norm(const float *x, const float *w, float eps, int ncols, int nrows,
                            float *out, cudaStream_t st);
cudaError_t launch_matvec_f32(const float *a, int nrows, int ncols, int stride_a, const float *x,
                              float *d, cudaStream_t st);
cudaError_t launch_topk(const float *logits, int n, int k, int renorm, const uint32_t *remap,
                        const uint32_t *pmap, float *weights, int32_t *ids64, cudaStream_t st);
cudaError_t launch_swiglu(const float *g, const float *u, float *out, int n, cudaStream_t st);
cudaError_t launch_moe_reduce(const float *d, const float *w, float *x, int ne, int k,
                              cudaStream_t st);
cudaError_t launch_combine_partial(const float *partial, float *x, int ne, int k, cudaStream_t st);
// the cross-rank sum + combine over peer memory (styx_ep_combine, moe_kernels.cu)
constexpr int kEpCols = 128;   // columns of x per CTA
struct EpCombineArgs {
    const float *partial;                         // this rank's f32[k][H]
    float *x;                                     // [H], += the slot-ordered sum
    const EpPeers *ep;                            // the ranks' inboxes, this rank's call counter (device memory)
    int H;
    int *err;
};
cudaError_t launch_ep_combine(const EpCombineArgs &a, cudaStream_t st);
cudaError_t launch_gather(const GatherArgs &a, cudaStream_t st);
cudaError_t launch_synth_quant(int qtype, uint8_t *dst, uint64_t nrows, int ncols, uint64_t seed,
                               float sigma, cudaStream_t st);
cudaError_t launch_synth_f32(float *dst, uint64_t n, uint64_t seed, uint64_t offset, float sigma,
                             cudaStream_t st);

// leaves `msg` for styx_last_error() and returns `code` (api.cu)
int set_error(int code, const char *msg);

// ------------------------------------------------ attention half of a decode layer (attn.cu)
struct QkRopeArgs {
    float *q, *k;                  // [n_heads][hd], [n_kv][hd]: normalised and rotated in place
    const float *v;                // [n_kv][hd]
    const float *q_norm, *k_norm;  // [hd] or null (no per-head norm)
    float eps;
    const int32_t *pos;            // device: the token's position
    double theta_scale;            // freq_base^(-2/hd)
    int n_heads, n_kv, hd, kv_dim, n_tokens, n_ctx;
    float *kcache, *vcache;        // [n_ctx][kv_dim] or null
    int *err;                      // device error word (a position outside the caches)
};
struct AttnArgs {
    const float *q, *kcache, *vcache;
    float *out;
    float *part_acc, *part_ml;     // workspace: [n_heads][n_splits][hd], [n_heads][n_splits][2]
    int n_t, hd, kv_dim, gqa, n_kv;
    float scale;
    int tps, n_splits;             // tokens per split, splits
};
struct GetRowsArgs {
    const uint8_t *w;              // [nrows][row_bytes] blocks of qtype
    long long row_bytes;
    int qtype, nrows, ncols;
    const int32_t *rows;           // device: n row indices
    int n;
    float *out;                    // [n][ncols]
    int *err;
};
cudaError_t launch_get_rows(const GetRowsArgs &a, cudaStream_t st);
// scratch: u64[kArgmaxCtas] partial maxima, then a u32 ticket (zero between calls)
cudaError_t launch_argmax(const float *x, int n, int32_t *out, void *scratch, cudaStream_t st);
// the attention half of a layer in one cooperative kernel (attn_fused.cu);
// head_dim 128
struct AttnFusedArgs {
    float *x;                          // [H] in/out
    const float *attn_norm;
    float eps;
    const uint8_t *wq, *wk, *wv, *wo;  // row-major blocks; q, k, o of one qtype, v of another
    int rb_q, rb_v, rb_o;              // row bytes (k as q)
    int H, n_heads, n_kv;
    const float *q_norm, *k_norm;      // [128] or null
    double theta_scale;
    float scale;
    int n_t;                           // cache rows read; the token's position is n_t - 1
    float *kcache, *vcache;            // [n_ctx][n_kv * 128]
    int tps, n_splits;
    // workspace
    float *qkv;                        // [n_heads*128 + 2*n_kv*128]
    float *part_acc, *part_ml;         // [n_heads][n_splits][128], [n_heads][n_splits][2]
    int8_t *att_d1;                    // att as digits ([n_heads*128] each, scales [n_heads*4])
    uint8_t *att_d2, *att_d3;
    float *att_sc;
    unsigned long long *gen, *head_cnt, *split_cnt, *att_cnt;   // zero at workspace init
    int *err;
    long long *trace;                  // STYX_OPT_TRACE: clock64 stamps [CTA][16], else null
    uint32_t off_dig, off_f32, off_w1, off_w2, off_kv, off_rope;
};
constexpr int kAttnTraceStamps = 16;
constexpr int kPreRows = 32;   // cache rows of K and of V a CTA prefetches (async copies)
bool attn_fused_supported(int qw, int qv);
int attn_fused_threads();
cudaError_t launch_attn_fused(const AttnFusedArgs &a, int qw, int qv, int grid, uint32_t smem, bool coop,
                              cudaStream_t st);

// The attention half of a decode layer as one launch of thread-block
// clusters (attn_cluster.cu): one cluster of C CTAs per kv head, head_dim
// 128.  The cluster computes its q heads, k and v rows, the attention of its
// q heads over the cache rows (split over its CTAs, merged through
// distributed shared memory), and its columns' share of Wo . att; the CTA
// that completes a row block last over the n_kv clusters adds the shares in
// cluster order into x.
struct AttnClusterArgs {
    float *x;                          // [H] in/out
    const float *attn_norm;
    float eps;
    const uint8_t *wq, *wk, *wv, *wo;  // row-major blocks; q, k, o of one qtype, v of another
    int rb_q, rb_v, rb_o;              // row bytes (k as q)
    int H, n_heads, n_kv;
    const float *q_norm, *k_norm;      // [128] or null
    double theta_scale;
    float scale;
    int n_t;                           // cache rows read; the token's position is n_t - 1
    float *kcache, *vcache;            // [n_ctx][n_kv * 128]
    float *opart;                      // workspace [n_kv][H]: each cluster's share of the o rows
    unsigned *cnt;                     // workspace: per row block (kCntStride apart) the clusters done; 0 between launches
    int *err;
    long long *trace;                  // STYX_OPT_TRACE: clock64 stamps [CTA][16], else null
    int C, tps, npre;                  // CTAs per cluster, cache rows per CTA, of them prefetched into shared memory
    uint32_t off_x, off_dig, off_q, off_rope, off_sc, off_acc, off_mrecv, off_att, off_adig, off_o, off_w, off_kv;
};
constexpr uint32_t kAttnClusterHeader = 128;   // shared-memory header bytes of the cluster form
bool attn_cluster_supported(int qw, int qv);
int attn_cluster_max_active(int qw, int qv, int C, uint32_t smem);
cudaError_t launch_attn_cluster(const AttnClusterArgs &a, int qw, int qv, uint32_t smem, cudaStream_t st);

constexpr int kAttnMaxSplits = 256;
constexpr int kArgmaxCtas = 296;   // partial maxima of styx_argmax_f32
size_t attn_smem_bytes(int gqa, int hd, int tps);
cudaError_t launch_qk_norm_rope_kv(const QkRopeArgs &a, cudaStream_t st);
cudaError_t launch_attn_decode(const AttnArgs &a, cudaStream_t st);
cudaError_t launch_add_f32(const float *x, const float *y, float *d, int n, cudaStream_t st);

// A launch with programmatic stream serialisation: the kernel may be
// scheduled while the previous one on the stream drains (its CTAs start once
// every CTA of the previous kernel has started).  Every kernel launched this
// way begins with griddepcontrol.launch_dependents + griddepcontrol.wait, so
// nothing it reads or writes is touched before the previous grid completed.
template <class Kern, class... Args>
inline cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Whether `grid` CTAs of `kern` (threads, smem bytes each) can all be
// resident on the current device: cudaSuccess or
// cudaErrorCooperativeLaunchTooLarge.  The function attribute and the
// occupancy query run once per (kernel, device, smem) and are cached, so an
// eager caller does not pay them on every launch.
cudaError_t resident_fit(const void *kern, int threads, uint32_t smem, int grid);

// coop: a cooperative launch; false when the caller promised the device to
// itself (STYX_OPT_EXCLUSIVE)
cudaError_t launch_fused(const FusedArgs &a, const LayerLink &lk, int qg, int qd, int grid, uint32_t smem,
                         bool coop, cudaStream_t st);
cudaError_t launch_fused_layers(const FusedLaunch &a, int qg, int qd, int grid, uint32_t smem, bool coop,
                                cudaStream_t st);
bool fused_supported(int qg, int qd);
int fused_block_threads();
constexpr uint32_t kFusedHeader = 1792;

// The MoE block as one launch of thread-block clusters (moe_cluster.cu): one
// cluster of C CTAs per selected slot.  Every cluster routes the token itself
// (its CTAs split the router rows and exchange the logits through
// distributed shared memory), streams slot s's gate/up rows and down rows
// split over its CTAs, exchanges h through distributed shared memory, and
// writes slot s's down rows; the CTA that completes a row block last (one
// counter per block) adds the k slots in slot order into x.
struct ClusterArgs {
    float *x;                // residual f32[H]: read, then += the block (unless partial)
    const float *norm_w;
    float eps;
    const float *router;     // f32[E][H]
    int E, H, F, k, renorm;
    const uint32_t *remap, *pmap;
    ExpSrc gate, up, down;
    int32_t *ids64;
    float *weights;
    float *logits;           // debug views, written by cluster 0's first CTA (h: by every CTA, its rows)
    float *xnorm;
    float *h;                // [k][F]
    float *y;                // workspace f32[k][H]: the down rows of each slot
    unsigned *cnt;           // workspace: per row block (kCntStride apart) the slots done; 0 between launches
    int *err;
    long long *trace;        // optional: kTraceStamps clock64 stamps per CTA
    float *partial;          // expert parallelism: w[s] * d[s][r] per slot instead of the combine
    int quiet;
    // plan
    int C;                   // CTAs per cluster
    int rb_g, rb_u, rb_d;
    int units_g, gs_g, units_d, gs_d;
    int ng, chg;             // gate/up chunks per CTA (<= 8) and row pairs per chunk
    uint32_t off_lg, off_x, off_xd, off_hf, off_hd, off_y, off_gu, off_dn;   // shared-memory regions
    uint32_t gu_stride, gu_up_off;
};
constexpr int kCntStride = 32;          // u32 words between the row-block counters (one 128-byte line each)
constexpr int kClusterMaxC = 16;
constexpr uint32_t kClusterHeader = 2048;
bool cluster_supported(int qg, int qd);
cudaError_t launch_cluster(const ClusterArgs &a, int qg, int qd, uint32_t smem, cudaStream_t st);
// clusters of a launch that can be resident at once (0 if the query fails)
int cluster_max_active(int qg, int qd, int C, uint32_t smem);
constexpr int kTraceStamps = 32;   // phase stamps per CTA (STYX_OPT_TRACE)

// shared-memory plan of the fused kernels (computed on the host)
int gate_up_smem(const GateUpArgs &a);
constexpr int kConsumerWarps = 8;
constexpr int kWideConsumerWarps = 16;
constexpr int kFusedThreads = 32 * (kConsumerWarps + 1);

}  // namespace styx
