/*
 * styx_moe.h -- C ABI of libstyx_moe.so: the Qwen3-MoE MoE block of
 * aDirtyScoundrel/styx on NVIDIA B200 (sm_100a).
 *
 * The library replaces, for the MoE-block hot path, the operator layer that
 * crates/model's MoeModel drives through crates/vk-backend (ash/Vulkan +
 * SPIR-V).  Each entry point below names the reference interface it takes
 * the place of (path:line inside the reference project).
 *
 * Conventions
 *   - Every function returns 0 (STYX_OK) or a negative STYX_E* code and, on
 *     error, leaves a message for styx_last_error() (thread-local).  The
 *     reference returns Result<_, String> (crates/vk-backend/src/lib.rs).
 *   - Pointers are device pointers (or STYX_MEM_HOST pinned, device-mapped
 *     host pointers where stated); sizes are in bytes unless stated.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *     Every op is stream-ordered and asynchronous; nothing here waits for the
 *     device unless stated (styx_stream_sync, styx_download to pageable).
 *   - No function allocates device memory during a hot-path op: the MoE
 *     block uses a caller-provided workspace (styx_moe_workspace_bytes).
 *   - A ctx is not thread-safe; use one ctx per host thread.  Calls made on
 *     different streams with the same workspace race.
 */
#ifndef STYX_MOE_H
#define STYX_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STYX_OK 0
#define STYX_EINVAL (-1)      /* bad argument / unsupported shape */
#define STYX_ECUDA (-2)       /* CUDA runtime error */
#define STYX_ENOMEM (-3)      /* allocation failed */
#define STYX_ETIMEOUT (-4)    /* a device-side bounded wait gave up */
#define STYX_EUNSUPPORTED (-5)

/* expert id meaning "no expert" in the id rows (topk_softmax_f32.comp:27) */
#define STYX_SKIP 0xFFFFFFFFu
/* i32 per layer in the ids buffer: rows [0,16) original ids, [16,32) hot
 * index, [32,48) arena slot, [48,64) full-tensor id (moe.rs:1158-1162,
 * topk_softmax_f32.comp:5-11).  256 bytes, as bids is laid out there. */
#define STYX_IDS_PER_LAYER 64
#define STYX_MAX_TOPK 16      /* moe.rs:587 */
#define STYX_MAX_EXPERTS 512  /* topk_softmax_f32.comp:3, onboard.rs:24 */

/* ggml quantisation types accepted for expert matrices (moe.rs:24-40) */
typedef enum {
    STYX_F32 = 0,
    STYX_Q8_0 = 8,
    STYX_Q4_K = 12,
    STYX_Q5_K = 13,
    STYX_Q6_K = 14
} styx_qtype;

/* memory kinds for styx_alloc */
typedef enum {
    STYX_MEM_DEVICE = 0,      /* HBM (create_buffer, lib.rs:568) */
    STYX_MEM_HOST = 1         /* pinned + device-mapped host memory, the GTT
                                 tier (create_buffer_host[_shared],
                                 lib.rs:756, 802) */
} styx_mem_kind;

typedef struct styx_ctx styx_ctx;
typedef void *styx_stream;
typedef void *styx_event;

/* ------------------------------------------------------------ device */
const char *styx_last_error(void);
/* Gpu::new (crates/vk-backend/src/lib.rs:356): bind CUDA device `device`. */
int styx_init(int device, styx_ctx **out);
/* Drop for Gpu (lib.rs:1602-1612). */
void styx_destroy(styx_ctx *ctx);
/* Gpu::vram_bytes (lib.rs:534-554): total device memory. */
int styx_vram_bytes(styx_ctx *ctx, uint64_t *out);
/* SM count and name of the bound device (Gpu::device_name). */
int styx_device_info(styx_ctx *ctx, int *sm_count, char *name, int name_len);
/* Reads and clears the device-side error word that bounded waits and
 * device-side id bounds checks set (STYX_ETIMEOUT / STYX_EINVAL if one fired
 * since the last call).  Synchronises the stream.  After a timeout, re-run
 * styx_moe_workspace_init on the workspaces in use. */
int styx_check_device_error(styx_ctx *ctx, styx_stream stream);

/* Options.  STYX_OPT_MOE_KERNELS selects how styx_moe_block (and
 * styx_moe_block_ep) runs: 0 = auto (the cluster form when the shape and
 * formats fit, else the single cooperative kernel when they fit, else three
 * kernels), 1 = single kernel only (STYX_EUNSUPPORTED if it does not fit),
 * 2 = three kernels, 3 = cluster form only (STYX_EUNSUPPORTED if it does not
 * fit).  The cluster form is one launch of thread-block clusters, one
 * cluster per selected slot; it needs no co-resident grid.
 * STYX_OPT_MOE_LAST_PATH (read only) = 1 (single kernel), 2 (three kernels),
 * 3 (host-read form: some full tensor is in STYX_MEM_HOST memory), 4 (single
 * kernel, several layers per launch, styx_moe_blocks), 5 (single kernel, one
 * chained launch per layer, styx_moe_blocks) or 6 (cluster form), the form
 * the last styx_moe_block[s] call used.  STYX_OPT_TRACE = 1 makes the single
 * kernel and the cluster form record 32 clock64 stamps per CTA at their
 * phase boundaries into the workspace (styx_moe_workspace_view 4:
 * int64[CTAs][32]).
 * STYX_OPT_MOE_LAYERS picks how styx_moe_blocks runs single-kernel layers:
 * 0 (default) one independent styx_moe_block call per layer, 1 up to 80
 * layers in one persistent launch (its layer loop spills registers), 2 one
 * launch per layer, chained (a layer starts without waiting for the
 * previous grid and takes x from it as tagged words).  On B200 the default
 * measures fastest. */
#define STYX_OPT_MOE_KERNELS 1
#define STYX_OPT_MOE_LAST_PATH 2
#define STYX_OPT_TRACE 3
#define STYX_OPT_MOE_LAYERS 4
/* STYX_OPT_EXCLUSIVE = 1: the caller promises that nothing else runs on the
 * device while the single MoE kernel does (no other stream, process or
 * MPS client).  Its CTAs must all be resident at once; by default a
 * cooperative launch makes sure of that, which holds each launch until the
 * whole grid fits.  With the promise the launch is a plain one (one CTA per
 * SM, so an otherwise idle device holds them all) and each CTA starts as
 * soon as its SM frees: ~0.7 us less per layer on B200.  Broken, the
 * promise costs no hang: a wait that cannot finish gives up after about a
 * second with STYX_ETIMEOUT. */
#define STYX_OPT_EXCLUSIVE 5
/* STYX_OPT_ATTN_KERNELS: styx_attn_block as one cooperative kernel, else as
 * one launch of thread-block clusters (one cluster per kv head), when the
 * shape fits (0, default); the cooperative kernel always (1:
 * STYX_EUNSUPPORTED otherwise); seven kernels (2); the cluster form always
 * (3: STYX_EUNSUPPORTED otherwise).  STYX_OPT_ATTN_LAST_PATH (read only): 1
 * (one cooperative kernel), 2 (seven) or 3 (cluster form), the form the last
 * styx_attn_block used. */
#define STYX_OPT_ATTN_KERNELS 6
#define STYX_OPT_ATTN_LAST_PATH 7
/* STYX_OPT_MOE_LAST_CLUSTER (read only): CTAs per cluster of the last
 * cluster-form launch (16 when the device holds k such clusters at once, else
 * the largest smaller size that it does). */
#define STYX_OPT_MOE_LAST_CLUSTER 8
int styx_set_option(styx_ctx *ctx, int option, int64_t value);
int styx_get_option(styx_ctx *ctx, int option, int64_t *value);

/* ------------------------------------------------------------ memory */
/* create_buffer / create_buffer_host / create_buffer_host_shared
 * (lib.rs:568, 756, 802).  Returned pointers are 256-byte aligned. */
int styx_alloc(styx_ctx *ctx, uint64_t bytes, int kind, void **out);
/* destroy_buffer (lib.rs:1517) */
int styx_free(styx_ctx *ctx, void *ptr);
/* upload (lib.rs:1033): dst[dst_off..+n] = src[0..n] (host -> device). */
int styx_upload(styx_ctx *ctx, void *dst, uint64_t dst_off, const void *src,
                uint64_t n, styx_stream stream);
/* download (lib.rs:1175): dst[0..n] = src[src_off..+n] (device -> host). */
int styx_download(styx_ctx *ctx, void *dst, const void *src, uint64_t src_off,
                  uint64_t n, styx_stream stream);
/* copy_region (lib.rs:1192-1217), any direction the pointers allow. */
int styx_copy(styx_ctx *ctx, const void *src, uint64_t src_off, void *dst,
              uint64_t dst_off, uint64_t n, styx_stream stream);
int styx_memset(styx_ctx *ctx, void *dst, int value, uint64_t n,
                styx_stream stream);

/* ----------------------------------------------------- streams / events
 * Replace Batch submit / submit_async / timeline semaphores
 * (lib.rs:200-333, 700-712). */
int styx_stream_create(styx_ctx *ctx, styx_stream *out);
int styx_stream_destroy(styx_ctx *ctx, styx_stream stream);
int styx_stream_sync(styx_ctx *ctx, styx_stream stream);
int styx_event_create(styx_ctx *ctx, styx_event *out);
int styx_event_destroy(styx_ctx *ctx, styx_event ev);
int styx_event_record(styx_ctx *ctx, styx_event ev, styx_stream stream);
int styx_stream_wait_event(styx_ctx *ctx, styx_stream stream, styx_event ev);

/* Recorded per-token work (Batch::begin / submit, lib.rs:56-231): ops issued
 * on `stream` between styx_graph_begin and styx_graph_end are recorded, not
 * run; styx_graph_launch replays them on any stream.  The recording keeps
 * the pointers it was given: the buffers must outlive the graph. */
typedef void *styx_graph;
int styx_graph_begin(styx_ctx *ctx, styx_stream stream);
int styx_graph_end(styx_ctx *ctx, styx_stream stream, styx_graph *out);
int styx_graph_launch(styx_ctx *ctx, styx_graph graph, styx_stream stream);
int styx_graph_destroy(styx_ctx *ctx, styx_graph graph);

/* ------------------------------------------------------- single ops
 * One entry point per dispatch that MoeModel::forward_token records for the
 * MoE block (crates/model/src/moe.rs:1974-2062). */

/* rms_norm_f32 with weight multiply (moe.rs:1975-1982; semantics
 * kernels.rs:58-67): out[r][c] = x[r][c] * 1/sqrt(mean_c(x^2)+eps) * w[c].
 * w may be NULL (no multiply). */
int styx_rms_norm(styx_ctx *ctx, styx_stream stream, const float *x,
                  const float *w, float eps, int ncols, int nrows, float *out);

/* matvec_strided_f32 (shaders/matvec_strided_f32.comp, moe.rs:1984-1996):
 * d[r] = sum_c a[r*stride_a + c] * x[c]. */
int styx_matvec_f32(styx_ctx *ctx, styx_stream stream, const float *a,
                    int nrows, int ncols, int stride_a, const float *x,
                    float *d);

/* topk_softmax_f32 (shaders/topk_softmax_f32.comp, moe.rs:1998-2016).
 * remap / pmap may be NULL (all SKIP).  ids64: the layer's 64-int block. */
int styx_topk_softmax(styx_ctx *ctx, styx_stream stream, const float *logits,
                      int n, int k, int renorm, const uint32_t *remap,
                      const uint32_t *pmap, float *weights, int32_t *ids64);

/* mul_mat_vec_id_<type>_f32_f32 with the MatVecIdPush meaning
 * (crates/vk-backend/src/ops.rs:120-147, moe.rs:1561-1606; offsets per
 * kernels.rs:124-131), for slot s < n_ids with ids[s] != SKIP:
 *   y[s*stride_d + r] = sum_c deq(A_e)[r][c] * x[(s % ne11)*stride_b + c]
 *   A_e = a + e * expert_bytes, e = ids[s], rows of row_bytes(qtype, ncols).
 * SKIP slots leave y untouched (the patched SKIP early-out).  Ids >= n_expert
 * are skipped too and reported through styx_check_device_error. */
int styx_mul_mat_vec_id(styx_ctx *ctx, styx_stream stream, int qtype,
                        const void *a, uint64_t expert_bytes, int n_expert,
                        int nrows, int ncols, const int32_t *ids, int n_ids,
                        const float *x, int stride_b, int ne11, float *y,
                        int stride_d);

/* swiglu_f32 split mode (ops.rs:337-370, moe.rs:2025-2038; CPU form
 * ops2.rs:305-308): out[i] = g[i] / (1 + exp(-g[i])) * u[i]. */
int styx_swiglu(styx_ctx *ctx, styx_stream stream, const float *g,
                const float *u, float *out, int n);

/* moe_reduce_f32 (shaders/moe_reduce_f32.comp, moe.rs:2050-2062):
 * x[i] += sum_{s<k} w[s] * d[s*ne + i], slot order. */
int styx_moe_reduce(styx_ctx *ctx, styx_stream stream, const float *d,
                    const float *w, float *x, int ne, int k);

/* gather_slabs_f32 (shaders/gather_slabs_f32.comp:40-85, recorder
 * moe.rs:1706-1744): for s < k with ids[s] != SKIP copy the three source
 * slabs of expert ids[s] into arena slot layer*k+s.  Sources may be
 * STYX_MEM_HOST (the GTT tier); ids are device memory.  All byte counts
 * must be multiples of 16.  Ids >= n_expert are skipped and reported
 * through styx_check_device_error. */
int styx_gather_slabs(styx_ctx *ctx, styx_stream stream, const void *src_g,
                      const void *src_u, const void *src_d,
                      uint64_t src_bytes_g, uint64_t src_bytes_u,
                      uint64_t src_bytes_d, void *arena_g, void *arena_u,
                      void *arena_d, uint64_t dst_bytes_g,
                      uint64_t dst_bytes_u, uint64_t dst_bytes_d,
                      const int32_t *ids, int n_expert, int layer, int k);

/* The prefetch form of the same copy, driven by host-known ids (the
 * prepare_prefetch path, moe.rs:2169-2383): one cudaMemcpyAsync per slab on
 * `stream` (a copy-engine transfer from pinned host memory). */
int styx_gather_slabs_async(styx_ctx *ctx, styx_stream stream,
                            const void *src_g, const void *src_u,
                            const void *src_d, uint64_t src_bytes_g,
                            uint64_t src_bytes_u, uint64_t src_bytes_d,
                            void *arena_g, void *arena_u, void *arena_d,
                            uint64_t dst_bytes_g, uint64_t dst_bytes_u,
                            uint64_t dst_bytes_d, const int32_t *host_ids,
                            int n_expert, int layer, int k);

/* ----------------------------------------------------- fused MoE block */

/* One expert tensor (ExpMat, moe.rs:97-106) with its placement.  For slot
 * s the kernels read, in this order of precedence:
 *   hot   + ids[16+s] * slab_bytes        if ids[16+s] != SKIP
 *   arena + ids[32+s] * arena_slab_bytes  if ids[32+s] != SKIP
 *   full  + ids[48+s] * slab_bytes        otherwise
 * which is the three-way split of rec_matvec_id (moe.rs:1649-1700) in one
 * kernel.  `hot` and `arena` are device memory.  `full` is device memory, or
 * STYX_MEM_HOST memory for the cold tier: styx_moe_block then reads those
 * slabs in place over the host link (mul_mat_vec_id dispatches per source, as
 * the reference reads its GTT tensors), and styx_gather_slabs[_async] can
 * bring predicted cold slabs into the arena ahead of time.
 * Bases 16-byte aligned; slab_bytes and arena_slab_bytes multiples of 16.
 * n_hot / n_arena bound the hot indices and arena slots (full ids are
 * bounded by n_expert): an id out of range is skipped and reported through
 * styx_check_device_error. */
typedef struct styx_expert_tensor {
    const void *full;
    const void *hot;
    const void *arena;
    uint64_t slab_bytes;
    uint64_t arena_slab_bytes;
    int32_t qtype;
    uint32_t n_hot;
    uint32_t n_arena;
} styx_expert_tensor;

/* Per-layer MoE weights (Layer, moe.rs:108-144). */
typedef struct styx_moe_layer {
    const float *ffn_norm;     /* f32[n_embd] */
    const float *router;       /* f32[n_expert][n_embd] (ffn_gate_inp) */
    const uint32_t *remap;     /* u32[n_expert] expert -> hot index, or NULL */
    const uint32_t *pmap;      /* u32[n_expert] expert -> arena slot, or NULL */
    styx_expert_tensor gate, up, down;
} styx_moe_layer;

/* Hyper-parameters (HParams, moe.rs:550-587). */
typedef struct styx_moe_dims {
    int32_t n_embd;            /* H */
    int32_t n_ff;              /* F, expert_feed_forward_length */
    int32_t n_expert;          /* E */
    int32_t n_expert_used;     /* k */
    int32_t norm_topk;         /* renormalise top-k weights (ArchCfg.norm_topk) */
    float rms_eps;
} styx_moe_dims;

/* Workspace bytes styx_moe_block needs for these dims. */
int styx_moe_workspace_bytes(const styx_moe_dims *dims, uint64_t *out);
/* Zeroes a workspace (required once before its first use). */
int styx_moe_workspace_init(styx_ctx *ctx, styx_stream stream, void *ws,
                            uint64_t bytes);

/* The MoE block of one layer (moe.rs:1974-2062):
 *   xnorm = rms(x, ffn_norm); logits = router . xnorm; topk_softmax;
 *   h = silu(gate_e . xnorm) * (up_e . xnorm); d = down_e . h;
 *   x += sum_s w[s] d[s]  (slot order).
 * x: f32[n_embd], updated in place.  ids: the ids buffer; this layer's
 * 64-int block at ids + layer*64 is written.  weights_out: f32[k] or NULL.
 * Three kernels on `stream`: route, gate/up+SiLU, down+combine. */
int styx_moe_block(styx_ctx *ctx, styx_stream stream,
                   const styx_moe_dims *dims, const styx_moe_layer *layer_w,
                   int layer, float *x, int32_t *ids, float *weights_out,
                   void *workspace, uint64_t workspace_bytes);

/* The MoE blocks of n_layers consecutive layers of one token, first_layer
 * + i using layers[i], each layer's x the previous one's output: the same
 * results as n_layers styx_moe_block calls in order (weights_out, when not
 * NULL, is f32[n_layers][k]).  When every layer takes the single-kernel
 * form (the MoE sections of forward_token, moe.rs:1974-2062, when nothing
 * runs between them, as in a stack of MoE blocks), STYX_OPT_MOE_LAYERS = 1
 * or 2 pass x from layer to layer as tagged words in the workspace instead
 * of through the caller's x: 1 runs up to 80 layers (with the same formats)
 * in one launch, 2 chains one launch per layer.  Otherwise, and by default,
 * the layers run as separate calls. */
int styx_moe_blocks(styx_ctx *ctx, styx_stream stream,
                    const styx_moe_dims *dims, const styx_moe_layer *layers,
                    int n_layers, int first_layer, float *x, int32_t *ids,
                    float *weights_out, void *workspace, uint64_t workspace_bytes);

/* Expert parallelism (no counterpart in the reference, which runs on one
 * device): the form of styx_moe_block for a model whose experts are split
 * over ranks.  Every rank routes (the same kernels on the same data give
 * every rank the same ids and weights); this rank holds only its own
 * experts, in layer_w's hot buffers (remap: expert -> local slot or SKIP)
 * and/or arena, with `full` NULL in each tensor, and a slot whose expert it
 * does not hold contributes zero.  partial: f32[k * n_embd], written
 * partial[s*n_embd + r] = w[s] * d[s][r] for the slots held here and 0 for
 * the others; x is read (RMSNorm, router), not updated.  Sum `partial` over
 * the ranks (one all-reduce per layer, e.g. NCCL), then styx_moe_combine
 * adds it into x.  Runs the single kernel (its partial-output epilogue)
 * when the shape fits and STYX_OPT_MOE_KERNELS is not 2, else the
 * three-kernel form (STYX_OPT_MOE_LAST_PATH says which). */
int styx_moe_block_ep(styx_ctx *ctx, styx_stream stream,
                      const styx_moe_dims *dims, const styx_moe_layer *layer_w,
                      int layer, const float *x, int32_t *ids,
                      float *weights_out, float *partial, void *workspace,
                      uint64_t workspace_bytes);
/* ------------------------------------------------- batched decode
 * The MoE block for a batch of n_tokens (1..STYX_MAX_BATCH) tokens of one
 * layer; no counterpart in the reference, which decodes one token at a time
 * (examples/generate_moe.rs:46-53).  x: f32[n_tokens][n_embd], updated in
 * place as n_tokens separate styx_moe_block calls would; ids: n_tokens id
 * blocks (STYX_IDS_PER_LAYER ints each, layout of topk_softmax_f32.comp);
 * weights_out: f32[n_tokens][k].  The tokens routed to one expert share its
 * bytes: per used expert a grouped GEMM on the tensor cores (tcgen05, f16
 * operands dequantised from the blocks, f32 accumulation in TMEM), M = 128
 * weight rows per tile, N = the expert's tokens.  Operands rounded to f16:
 * within 1e-3 of max|dx| of the f32 path.  Formats q4_K, q5_K, q6_K (q8_0
 * is rejected with STYX_EINVAL); gate and up share one format; experts must
 * be in device memory (hot / arena / full), x, router and ffn_norm 16-byte
 * aligned.  The result is a function of the inputs alone (bit-identical on
 * repeat and for any expert placement).  The workspace:
 * styx_moe_batch_workspace_bytes(dims, n_tokens), no initialisation. */
#define STYX_MAX_BATCH 64
int styx_moe_batch_workspace_bytes(const styx_moe_dims *dims, int n_tokens, uint64_t *out);
int styx_moe_block_batch(styx_ctx *ctx, styx_stream stream,
                         const styx_moe_dims *dims, const styx_moe_layer *layer_w,
                         int n_tokens, float *x, int32_t *ids,
                         float *weights_out, void *workspace,
                         uint64_t workspace_bytes);

/* x[i] += sum_{s<k} partial[s*ne + i], summed in slot order
 * (moe_reduce_f32.comp:8-13 with the weights already applied).  With one
 * non-zero contributor per slot the cross-rank sum is exact, so the result
 * equals the single-device styx_moe_block bit for bit. */
int styx_moe_combine(styx_ctx *ctx, styx_stream stream, const float *partial,
                     float *x, int ne, int k);

/* The cross-rank sum and the combine over NVLink peer memory (no
 * counterpart in the reference: it replaces "all-reduce partial, then
 * styx_moe_combine" for the ranks of one node).  Each rank owns an inbox of
 * 2 x world x k x n_embd 8-byte words (two halves, by call parity) in its
 * own device memory; styx_ep_open allocates it and returns its CUDA IPC
 * handle (STYX_EP_HANDLE_BYTES), the caller gathers every rank's handle
 * (e.g. with torch.distributed) and passes them, in rank order, to
 * styx_ep_connect, which maps the peers'.
 *
 * styx_ep_combine (one kernel) sends each value of this rank's partial to
 * every peer's inbox over NVLink as one word tagged with the call's
 * generation (an 8-byte store is atomic, so a word with this call's tag
 * holds this call's value: no fence or flag), waits (bounded: STYX_ETIMEOUT
 * after about a second) for the peers' words of its columns in its own
 * inbox, and adds sum_s (sum_r partial_r[s][i]) into x[i], ranks then slots
 * in order: with one non-zero contributor per slot the result equals the
 * single-device block bit for bit, as the NCCL form does.
 *
 * styx_ep_moe_block is styx_moe_block_ep + styx_ep_combine in one call: x
 * ends as the single-device styx_moe_block leaves it, bit for bit.  Where
 * the single-kernel form fits (STYX_OPT_MOE_KERNELS 0 or 1) the exchange is
 * that kernel's epilogue -- each CTA pushes its own rows of every slot as
 * soon as they are computed, and adds the ranks' sum of the same rows into
 * x -- so the block and the exchange are one launch; otherwise the block's
 * partial goes through styx_ep_combine (workspace as for styx_moe_block_ep,
 * plus k x n_embd floats held by the styx_ep).
 *
 * Every rank must make the same calls on one styx_ep (either entry point,
 * once per layer) in the same order; calls on one styx_ep must not overlap
 * on the GPU (one stream).  The call's generation is a counter in the
 * rank's own memory (advanced by the call's last CTA), so a launch recorded
 * once can be replayed.  No multicast, no library collective, no load from
 * a peer's memory.  styx_ep_close synchronises the device, unmaps the peers
 * and frees the inbox: call it on every rank after a barrier. */
#define STYX_EP_HANDLE_BYTES 64
#define STYX_EP_MAX_RANKS 8
typedef struct styx_ep styx_ep;
int styx_ep_open(styx_ctx *ctx, int rank, int world, int k, int n_embd, styx_ep **out, void *handle);
int styx_ep_connect(styx_ep *ep, const void *handles);
int styx_ep_combine(styx_ctx *ctx, styx_ep *ep, styx_stream stream, const float *partial, float *x);
int styx_ep_moe_block(styx_ctx *ctx, styx_ep *ep, styx_stream stream, const styx_moe_dims *dims,
                      const styx_moe_layer *lw, int layer, float *x, int32_t *ids, float *weights_out,
                      void *workspace, uint64_t workspace_bytes);
int styx_ep_close(styx_ep *ep);

/* styx_moe_block without a caller workspace; it has no counterpart in the
 * reference.  For callers that cannot allocate device memory (a host that
 * binds only the compute entry points, or one whose whole device budget is
 * committed to expert tensors and arenas): the scratch is a static device
 * array of STYX_NOALLOC_SCRATCH_BYTES per device, and nothing is allocated.
 *   - Dims whose styx_moe_workspace_bytes exceeds that size are rejected
 *     (STYX_EINVAL).
 *   - The first call on a device looks up the array's device address; make
 *     it before any stream capture (it fails while the stream is capturing).
 *     The address is looked up again once every context on that device has
 *     been destroyed.
 *   - Every call first clears, on `stream`, all the words one call leaves for
 *     the next (launch and arrival counters, tagged logit and x words), so
 *     a call after one with other dims, or after one whose bounded wait ran
 *     out (STYX_ETIMEOUT), starts clean; no reset call is needed.
 *   - All calls on one device share the one scratch: calls that overlap (on
 *     different streams or host threads) race.  Serialise them.
 *   - styx_moe_workspace_view does not apply to it. */
#define STYX_NOALLOC_SCRATCH_BYTES (512u * 1024u)
int styx_moe_block_noalloc(styx_ctx *ctx, styx_stream stream,
                           const styx_moe_dims *dims,
                           const styx_moe_layer *layer_w, int layer, float *x,
                           int32_t *ids, float *weights_out);

/* Debug / test views of the last styx_moe_block's intermediates kept in the
 * workspace: which = 0 xnorm f32[H], 1 logits f32[E], 2 h f32[k*F],
 * 3 weights f32[k], 4 phase trace int64[CTAs][32] (STYX_OPT_TRACE).  Returns a
 * device pointer into the workspace. */
int styx_moe_workspace_view(const styx_moe_dims *dims, void *workspace,
                            int which, void **out);

/* ------------------------------------------------- synthetic weights
 * Device-side generator for benchmark-sized synthetic expert tensors:
 * values N(0, sigma) from a counter-based hash of (seed, index), quantised
 * per block with the same min/max scheme as the test oracle's quantiser.
 * Writes nrows rows of ncols elements of `qtype` to dst. */
int styx_synth_quant(styx_ctx *ctx, styx_stream stream, int qtype, void *dst,
                     uint64_t nrows, int ncols, uint64_t seed, float sigma);
/* Same values as float32 (for checks): dst f32[nrows*ncols]. */
int styx_synth_f32(styx_ctx *ctx, styx_stream stream, float *dst, uint64_t n,
                   uint64_t seed, uint64_t offset, float sigma);

#ifdef __cplusplus
}
#endif
#endif
