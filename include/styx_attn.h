/* styx_attn.h -- the attention half of a decode layer, C ABI.
 *
 * The part of MoeModel::forward_token (crates/model/src/moe.rs:1845-1972)
 * that runs before each layer's MoE block, as ops that mirror the
 * reference's dispatches plus one call for the whole sequence:
 *
 *   styx_mul_mat_vec       rec_matvec_b (moe.rs:1523-1551): y = W x, W a
 *                          quantised row-major matrix (ggml mul_mat_vec_<type>)
 *   styx_qk_norm_rope_kv   the per-head q/k RMSNorm (QkNorm::PerHead,
 *                          moe.rs:1880-1897), NEOX RoPE (rope_neox_f32 with
 *                          RopePush::neox, crates/vk-backend/src/ops.rs:413-445;
 *                          moe.rs:1914-1932) and the K / V cache rows at the
 *                          token's position (moe.rs:1933-1945), in one launch
 *   styx_rope_neox         the RoPE alone (the rope dispatch, n_tokens rows)
 *   styx_attn_decode       shaders/attn_decode_f32.comp (moe.rs:1946-1964)
 *   styx_add_f32           shaders/add_flat_f32.comp (rec_add, moe.rs:1972)
 *   styx_attn_block        all of the above for one layer: rms(attn_norm) ->
 *                          q, k, v -> norms, RoPE, cache rows -> attention ->
 *                          o -> x += o
 *
 * Layouts are the reference's: q f32[n_heads][head_dim], k and v
 * f32[n_kv_heads][head_dim], caches f32[n_ctx][kv_dim] row-major with
 * kv_dim = n_kv_heads * head_dim (V not transposed), q head h reads kv head
 * h / gqa.  Error codes and styx_last_error() as in styx_moe.h.
 */
#ifndef STYX_ATTN_H
#define STYX_ATTN_H

#include <stdint.h>

#include "styx_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* y[r] = sum_c deq(W)[r][c] * x[c] for r < nrows; W row-major, qtype
 * STYX_Q8_0 / Q4_K / Q5_K / Q6_K (ncols a multiple of 64 for q8_0, 256 for
 * the k-quants; q4_K / q5_K matrices 16-byte aligned, the others 2-byte).
 * The MoE kernels' dot products; the rows stream through shared memory by
 * bulk copies, x is converted once per CTA. */
int styx_mul_mat_vec(styx_ctx *ctx, styx_stream stream, int qtype, const void *a, int nrows, int ncols,
                     const float *x, float *y);

/* y[r] += sum_c deq(W)[r][c] * x[c]: the GEMV with the residual add fused
 * (rounds exactly as styx_mul_mat_vec into a temporary, then styx_add_f32). */
int styx_mul_mat_vec_add(styx_ctx *ctx, styx_stream stream, int qtype, const void *a, int nrows, int ncols,
                         const float *x, float *y);

/* d[i] = a[i] + b[i], i < n (d may alias a or b). */
int styx_add_f32(styx_ctx *ctx, styx_stream stream, const float *a, const float *b, float *d, int n);

/* For each of n_tokens tokens t (positions pos[t], device int32):
 *   q[t][h] (h < n_heads):  RMSNorm with q_norm (if not NULL), then RoPE;
 *   k[t][j] (j < n_kv):     RMSNorm with k_norm (if not NULL), then RoPE,
 *                           and written to kcache row pos[t] (if not NULL);
 *   v[t][j]:                copied to vcache row pos[t] (if not NULL).
 * q and k are updated in place.  RoPE is NEOX with full rotation
 * (n_dims = head_dim): pairs (i, i + head_dim/2), theta = pos *
 * freq_base^(-2i/head_dim).  head_dim even, <= 256.  Cache rows are
 * f32[kv_dim] with kv_dim = n_kv * head_dim, n_ctx of them; pos must be
 * < n_ctx (checked on the device: a row outside is skipped and reported
 * through styx_check_device_error as STYX_EINVAL). */
int styx_qk_norm_rope_kv(styx_ctx *ctx, styx_stream stream, float *q, float *k, const float *v,
                         const float *q_norm, const float *k_norm, float eps, int n_heads, int n_kv,
                         int head_dim, int n_tokens, float freq_base, const int32_t *pos, float *kcache,
                         float *vcache, int n_ctx);

/* rope_neox_f32 over x f32[n_tokens][n_heads][head_dim] in place (RopePush::
 * neox(head_dim, n_heads, n_tokens, freq_base); pos int32[n_tokens] on the
 * device). */
int styx_rope_neox(styx_ctx *ctx, styx_stream stream, float *x, int head_dim, int n_heads, int n_tokens,
                   float freq_base, const int32_t *pos);

/* Workspace bytes styx_attn_decode needs for n_heads heads of head_dim. */
int styx_attn_workspace_bytes(int n_heads, int head_dim, uint64_t *out);

/* attn_decode_f32 (push {n_t, hd, kv_dim, gqa, scale}, one workgroup per q
 * head): for q head h and kv head h / gqa,
 *   s[t] = scale * q[h] . K[t][kvh],  p = softmax(s over t < n_t),
 *   out[h] = sum_t p[t] V[t][kvh].
 * n_heads = gqa * (kv_dim / head_dim); head_dim a multiple of 4, <= 256; q,
 * caches and out 16-byte aligned.  The kernel splits the sequence over CTAs
 * (each reads a kv head's rows once for its gqa q heads) and merges the
 * splits' softmax statistics; the workspace holds the partials. */
int styx_attn_decode(styx_ctx *ctx, styx_stream stream, const float *q, const float *kcache,
                     const float *vcache, float *out, int n_t, int head_dim, int kv_dim, int gqa, float scale,
                     void *workspace, uint64_t workspace_bytes);

/* ------------------------------------------------- the ends of a token */
/* out[r] = deq(W)[rows[r]] for r < n: W row-major [nrows][ncols] of qtype
 * (STYX_Q8_0 / Q4_K / Q5_K / Q6_K), rows a device int32[n].  The token
 * embedding (the reference dequantises the q4_K row on the host,
 * moe.rs:1824-1835); values identical to a CPU decode of the blocks.  A row
 * index outside [0, nrows) gives zeros and STYX_EINVAL from
 * styx_check_device_error. */
int styx_get_rows(styx_ctx *ctx, styx_stream stream, int qtype, const void *w, int nrows, int ncols,
                  const int32_t *rows, int n, float *out);

/* *out = the index of the largest x[i] under IEEE total order, the last one
 * among equals: the greedy pick of generate_moe (examples/generate_moe.rs:29,
 * max_by(total_cmp) over the downloaded logits), on the device.  Uses a
 * scratch area of the context: calls on one context must not run at the same
 * time on different streams. */
int styx_argmax_f32(styx_ctx *ctx, styx_stream stream, const float *x, int n, int32_t *out);

/* ------------------------------------------------- one layer's attention */
typedef struct styx_dense_tensor {
    const void *data;          /* row-major [nrows][ncols] of qtype */
    int32_t qtype;
} styx_dense_tensor;

/* HParams (moe.rs:550-587) that the attention half reads. */
typedef struct styx_attn_dims {
    int32_t n_embd;            /* H */
    int32_t n_heads;
    int32_t n_kv_heads;
    int32_t head_dim;
    int32_t qk_norm;           /* 1: per-head q/k RMSNorm (QkNorm::PerHead), 0: none */
    float rms_eps;
    float rope_base;
} styx_attn_dims;

/* Layer weights of the attention half (Layer, moe.rs:108-144). */
typedef struct styx_attn_layer {
    const float *attn_norm;    /* f32[H] */
    styx_dense_tensor wq;      /* [n_heads*head_dim][H] */
    styx_dense_tensor wk;      /* [n_kv*head_dim][H] */
    styx_dense_tensor wv;      /* [n_kv*head_dim][H] */
    styx_dense_tensor wo;      /* [H][n_heads*head_dim] */
    const float *q_norm;       /* f32[head_dim] (qk_norm) */
    const float *k_norm;       /* f32[head_dim] (qk_norm) */
} styx_attn_layer;

/* Workspace bytes styx_attn_block needs, and its initialisation (zeroes;
 * once after allocation, and after a STYX_ETIMEOUT from
 * styx_check_device_error). */
int styx_attn_block_workspace_bytes(const styx_attn_dims *dims, uint64_t *out);
int styx_attn_block_workspace_init(styx_ctx *ctx, styx_stream stream, void *workspace, uint64_t workspace_bytes);

/* x += o(attention(rope(norm(q, k, v of rms_norm(x) * attn_norm)))) for the
 * token at position `pos` (n_t = pos + 1 cache rows are read; row pos is
 * written first).  pos_dev is the same position as a device int32 (the
 * reference's bpos buffer).  One cooperative kernel or one launch of
 * thread-block clusters (one cluster per kv head) when the shape fits
 * (head_dim 128, n_embd <= 2048, q/k/o of one format, STYX_OPT_ATTN_KERNELS;
 * both read the position from `pos`), else seven launches, stream-ordered
 * (the o GEMV adds into x).  The workspace keeps counters: initialise it
 * once with styx_attn_block_workspace_init. */
int styx_attn_block(styx_ctx *ctx, styx_stream stream, const styx_attn_dims *dims, const styx_attn_layer *lw,
                    float *x, int pos, const int32_t *pos_dev, float *kcache, float *vcache, int n_ctx,
                    void *workspace, uint64_t workspace_bytes);

#ifdef __cplusplus
}
#endif
#endif
