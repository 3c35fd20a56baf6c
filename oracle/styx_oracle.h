/*
 * styx_oracle.h -- CPU oracle for the Qwen3-MoE block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library.
 * The product (styx_b200, libstyx_moe.so) never links or calls it.
 *
 * Each function restates, in plain C, the arithmetic of one step of the
 * reference (aDirtyScoundrel/styx) in the reference's own order; the file and
 * line each one follows are cited beside it in styx_oracle.c.
 *
 * Parity pins:
 *   - q4_K / q5_K / q6_K / q8_0 block decoding is checked against golden
 *     vectors produced by llama.cpp's gguf-py 0.19.0 (tests/golden/).
 *   - topk_softmax / router GEMV / moe_reduce / gather_slabs are checked
 *     against the reference's own GLSL sources compiled as C++ through a shim
 *     (oracle/_ref, built by oracle/Makefile when the reference tree exists).
 */
#ifndef STYX_ORACLE_H
#define STYX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids as stored in GGUF (crates/model/src/moe.rs:24-40). */
enum { OR_F32 = 0, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14 };
#define OR_SKIP 0xFFFFFFFFu

/* elements / bytes per quant block (gguf-rs/src/lib.rs:287-294, moe.rs:1610-1618) */
int or_block_elems(int qtype);
int or_block_bytes(int qtype);
/* bytes of one row of `ncols` elements, 0 if ncols is not a block multiple */
size_t or_row_bytes(int qtype, int ncols);

float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f); /* round to nearest even */

/* one block -> out[or_block_elems(qtype)] */
void or_dequant_block(int qtype, const uint8_t *blk, float *out);
/* one row of ncols elements */
int or_dequant_row(int qtype, const uint8_t *row, int ncols, float *out);

/* Test-data quantizers (NOT a restatement of ggml's quantizers: a simple,
 * deterministic min/max scheme producing valid blocks of each format). */
int or_quantize_row(int qtype, const float *x, int ncols, uint8_t *out);
/* nrows rows at once (OpenMP over rows) */
int or_quantize_rows(int qtype, const float *x, long long nrows, int ncols, uint8_t *out);

/* y[r] = sum_c deq(W)[r][c] * x[c], column order, f32 (kernels.rs:380-392) */
void or_matvec_q(int qtype, const uint8_t *w, int nrows, int ncols,
                 const float *x, float *y);

/* Expert-indexed quant GEMV (kernels.rs:124-131, 183-198):
 *   y[s*nrows + r] = sum_c deq(W[ids[s]])[r][c] * x[(s % ne11)*ncols + c] */
void or_mul_mat_vec_id(int qtype, const uint8_t *w, size_t expert_bytes,
                       int nrows, int ncols, const int32_t *ids, int n_ids,
                       const float *x, int ne11, float *y);

/* RMSNorm with weight multiply (kernels.rs:58-67, moe.rs:1975-1982) */
void or_rms_norm(const float *x, const float *w, int n, float eps, float *out);

/* Router GEMV in the order of shaders/matvec_strided_f32.comp:20-35 */
void or_matvec_strided_f32(const float *a, int nrows, int ncols, int stride_a,
                           const float *x, float *d);

/* shaders/topk_softmax_f32.comp:29-67 (ids64 = the 64-int id block) */
void or_topk_softmax(const float *logits, int n, int k, int renorm,
                     const uint32_t *remap, const uint32_t *pmap,
                     float *weights, int32_t *ids64);

/* split swiglu: out = g / (1 + exp(-g)) * u  (ops2.rs:305-308) */
void or_swiglu(const float *g, const float *u, int n, float *out);

/* shaders/moe_reduce_f32.comp:8-13: x[i] += sum_s w[s] * d[s*ne + i] */
void or_moe_reduce(const float *d, const float *w, int ne, int k, float *x);

/* shaders/gather_slabs_f32.comp:40-85 (byte-exact copy, SKIP early-out).
 * slab strides are in bytes; arena slot = layer*k + s. */
void or_gather_slabs(const uint8_t *src_g, const uint8_t *src_u,
                     const uint8_t *src_d, uint64_t src_bg, uint64_t src_bu,
                     uint64_t src_bd, uint8_t *arena_g, uint8_t *arena_u,
                     uint8_t *arena_d, uint64_t dst_bg, uint64_t dst_bu,
                     uint64_t dst_bd, const int32_t *ids, int layer, int k);

/* The whole MoE block (moe.rs:1974-2062) with every expert in one tensor:
 *   xnorm = rms(x); logits = R.xnorm; topk; g,u = id-GEMV; h = swiglu;
 *   d = id-GEMV(down, h, ne11=k); x += sum_s w[s] d[s].
 * Optional outputs (may be NULL): xnorm[H], logits[E], weights[k], ids64[64],
 * h[k*F], d[k*H].  remap/pmap may be NULL (all SKIP). */
void or_moe_block(const float *ffn_norm, float eps, const float *router, int E,
                  int H, int F, int k, int renorm, int qt_gate, int qt_up,
                  int qt_down, const uint8_t *gate, const uint8_t *up,
                  const uint8_t *down, const uint32_t *remap,
                  const uint32_t *pmap, float *x, float *xnorm, float *logits,
                  float *weights, int32_t *ids64, float *h, float *d);

/* Threaded variant for CPU timing: the expert GEMVs split rows over
 * `nthreads` OpenMP threads (1 = the scalar oracle). */
void or_moe_block_mt(const float *ffn_norm, float eps, const float *router,
                     int E, int H, int F, int k, int renorm, int qt_gate,
                     int qt_up, int qt_down, const uint8_t *gate,
                     const uint8_t *up, const uint8_t *down, float *x,
                     int nthreads);

/* ---- the attention half of a decode layer (moe.rs:1845-1972) ---- */

/* rope_neox_f32 as crates/vk-backend/tests/ops2.rs:425-440 computes it on the
 * CPU: x f32[n_tokens][n_heads][head_dim] in place, pairs (i, i + hd/2),
 * theta = pos[t] * (freq_base^(-2/hd))^i, all in double. */
void or_rope_neox(float *x, int head_dim, int n_heads, int n_tokens,
                  float freq_base, const int32_t *pos);

/* shaders/attn_decode_f32.comp:29-75 for every q head: 128 invocations,
 * strided partial dots reduced by the shared tree s = 64..1, the online
 * softmax update per token, acc = acc*corr + pr*v, out = acc * (1/l). */
void or_attn_decode(const float *q, const float *kcache, const float *vcache,
                    float *out, int n_heads, int n_t, int hd, int kv_dim,
                    int gqa, float scale);

/* One layer's attention half (moe.rs:1857-1972) for the token at pos:
 * xn = rms(x)*attn_norm; q,k,v = W xn; per-head rms of q and k (when
 * q_norm); RoPE; K/V cache row pos; attention over pos+1 rows; x += Wo att. */
void or_attn_block(float *x, const float *attn_norm, float eps, int H,
                   int n_heads, int n_kv, int hd, int qk_norm,
                   const float *q_norm, const float *k_norm, float rope_base,
                   int qt_q, const uint8_t *wq, int qt_k, const uint8_t *wk,
                   int qt_v, const uint8_t *wv, int qt_o, const uint8_t *wo,
                   int pos, float *kcache, float *vcache);

#ifdef __cplusplus
}
#endif
#endif
