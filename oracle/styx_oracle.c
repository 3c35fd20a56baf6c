/*
 * styx_oracle.c -- CPU oracle for the Qwen3-MoE block hot path, and for the
 * attention half of a decode layer (or_rope_neox, or_attn_decode,
 * or_attn_block: moe.rs:1857-1972, shaders/attn_decode_f32.comp).
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU legs of bench.py as the checker; never by the product library.
 *
 * Restates the reference (aDirtyScoundrel/styx) in plain C, step by step and
 * in the reference's summation order.  Citations are paths inside the
 * reference project.  Built with -ffp-contract=off so that every `a*b + c`
 * rounds twice, like the Rust expressions it restates.
 *
 * Third-party formats: q5_K and q6_K have no CPU decoder in the reference
 * (their GPU kernels are ggml's, vendored and absent).  They are restated
 * from the published GGUF block layouts and pinned against llama.cpp's
 * gguf-py 0.19.0 `quants.dequantize` (tests/golden/quant_golden.npz).
 */
#include "styx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256

int or_block_elems(int qtype) {
    switch (qtype) {
    case OR_Q8_0: return 32;
    case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return QK_K;
    case OR_F32: return 1;
    default: return 0;
    }
}

int or_block_bytes(int qtype) {
    switch (qtype) {           /* gguf-rs/src/lib.rs:287-294 */
    case OR_Q8_0: return 34;
    case OR_Q4_K: return 144;
    case OR_Q5_K: return 176;
    case OR_Q6_K: return 210;
    case OR_F32: return 4;
    default: return 0;
    }
}

size_t or_row_bytes(int qtype, int ncols) {
    int be = or_block_elems(qtype);
    if (be <= 0 || ncols % be) return 0;
    return (size_t)(ncols / be) * (size_t)or_block_bytes(qtype);
}

/* IEEE binary16 -> binary32, exact (the `half` 2.7.1 widening used at
 * crates/model/src/moe.rs:508). */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {               /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = mant >> 13;
    uint32_t rem = mant & 0x1FFFu;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)h;
}

static float rd_f16(const uint8_t *p) {
    return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

/* q8_0: {f16 d; i8 q[32]}; value = d * q
 * (crates/model/src/lib.rs:103-113, crates/vk-backend/tests/ops2.rs:105-110) */
static void deq_q8_0(const uint8_t *b, float *out) {
    float d = rd_f16(b);
    for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)b[2 + i];
}

/* q4_K 6-bit scale/min unpacking (crates/model/src/moe.rs:512-521) */
static void get_scale_min(const uint8_t *s, int j, float *sc, float *m) {
    if (j < 4) {
        *sc = (float)(s[j] & 63);
        *m = (float)(s[j + 4] & 63);
    } else {
        *sc = (float)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* q4_K: {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}
 * value = d*sc*q - dmin*m, 64-element groups, low nibbles then high nibbles
 * (crates/model/src/moe.rs:506-533 == crates/vk-backend/tests/kernels.rs:295-333) */
static void deq_q4_K(const uint8_t *b, float *out) {
    float d = rd_f16(b), dmin = rd_f16(b + 2);
    const uint8_t *scales = b + 4, *qs = b + 16;
    int ql = 0, o = 0;
    for (int j = 0; j < QK_K / 64; j++) {
        float sc1, m1, sc2, m2;
        get_scale_min(scales, 2 * j, &sc1, &m1);
        get_scale_min(scales, 2 * j + 1, &sc2, &m2);
        for (int l = 0; l < 32; l++) {
            out[o + l] = d * sc1 * (float)(qs[ql + l] & 0x0F) - dmin * m1;
            out[o + 32 + l] = d * sc2 * (float)(qs[ql + l] >> 4) - dmin * m2;
        }
        o += 64;
        ql += 32;
    }
}

/* q5_K: {f16 d; f16 dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]}
 * As q4_K with a fifth bit: element 64j+l takes bit 2j of qh[l], element
 * 64j+32+l takes bit 2j+1.  Published GGUF layout (ggml block_q5_K). */
static void deq_q5_K(const uint8_t *b, float *out) {
    float d = rd_f16(b), dmin = rd_f16(b + 2);
    const uint8_t *scales = b + 4, *qh = b + 16, *qs = b + 48;
    for (int j = 0; j < QK_K / 64; j++) {
        float sc1, m1, sc2, m2;
        get_scale_min(scales, 2 * j, &sc1, &m1);
        get_scale_min(scales, 2 * j + 1, &sc2, &m2);
        for (int l = 0; l < 32; l++) {
            int q1 = (qs[32 * j + l] & 0x0F) + (((qh[l] >> (2 * j)) & 1) << 4);
            int q2 = (qs[32 * j + l] >> 4) + (((qh[l] >> (2 * j + 1)) & 1) << 4);
            out[64 * j + l] = d * sc1 * (float)q1 - dmin * m1;
            out[64 * j + 32 + l] = d * sc2 * (float)q2 - dmin * m2;
        }
    }
}

/* q6_K: {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d}
 * Two 128-element halves n; for l < 32 the four elements 128n+l+32q take
 * 4 low bits from ql (q=0,1 low nibbles of ql[64n+l], ql[64n+32+l]; q=2,3 the
 * high nibbles) and 2 high bits from qh[32n+l] bits 2q..2q+1; value =
 * d*scale[8n + l/16 + 2q]*(q6 - 32).  Published GGUF layout (ggml block_q6_K). */
static void deq_q6_K(const uint8_t *b, float *out) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = rd_f16(b + 208);
    for (int n = 0; n < 2; n++) {
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            uint8_t h = qh[32 * n + l];
            int q1 = ((ql[64 * n + l] & 0x0F) | (((h >> 0) & 3) << 4)) - 32;
            int q2 = ((ql[64 * n + l + 32] & 0x0F) | (((h >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[64 * n + l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[64 * n + l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
            out[128 * n + l] = d * (float)sc[8 * n + is + 0] * (float)q1;
            out[128 * n + l + 32] = d * (float)sc[8 * n + is + 2] * (float)q2;
            out[128 * n + l + 64] = d * (float)sc[8 * n + is + 4] * (float)q3;
            out[128 * n + l + 96] = d * (float)sc[8 * n + is + 6] * (float)q4;
        }
    }
}

void or_dequant_block(int qtype, const uint8_t *blk, float *out) {
    switch (qtype) {
    case OR_Q8_0: deq_q8_0(blk, out); break;
    case OR_Q4_K: deq_q4_K(blk, out); break;
    case OR_Q5_K: deq_q5_K(blk, out); break;
    case OR_Q6_K: deq_q6_K(blk, out); break;
    case OR_F32: memcpy(out, blk, 4); break;
    default: break;
    }
}

int or_dequant_row(int qtype, const uint8_t *row, int ncols, float *out) {
    int be = or_block_elems(qtype), bb = or_block_bytes(qtype);
    if (be <= 0 || ncols % be) return -1;
    for (int b = 0; b < ncols / be; b++)
        or_dequant_block(qtype, row + (size_t)b * bb, out + (size_t)b * be);
    return 0;
}

/* ---------------------------------------------------------------- quantizers
 * Test-data generation only.  Simple per-sub-block min/max quantizers that
 * emit well-formed blocks; round-to-nearest-even everywhere so that a GPU
 * implementation can reproduce the bytes exactly. */
static float fmaxabs(const float *x, int n) {
    float m = 0.f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > m) m = a;
    }
    return m;
}

static void q_q8_0(const float *x, uint8_t *b) {
    float amax = fmaxabs(x, 32);
    float d = amax / 127.f;
    uint16_t dh = or_f32_to_f16(d);
    float df = or_f16_to_f32(dh);
    b[0] = (uint8_t)(dh & 0xFF);
    b[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; i++) {
        int q = df > 0.f ? (int)rintf(x[i] / df) : 0;
        if (q > 127) q = 127;
        if (q < -127) q = -127;
        b[2 + i] = (uint8_t)(int8_t)q;
    }
}

/* shared by q4_K (nmax 15) and q5_K (nmax 31): per 32-element sub-block
 * scale = (max - min)/nmax, offset = -min (min clamped to <= 0); 6-bit
 * super-block quantisation of both against d = max/63, dmin = max/63. */
static void kq_scales(const float *x, int nmax, uint8_t sc[8], uint8_t mn[8],
                      uint16_t *dh, uint16_t *dmh, float *df, float *dmf) {
    float scf[8], mf[8], smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; j++) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; i++) {
            float v = x[32 * j + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.f) lo = 0.f;
        scf[j] = (hi - lo) / (float)nmax;
        mf[j] = -lo;
        if (scf[j] > smax) smax = scf[j];
        if (mf[j] > mmax) mmax = mf[j];
    }
    *dh = or_f32_to_f16(smax / 63.f);
    *dmh = or_f32_to_f16(mmax / 63.f);
    *df = or_f16_to_f32(*dh);
    *dmf = or_f16_to_f32(*dmh);
    for (int j = 0; j < 8; j++) {
        int s = *df > 0.f ? (int)rintf(scf[j] / *df) : 0;
        int m = *dmf > 0.f ? (int)rintf(mf[j] / *dmf) : 0;
        sc[j] = (uint8_t)(s < 0 ? 0 : s > 63 ? 63 : s);
        mn[j] = (uint8_t)(m < 0 ? 0 : m > 63 ? 63 : m);
    }
}

/* inverse of get_scale_min (moe.rs:512-521) */
static void kq_pack_scales(const uint8_t sc[8], const uint8_t mn[8], uint8_t *s) {
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((mn[j + 4] & 0x0F) << 4));
    }
}

static int kq_level(float v, float dsc, float off, int nmax) {
    if (!(dsc > 0.f)) return 0;
    int q = (int)rintf((v + off) / dsc);
    return q < 0 ? 0 : q > nmax ? nmax : q;
}

static void q_q4_K(const float *x, uint8_t *b) {
    uint8_t sc[8], mn[8];
    uint16_t dh, dmh;
    float d, dmin;
    kq_scales(x, 15, sc, mn, &dh, &dmh, &d, &dmin);
    b[0] = (uint8_t)(dh & 0xFF); b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)(dmh & 0xFF); b[3] = (uint8_t)(dmh >> 8);
    kq_pack_scales(sc, mn, b + 4);
    uint8_t *qs = b + 16;
    for (int j = 0; j < 4; j++) {
        int s1 = 2 * j, s2 = 2 * j + 1;
        float ds1 = d * (float)sc[s1], o1 = dmin * (float)mn[s1];
        float ds2 = d * (float)sc[s2], o2 = dmin * (float)mn[s2];
        for (int l = 0; l < 32; l++) {
            int lo = kq_level(x[64 * j + l], ds1, o1, 15);
            int hi = kq_level(x[64 * j + 32 + l], ds2, o2, 15);
            qs[32 * j + l] = (uint8_t)(lo | (hi << 4));
        }
    }
}

static void q_q5_K(const float *x, uint8_t *b) {
    uint8_t sc[8], mn[8];
    uint16_t dh, dmh;
    float d, dmin;
    kq_scales(x, 31, sc, mn, &dh, &dmh, &d, &dmin);
    b[0] = (uint8_t)(dh & 0xFF); b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)(dmh & 0xFF); b[3] = (uint8_t)(dmh >> 8);
    kq_pack_scales(sc, mn, b + 4);
    uint8_t *qh = b + 16, *qs = b + 48;
    memset(qh, 0, 32);
    for (int j = 0; j < 4; j++) {
        int s1 = 2 * j, s2 = 2 * j + 1;
        float ds1 = d * (float)sc[s1], o1 = dmin * (float)mn[s1];
        float ds2 = d * (float)sc[s2], o2 = dmin * (float)mn[s2];
        for (int l = 0; l < 32; l++) {
            int lo = kq_level(x[64 * j + l], ds1, o1, 31);
            int hi = kq_level(x[64 * j + 32 + l], ds2, o2, 31);
            qs[32 * j + l] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            qh[l] |= (uint8_t)(((lo >> 4) & 1) << (2 * j));
            qh[l] |= (uint8_t)(((hi >> 4) & 1) << (2 * j + 1));
        }
    }
}

static void q_q6_K(const float *x, uint8_t *b) {
    float scf[16], smax = 0.f;
    for (int s = 0; s < 16; s++) {
        scf[s] = fmaxabs(x + 16 * s, 16) / 31.f;
        if (scf[s] > smax) smax = scf[s];
    }
    uint16_t dh = or_f32_to_f16(smax / 127.f);
    float d = or_f16_to_f32(dh);
    int8_t sc[16];
    for (int s = 0; s < 16; s++) {
        int v = d > 0.f ? (int)rintf(scf[s] / d) : 0;
        sc[s] = (int8_t)(v < 0 ? 0 : v > 127 ? 127 : v);
    }
    uint8_t q[QK_K];
    for (int i = 0; i < QK_K; i++) {
        float ds = d * (float)sc[i / 16];
        int v = ds > 0.f ? (int)rintf(x[i] / ds) : 0;
        v = v < -32 ? -32 : v > 31 ? 31 : v;
        q[i] = (uint8_t)(v + 32);
    }
    uint8_t *ql = b, *qh = b + 128;
    for (int n = 0; n < 2; n++) {
        for (int l = 0; l < 32; l++) {
            uint8_t q1 = q[128 * n + l], q2 = q[128 * n + 32 + l];
            uint8_t q3 = q[128 * n + 64 + l], q4 = q[128 * n + 96 + l];
            ql[64 * n + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * n + 32 + l] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) |
                                       ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    memcpy(b + 192, sc, 16);
    b[208] = (uint8_t)(dh & 0xFF);
    b[209] = (uint8_t)(dh >> 8);
}

int or_quantize_row(int qtype, const float *x, int ncols, uint8_t *out) {
    int be = or_block_elems(qtype), bb = or_block_bytes(qtype);
    if (be <= 1 || ncols % be) return -1;
    for (int b = 0; b < ncols / be; b++) {
        const float *xb = x + (size_t)b * be;
        uint8_t *ob = out + (size_t)b * bb;
        switch (qtype) {
        case OR_Q8_0: q_q8_0(xb, ob); break;
        case OR_Q4_K: q_q4_K(xb, ob); break;
        case OR_Q5_K: q_q5_K(xb, ob); break;
        case OR_Q6_K: q_q6_K(xb, ob); break;
        default: return -1;
        }
    }
    return 0;
}

int or_quantize_rows(int qtype, const float *x, long long nrows, int ncols, uint8_t *out) {
    size_t rb = or_row_bytes(qtype, ncols);
    if (rb == 0) return -1;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long long r = 0; r < nrows; r++)
        bad |= or_quantize_row(qtype, x + (size_t)r * ncols, ncols, out + (size_t)r * rb) != 0;
    return bad ? -1 : 0;
}

/* ----------------------------------------------------------------- GEMVs */

/* one row: dequantise, then a column-order f32 dot, products rounded before
 * the add (kernels.rs:187-196: row_f.iter().zip(&x).map(|(w,v)| w*v).sum()) */
static float row_dot(int qtype, const uint8_t *row, int ncols, const float *x,
                     float *scratch) {
    or_dequant_row(qtype, row, ncols, scratch);
    float s = 0.f;
    for (int c = 0; c < ncols; c++) s += scratch[c] * x[c];
    return s;
}

void or_matvec_q(int qtype, const uint8_t *w, int nrows, int ncols,
                 const float *x, float *y) {
    size_t rb = or_row_bytes(qtype, ncols);
    float tmp[16384];
    if (ncols > 16384 || rb == 0) return;
    for (int r = 0; r < nrows; r++) y[r] = row_dot(qtype, w + (size_t)r * rb, ncols, x, tmp);
}

/* get_offsets() semantics documented at kernels.rs:124-131: expert =
 * ids[slot], a at expert*expert_bytes, x row = slot % ne11, y row = slot.
 * SKIP (-1) ids early-out and leave y untouched, like the patched kernels
 * (topk_softmax_f32.comp:16-18). */
void or_mul_mat_vec_id(int qtype, const uint8_t *w, size_t expert_bytes,
                       int nrows, int ncols, const int32_t *ids, int n_ids,
                       const float *x, int ne11, float *y) {
    size_t rb = or_row_bytes(qtype, ncols);
    float tmp[16384];
    if (ncols > 16384 || rb == 0) return;
    for (int s = 0; s < n_ids; s++) {
        if ((uint32_t)ids[s] == OR_SKIP) continue;
        const uint8_t *a = w + (size_t)ids[s] * expert_bytes;
        const float *xs = x + (size_t)(s % ne11) * ncols;
        for (int r = 0; r < nrows; r++)
            y[(size_t)s * nrows + r] = row_dot(qtype, a + (size_t)r * rb, ncols, xs, tmp);
    }
}

/* kernels.rs:60-66 (mean of squares, 1/sqrt(mean+eps)) with the ffn_norm
 * weight multiply that moe.rs:1975-1982 enables on rms_norm_f32. */
void or_rms_norm(const float *x, const float *w, int n, float eps, float *out) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float mean = ss / (float)n;
    float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * (w ? w[i] : 1.0f);
}

/* shaders/matvec_strided_f32.comp:20-35: 32 invocations; invocation t sums
 * columns t, t+32, ...; then a shared-memory tree s = 16, 8, 4, 2, 1. */
void or_matvec_strided_f32(const float *a, int nrows, int ncols, int stride_a,
                           const float *x, float *d) {
    for (int row = 0; row < nrows; row++) {
        float tmp[32];
        const float *ar = a + (size_t)row * stride_a;
        for (int t = 0; t < 32; t++) {
            float sum = 0.f;
            for (int c = t; c < ncols; c += 32) sum += ar[c] * x[c];
            tmp[t] = sum;
        }
        for (int s = 16; s > 0; s >>= 1)
            for (int t = 0; t < s; t++) tmp[t] += tmp[t + s];
        d[row] = tmp[0];
    }
}

/* GLSL max(x, y) = (x < y) ? y : x */
static float glsl_max(float x, float y) { return (x < y) ? y : x; }

/* shaders/topk_softmax_f32.comp:29-67, serial as written: softmax
 * normaliser over all n; k rounds picking the first untaken index with a
 * strictly greater raw logit (start -inf, so ties go to the lowest index and
 * -inf/NaN logits are never picked); weights optionally renormalised; ids
 * written in selection order into the four 16-wide rows of ids64. */
void or_topk_softmax(const float *logits, int n, int k, int renorm,
                     const uint32_t *remap, const uint32_t *pmap,
                     float *weights, int32_t *ids64) {
    float mx = logits[0];
    for (int i = 1; i < n; i++) mx = glsl_max(mx, logits[i]);
    float sum = 0.f;
    for (int i = 0; i < n; i++) sum += expf(logits[i] - mx);
    float picked[16];
    int pid[16];
    float wsum = 0.f;
    for (int s = 0; s < k; s++) {
        float best = -INFINITY;
        int bi = -1;
        for (int i = 0; i < n; i++) {
            int taken = 0;
            for (int t = 0; t < s; t++)
                if (pid[t] == i) taken = 1;
            if (!taken && logits[i] > best) {
                best = logits[i];
                bi = i;
            }
        }
        float w = expf(best - mx) / sum;
        picked[s] = w;
        pid[s] = bi;
        wsum += w;
    }
    for (int s = 0; s < k; s++) {
        weights[s] = renorm ? picked[s] / wsum : picked[s];
        uint32_t e = (uint32_t)pid[s];
        ids64[s] = pid[s];
        /* pid < 0 only when every untaken logit is -inf/NaN; the shader would
         * then index remap out of bounds.  Defined here as all-SKIP. */
        uint32_t h = (pid[s] >= 0 && remap) ? remap[e] : OR_SKIP;
        if (h != OR_SKIP) {
            ids64[16 + s] = (int32_t)h;
            ids64[32 + s] = (int32_t)OR_SKIP;
            ids64[48 + s] = (int32_t)OR_SKIP;
        } else {
            uint32_t a = (pid[s] >= 0 && pmap) ? pmap[e] : OR_SKIP;
            ids64[16 + s] = (int32_t)OR_SKIP;
            ids64[32 + s] = (a != OR_SKIP) ? (int32_t)a : (int32_t)OR_SKIP;
            ids64[48 + s] = (a != OR_SKIP) ? (int32_t)OR_SKIP : pid[s];
        }
    }
}

void or_swiglu(const float *g, const float *u, int n, float *out) {
    for (int i = 0; i < n; i++) out[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

void or_moe_reduce(const float *d, const float *w, int ne, int k, float *x) {
    for (int i = 0; i < ne; i++) {
        float acc = 0.f;
        for (int s = 0; s < k; s++) acc += w[s] * d[(size_t)s * ne + i];
        x[i] += acc;
    }
}

void or_gather_slabs(const uint8_t *src_g, const uint8_t *src_u,
                     const uint8_t *src_d, uint64_t src_bg, uint64_t src_bu,
                     uint64_t src_bd, uint8_t *arena_g, uint8_t *arena_u,
                     uint8_t *arena_d, uint64_t dst_bg, uint64_t dst_bu,
                     uint64_t dst_bd, const int32_t *ids, int layer, int k) {
    for (int s = 0; s < k; s++) {
        uint32_t e = (uint32_t)ids[s];
        if (e == OR_SKIP) continue;
        uint64_t slot = (uint64_t)layer * (uint64_t)k + (uint64_t)s;
        memcpy(arena_g + slot * dst_bg, src_g + e * src_bg, src_bg);
        memcpy(arena_u + slot * dst_bu, src_u + e * src_bu, src_bu);
        memcpy(arena_d + slot * dst_bd, src_d + e * src_bd, src_bd);
    }
}

/* ------------------------------------------------------------ MoE block */

static void moe_block_impl(const float *ffn_norm, float eps, const float *router,
                           int E, int H, int F, int k, int renorm, int qt_gate,
                           int qt_up, int qt_down, const uint8_t *gate,
                           const uint8_t *up, const uint8_t *down,
                           const uint32_t *remap, const uint32_t *pmap, float *x,
                           float *xnorm_o, float *logits_o, float *weights_o,
                           int32_t *ids_o, float *h_o, float *d_o, int nthreads) {
    static float xnorm[16384], logits[512], weights[16], g[16 * 8192],
        u[16 * 8192], hbuf[16 * 8192], dbuf[16 * 16384];
    int32_t ids64[64];
    if (H > 16384 || E > 512 || k > 16 || F > 8192) return;
    or_rms_norm(x, ffn_norm, H, eps, xnorm);
    or_matvec_strided_f32(router, E, H, H, xnorm, logits);
    or_topk_softmax(logits, E, k, renorm, remap, pmap, weights, ids64);
    size_t gb = or_row_bytes(qt_gate, H) * (size_t)F;
    size_t ub = or_row_bytes(qt_up, H) * (size_t)F;
    size_t db = or_row_bytes(qt_down, F) * (size_t)H;
    size_t grb = or_row_bytes(qt_gate, H), urb = or_row_bytes(qt_up, H);
    size_t drb = or_row_bytes(qt_down, F);
    (void)nthreads;
    /* gate/up (ne11 = 1) */
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
    for (int t = 0; t < k * F; t++) {
        float tmp[16384];
        int s = t / F, r = t % F;
        if (ids64[s] < 0) { g[t] = 0.f; u[t] = 0.f; continue; }
        const uint8_t *ga = gate + (size_t)ids64[s] * gb + (size_t)r * grb;
        const uint8_t *ua = up + (size_t)ids64[s] * ub + (size_t)r * urb;
        g[t] = row_dot(qt_gate, ga, H, xnorm, tmp);
        u[t] = row_dot(qt_up, ua, H, xnorm, tmp);
    }
    or_swiglu(g, u, k * F, hbuf);
    /* down (ne11 = k: slot s reads h row s) */
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
    for (int t = 0; t < k * H; t++) {
        float tmp[16384];
        int s = t / H, r = t % H;
        if (ids64[s] < 0) { dbuf[t] = 0.f; continue; }
        const uint8_t *da = down + (size_t)ids64[s] * db + (size_t)r * drb;
        dbuf[t] = row_dot(qt_down, da, F, hbuf + (size_t)s * F, tmp);
    }
    if (xnorm_o) memcpy(xnorm_o, xnorm, sizeof(float) * H);
    if (logits_o) memcpy(logits_o, logits, sizeof(float) * E);
    if (weights_o) memcpy(weights_o, weights, sizeof(float) * k);
    if (ids_o) memcpy(ids_o, ids64, sizeof(ids64));
    if (h_o) memcpy(h_o, hbuf, sizeof(float) * k * F);
    if (d_o) memcpy(d_o, dbuf, sizeof(float) * k * H);
    or_moe_reduce(dbuf, weights, H, k, x);
}

void or_moe_block(const float *ffn_norm, float eps, const float *router, int E,
                  int H, int F, int k, int renorm, int qt_gate, int qt_up,
                  int qt_down, const uint8_t *gate, const uint8_t *up,
                  const uint8_t *down, const uint32_t *remap,
                  const uint32_t *pmap, float *x, float *xnorm, float *logits,
                  float *weights, int32_t *ids64, float *h, float *d) {
    moe_block_impl(ffn_norm, eps, router, E, H, F, k, renorm, qt_gate, qt_up,
                   qt_down, gate, up, down, remap, pmap, x, xnorm, logits,
                   weights, ids64, h, d, 1);
}

void or_moe_block_mt(const float *ffn_norm, float eps, const float *router,
                     int E, int H, int F, int k, int renorm, int qt_gate,
                     int qt_up, int qt_down, const uint8_t *gate,
                     const uint8_t *up, const uint8_t *down, float *x,
                     int nthreads) {
    moe_block_impl(ffn_norm, eps, router, E, H, F, k, renorm, qt_gate, qt_up,
                   qt_down, gate, up, down, NULL, NULL, x, NULL, NULL, NULL,
                   NULL, NULL, NULL, nthreads < 1 ? 1 : nthreads);
}

/* ------------------------------------------------------------------ attention half */

void or_rope_neox(float *x, int head_dim, int n_heads, int n_tokens,
                  float freq_base, const int32_t *pos) {
    const int half = head_dim / 2;
    const double theta_scale = pow((double)freq_base, -2.0 / (double)head_dim);
    for (int t = 0; t < n_tokens; t++)
        for (int h = 0; h < n_heads; h++) {
            float *b = x + ((size_t)t * n_heads + h) * head_dim;
            for (int i = 0; i < half; i++) {
                const double theta = (double)pos[t] * pow(theta_scale, (double)i);
                const double s = sin(theta), c = cos(theta);
                const double x0 = b[i], x1 = b[i + half];
                b[i] = (float)(x0 * c - x1 * s);
                b[i + half] = (float)(x0 * s + x1 * c);
            }
        }
}

void or_attn_decode(const float *q, const float *kcache, const float *vcache,
                    float *out, int n_heads, int n_t, int hd, int kv_dim,
                    int gqa, float scale) {
    float acc0[128], acc1[128], red[128];
    for (int h = 0; h < n_heads; h++) {
        const int kvoff = (h / gqa) * hd, qbase = h * hd;
        for (int tid = 0; tid < 128; tid++) acc0[tid] = acc1[tid] = 0.f;
        float m = -INFINITY, l = 0.f;
        for (int t = 0; t < n_t; t++) {
            const float *kr = kcache + (size_t)t * kv_dim + kvoff;
            for (int tid = 0; tid < 128; tid++) {
                float part = 0.f;
                for (int i = tid; i < hd; i += 128) part += q[qbase + i] * kr[i];
                red[tid] = part;
            }
            for (int s = 64; s > 0; s >>= 1)
                for (int tid = 0; tid < s; tid++) red[tid] += red[tid + s];
            const float sc = red[0] * scale;
            const float m_new = glsl_max(m, sc);
            const float corr = expf(m - m_new);
            const float pr = expf(sc - m_new);
            l = l * corr + pr;
            m = m_new;
            const float *vr = vcache + (size_t)t * kv_dim + kvoff;
            for (int tid = 0; tid < 128; tid++) {
                if (tid < hd) acc0[tid] = acc0[tid] * corr + pr * vr[tid];
                if (tid + 128 < hd) acc1[tid] = acc1[tid] * corr + pr * vr[tid + 128];
            }
        }
        /* 1.0 / l: a float division in GLSL (double-then-float rounds the same) */
        const float inv_l = 1.0f / l;
        for (int tid = 0; tid < 128; tid++) {
            if (tid < hd) out[qbase + tid] = acc0[tid] * inv_l;
            if (tid + 128 < hd) out[qbase + tid + 128] = acc1[tid] * inv_l;
        }
    }
}

void or_attn_block(float *x, const float *attn_norm, float eps, int H,
                   int n_heads, int n_kv, int hd, int qk_norm,
                   const float *q_norm, const float *k_norm, float rope_base,
                   int qt_q, const uint8_t *wq, int qt_k, const uint8_t *wk,
                   int qt_v, const uint8_t *wv, int qt_o, const uint8_t *wo,
                   int pos, float *kcache, float *vcache) {
    const int qd = n_heads * hd, kvd = n_kv * hd;
    float *xn = (float *)malloc(sizeof(float) * (size_t)(H + 2 * qd + 2 * kvd + H));
    float *q = xn + H, *k = q + qd, *v = k + kvd, *att = v + kvd, *proj = att + qd;
    or_rms_norm(x, attn_norm, H, eps, xn);                       /* moe.rs:1857-1864 */
    or_matvec_q(qt_q, wq, qd, H, xn, q);                         /* :1865-1885 */
    or_matvec_q(qt_k, wk, kvd, H, xn, k);
    or_matvec_q(qt_v, wv, kvd, H, xn, v);
    if (qk_norm) {                                               /* :1886-1897 */
        for (int h = 0; h < n_heads; h++) or_rms_norm(q + h * hd, q_norm, hd, eps, q + h * hd);
        for (int h = 0; h < n_kv; h++) or_rms_norm(k + h * hd, k_norm, hd, eps, k + h * hd);
    }
    const int32_t p32 = pos;
    or_rope_neox(q, hd, n_heads, 1, rope_base, &p32);            /* :1914-1932 */
    or_rope_neox(k, hd, n_kv, 1, rope_base, &p32);
    memcpy(kcache + (size_t)pos * kvd, k, sizeof(float) * (size_t)kvd);   /* :1933-1945 */
    memcpy(vcache + (size_t)pos * kvd, v, sizeof(float) * (size_t)kvd);
    or_attn_decode(q, kcache, vcache, att, n_heads, pos + 1, hd, kvd, n_heads / n_kv,
                   1.0f / sqrtf((float)hd));                     /* :1946-1964 */
    or_matvec_q(qt_o, wo, H, qd, att, proj);                     /* :1965-1971 */
    for (int i = 0; i < H; i++) x[i] = x[i] + proj[i];          /* :1972 */
    free(xn);
}
