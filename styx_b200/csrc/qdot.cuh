// qdot.cuh -- in-register GGUF block decoding and dot products on dp4a.
//
// A row of a quantised matrix is split into 64-element "units"; one lane
// owns one unit and keeps that unit's activation digits (common.cuh) in
// registers for every row it visits, so the inner loop is: load packed
// codes, mask them into byte lanes, three dp4a per 4 codes.  Per-sub-block
// scales are applied once to the integer sums:
//   sum_i w_i * x_i = d*sc * s * (I1 + I2/256 + I3/65536) - dmin*m * sum_i x_i
// where I_k = sum_i q_i * D_k[i] are exact integer dot products.
//
// Unit layouts (e = element index within the row):
//   q4_K / q5_K : unit u = (block b = u/4, group j = u%4), e = 64u .. 64u+63
//                 (qs bytes 32j..32j+31: low nibbles e = 64u+l, high nibbles
//                  e = 64u+32+l; crates/model/src/moe.rs:506-533)
//   q6_K        : unit u = (b = u/4, half n = (u/2)%2, t = u%2); l in
//                 [16t, 16t+16); the four elements 256b+128n+32q+l, q < 4
//   q8_0        : unit u = blocks 2u, 2u+1, e = 64u .. 64u+63
// Quarter q (16 elements, 4 words per digit plane) of a unit always lies in
// one 32-element activation group.
#pragma once

#include "common.cuh"

namespace styx {

struct XUnit {
    uint32_t d1[16], d2[16], d3[16];
    float s[4];    // group scale of each quarter
    float xs[4];   // sum of the represented activations over each quarter
};

__host__ __device__ constexpr int block_elems(int qt) {
    return qt == STYX_Q8_0 ? 32 : 256;
}
__host__ __device__ constexpr int block_bytes(int qt) {
    return qt == STYX_Q8_0 ? 34 : qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : qt == STYX_Q6_K ? 210 : 0;
}

// element offset of quarter q of unit u
template <int QT>
__device__ __forceinline__ int quarter_base(int u, int q) {
    if constexpr (QT == STYX_Q6_K) {
        return 256 * (u >> 2) + 128 * ((u >> 1) & 1) + 32 * q + 16 * (u & 1);
    } else {
        return 64 * u + 16 * q;
    }
}

// activation digits of unit u (from global or shared memory)
template <int QT>
__device__ __forceinline__ void load_xunit(XUnit &x, const int8_t *d1, const uint8_t *d2,
                                           const uint8_t *d3, const float *scale, int u) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int e = quarter_base<QT>(u, q);
        const uint4 a = *reinterpret_cast<const uint4 *>(d1 + e);
        const uint4 b = *reinterpret_cast<const uint4 *>(d2 + e);
        const uint4 c = *reinterpret_cast<const uint4 *>(d3 + e);
        x.d1[4 * q + 0] = a.x; x.d1[4 * q + 1] = a.y; x.d1[4 * q + 2] = a.z; x.d1[4 * q + 3] = a.w;
        x.d2[4 * q + 0] = b.x; x.d2[4 * q + 1] = b.y; x.d2[4 * q + 2] = b.z; x.d2[4 * q + 3] = b.w;
        x.d3[4 * q + 0] = c.x; x.d3[4 * q + 1] = c.y; x.d3[4 * q + 2] = c.z; x.d3[4 * q + 3] = c.w;
        int s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            s1 = dp4a_ss(x.d1[4 * q + i], 0x01010101u, s1);
            s2 = dp4a_uu(x.d2[4 * q + i], 0x01010101u, s2);
            s3 = dp4a_uu(x.d3[4 * q + i], 0x01010101u, s3);
        }
        const float s = scale[e >> 5];
        x.s[q] = s;
        x.xs[q] = s * (static_cast<float>(s1) +
                       (static_cast<float>(s2) + static_cast<float>(s3) * (1.f / 256.f)) * (1.f / 256.f));
    }
}

// I1 + I2/256 + I3/65536 with two conversions: I2*256 + I3 stays below 2^31
// for every code range used here (|I2| <= 32*255*255)
__device__ __forceinline__ float digits_to_f(int i1, int i2, int i3) {
    return static_cast<float>(i1) + static_cast<float>(i2 * 256 + i3) * (1.f / 65536.f);
}

// signed byte i of w as an exact float (bias the byte by 128, as byte_to_f)
__device__ __forceinline__ float sbyte_to_f(uint32_t w_xor80, uint32_t i) {
    return __uint_as_float(__byte_perm(w_xor80, 0x4B000000u, 0x7650u | i)) - 8388736.f;
}

// The 6-bit scales (sc) and mins (m) of four sub-blocks at once, one per
// byte: sub-blocks 0-3 (hi4 = false) or 4-7 (hi4 = true), from the 12 scale
// bytes in s0 (bytes 0-3), s1 (4-7), s2 (8-11).  Packed form of
// get_scale_min (crates/model/src/moe.rs:512-521):
//   j < 4:  sc = s[j] & 63,                        m = s[j+4] & 63
//   j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) | (s[j] >> 6) << 4
__device__ __forceinline__ void kq_scales4(uint32_t s0, uint32_t s1, uint32_t s2, bool hi4, uint32_t &sc,
                                           uint32_t &m) {
    const uint32_t sc_lo = s0 & 0x3F3F3F3Fu, m_lo = s1 & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    sc = hi4 ? sc_hi : sc_lo;
    m = hi4 ? m_hi : m_lo;
}

// ------------------------------------------------------------- q4_K
// block: f16 d, f16 dmin, 12 scale bytes, 128 qs bytes; 16-byte aligned.
// High nibbles are masked in place (16x their value) and the 1/16 folded
// into the scale, so each code word costs one LOP per half.
__device__ __forceinline__ float dot_q4K(const uint8_t *row, int u, const XUnit &x) {
    const int b = u >> 2, jj = u & 3;
    const uint8_t *blk = row + b * 144;
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * jj);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * jj);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t lo = q[i] & 0x0F0F0F0Fu, hi = q[i] & 0xF0F0F0F0u;
        l1 = dp4a_ss(lo, x.d1[i], l1);
        l2 = dp4a_uu(lo, x.d2[i], l2);
        l3 = dp4a_uu(lo, x.d3[i], l3);
        h1 = dp4a_us(hi, x.d1[8 + i], h1);
        h2 = dp4a_uu(hi, x.d2[8 + i], h2);
        h3 = dp4a_uu(hi, x.d3[8 + i], h3);
    }
    const float d = h2f(hd.x), dm = h2f(hd.x >> 16);
    uint32_t scw, mw;
    kq_scales4(hd.y, hd.z, hd.w, jj >= 2, scw, mw);
    const uint32_t bi = static_cast<uint32_t>((2 * jj) & 3);   // byte of sub-block 2jj; 2jj+1 is next
    const float sc1 = byte_to_f(scw, bi), sc2 = byte_to_f(scw, bi + 1);
    const float m1 = byte_to_f(mw, bi), m2 = byte_to_f(mw, bi + 1);
    const float flo = digits_to_f(l1, l2, l3) * x.s[0];
    const float fhi = digits_to_f(h1, h2, h3) * (x.s[2] * 0.0625f);
    return (d * sc1) * flo - (dm * m1) * (x.xs[0] + x.xs[1]) + (d * sc2) * fhi -
           (dm * m2) * (x.xs[2] + x.xs[3]);
}

// ------------------------------------------------------------- q5_K
// block: f16 d, f16 dmin, 12 scale bytes, qh[32], qs[128]; 16-byte aligned.
__device__ __forceinline__ float dot_q5K(const uint8_t *row, int u, const XUnit &x) {
    const int b = u >> 2, jj = u & 3;
    const uint8_t *blk = row + b * 176;
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const uint4 ha = *reinterpret_cast<const uint4 *>(blk + 16);
    const uint4 hb = *reinterpret_cast<const uint4 *>(blk + 32);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * jj);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * jj);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    const int sh = 2 * jj;
    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t lo = (q[i] & 0x0F0F0F0Fu) | (((h[i] >> sh) & 0x01010101u) << 4);
        const uint32_t hi = ((q[i] >> 4) & 0x0F0F0F0Fu) | (((h[i] >> (sh + 1)) & 0x01010101u) << 4);
        l1 = dp4a_ss(lo, x.d1[i], l1);
        l2 = dp4a_uu(lo, x.d2[i], l2);
        l3 = dp4a_uu(lo, x.d3[i], l3);
        h1 = dp4a_ss(hi, x.d1[8 + i], h1);
        h2 = dp4a_uu(hi, x.d2[8 + i], h2);
        h3 = dp4a_uu(hi, x.d3[8 + i], h3);
    }
    const float d = h2f(hd.x), dm = h2f(hd.x >> 16);
    uint32_t scw, mw;
    kq_scales4(hd.y, hd.z, hd.w, jj >= 2, scw, mw);
    const uint32_t bi = static_cast<uint32_t>((2 * jj) & 3);
    const float sc1 = byte_to_f(scw, bi), sc2 = byte_to_f(scw, bi + 1);
    const float m1 = byte_to_f(mw, bi), m2 = byte_to_f(mw, bi + 1);
    const float flo = digits_to_f(l1, l2, l3) * x.s[0];
    const float fhi = digits_to_f(h1, h2, h3) * x.s[2];
    return (d * sc1) * flo - (dm * m1) * (x.xs[0] + x.xs[1]) + (d * sc2) * fhi -
           (dm * m2) * (x.xs[2] + x.xs[3]);
}

// ------------------------------------------------------------- q6_K
// block: ql[128], qh[64], i8 scales[16], f16 d; 210 bytes, 2-byte aligned.
__device__ __forceinline__ float dot_q6K(const uint8_t *row, int u, const XUnit &x) {
    const int b = u >> 2, n = (u >> 1) & 1, t = u & 1;
    const uint8_t *blk = row + b * 210;
    const uint4 A = lds16_unaligned(blk + 64 * n + 16 * t);
    const uint4 B = lds16_unaligned(blk + 64 * n + 32 + 16 * t);
    const uint4 Hq = lds16_unaligned(blk + 128 + 32 * n + 16 * t);
    const uint2 S = lds8_unaligned(blk + 192 + 8 * n);
    const float d = h2f(*reinterpret_cast<const uint16_t *>(blk + 208));
    const uint32_t a[4] = {A.x, A.y, A.z, A.w}, bq[4] = {B.x, B.y, B.z, B.w};
    const uint32_t hh[4] = {Hq.x, Hq.y, Hq.z, Hq.w};
    int i1[4] = {0, 0, 0, 0}, i2[4] = {0, 0, 0, 0}, i3[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t c[4] = {
            (a[i] & 0x0F0F0F0Fu) | ((hh[i] << 4) & 0x30303030u),
            (bq[i] & 0x0F0F0F0Fu) | ((hh[i] << 2) & 0x30303030u),
            ((a[i] >> 4) & 0x0F0F0F0Fu) | (hh[i] & 0x30303030u),
            ((bq[i] >> 4) & 0x0F0F0F0Fu) | ((hh[i] >> 2) & 0x30303030u)};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            i1[q] = dp4a_ss(c[q], x.d1[4 * q + i], i1[q]);
            i2[q] = dp4a_uu(c[q], x.d2[4 * q + i], i2[q]);
            i3[q] = dp4a_uu(c[q], x.d3[4 * q + i], i3[q]);
        }
    }
    // scales[8n + t + 2q]: bytes t, t+2 of S.x (q = 0, 1) and of S.y (q = 2, 3)
    const uint32_t sx = S.x ^ 0x80808080u, sy = S.y ^ 0x80808080u;
    const uint32_t tb = static_cast<uint32_t>(t);
    const float sc0 = sbyte_to_f(sx, tb), sc1 = sbyte_to_f(sx, tb + 2);
    const float sc2 = sbyte_to_f(sy, tb), sc3 = sbyte_to_f(sy, tb + 2);
    const float acc = sc0 * (digits_to_f(i1[0], i2[0], i3[0]) * x.s[0] - 32.f * x.xs[0]) +
                      sc1 * (digits_to_f(i1[1], i2[1], i3[1]) * x.s[1] - 32.f * x.xs[1]) +
                      sc2 * (digits_to_f(i1[2], i2[2], i3[2]) * x.s[2] - 32.f * x.xs[2]) +
                      sc3 * (digits_to_f(i1[3], i2[3], i3[3]) * x.s[3] - 32.f * x.xs[3]);
    return d * acc;
}

// ------------------------------------------------------------- q8_0
// block: f16 d, i8 qs[32]; 34 bytes, 2-byte aligned.
__device__ __forceinline__ float dot_q8_0(const uint8_t *row, int u, const XUnit &x) {
    float acc = 0.f;
#pragma unroll
    for (int hb = 0; hb < 2; hb++) {
        const uint8_t *blk = row + (2 * u + hb) * 34;
        const float d = h2f(*reinterpret_cast<const uint16_t *>(blk));
        const uint4 qa = lds16_unaligned(blk + 2);
        const uint4 qb = lds16_unaligned(blk + 18);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        int i1 = 0, i2 = 0, i3 = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            i1 = dp4a_ss(q[i], x.d1[8 * hb + i], i1);
            i2 = dp4a_su(q[i], x.d2[8 * hb + i], i2);
            i3 = dp4a_su(q[i], x.d3[8 * hb + i], i3);
        }
        acc += d * (digits_to_f(i1, i2, i3) * x.s[2 * hb]);
    }
    return acc;
}

template <int QT>
__device__ __forceinline__ float unit_dot(const uint8_t *row, int u, const XUnit &x) {
    if constexpr (QT == STYX_Q4_K) return dot_q4K(row, u, x);
    else if constexpr (QT == STYX_Q5_K) return dot_q5K(row, u, x);
    else if constexpr (QT == STYX_Q6_K) return dot_q6K(row, u, x);
    else return dot_q8_0(row, u, x);
}

}  // namespace styx
