// synth.cu -- device generator of synthetic quantised expert tensors.
//
// Benchmark-sized models (tens of GB of expert slabs) are generated on the
// GPU: value(seed, i) = sigma * N(0,1) from a counter-based hash (splitmix64
// + Box-Muller), then quantised per block with the same min/max scheme the
// test oracle uses for its test data (oracle/styx_oracle.c, "quantizers").
// Built with -fmad=false so the quantiser rounds exactly like the C code.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace styx {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_value(uint64_t seed, uint64_t i, float sigma) {
    const uint64_t h = splitmix64(seed * 0xD1B54A32D192ED03ull ^ splitmix64(i));
    const float u1 = (static_cast<float>(static_cast<uint32_t>(h >> 40)) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>(static_cast<uint32_t>(h & 0xFFFFFFu)) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    return sigma * r * cospif(2.0f * u2);
}

__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float h2f16(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ void q_q8_0_dev(const float *x, uint8_t *b) {
    float amax = 0.f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
    const uint16_t dh = f2h(amax / 127.f);
    const float df = h2f16(dh);
    b[0] = dh & 0xFF;
    b[1] = dh >> 8;
    for (int i = 0; i < 32; i++) {
        int q = df > 0.f ? static_cast<int>(rintf(x[i] / df)) : 0;
        q = q > 127 ? 127 : q < -127 ? -127 : q;
        b[2 + i] = static_cast<uint8_t>(static_cast<int8_t>(q));
    }
}

__device__ void kq_scales_dev(const float *x, int nmax, uint8_t *sc, uint8_t *mn, uint16_t &dh, uint16_t &dmh,
                              float &df, float &dmf) {
    float scf[8], mf[8], smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; j++) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; i++) {
            const float v = x[32 * j + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.f) lo = 0.f;
        scf[j] = (hi - lo) / static_cast<float>(nmax);
        mf[j] = -lo;
        if (scf[j] > smax) smax = scf[j];
        if (mf[j] > mmax) mmax = mf[j];
    }
    dh = f2h(smax / 63.f);
    dmh = f2h(mmax / 63.f);
    df = h2f16(dh);
    dmf = h2f16(dmh);
    for (int j = 0; j < 8; j++) {
        int s = df > 0.f ? static_cast<int>(rintf(scf[j] / df)) : 0;
        int m = dmf > 0.f ? static_cast<int>(rintf(mf[j] / dmf)) : 0;
        sc[j] = static_cast<uint8_t>(s < 0 ? 0 : s > 63 ? 63 : s);
        mn[j] = static_cast<uint8_t>(m < 0 ? 0 : m > 63 ? 63 : m);
    }
}

__device__ void kq_pack_dev(const uint8_t *sc, const uint8_t *mn, uint8_t *s) {
    for (int j = 0; j < 4; j++) {
        s[j] = static_cast<uint8_t>(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = static_cast<uint8_t>(mn[j] | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 0x0F) | ((mn[j + 4] & 0x0F) << 4));
    }
}

__device__ __forceinline__ int kq_level_dev(float v, float dsc, float off, int nmax) {
    if (!(dsc > 0.f)) return 0;
    const int q = static_cast<int>(rintf((v + off) / dsc));
    return q < 0 ? 0 : q > nmax ? nmax : q;
}

__device__ void q_k45_dev(const float *x, uint8_t *b, bool five) {
    uint8_t sc[8], mn[8];
    uint16_t dh, dmh;
    float d, dmin;
    const int nmax = five ? 31 : 15;
    kq_scales_dev(x, nmax, sc, mn, dh, dmh, d, dmin);
    b[0] = dh & 0xFF;
    b[1] = dh >> 8;
    b[2] = dmh & 0xFF;
    b[3] = dmh >> 8;
    kq_pack_dev(sc, mn, b + 4);
    uint8_t *qh = b + 16, *qs = five ? b + 48 : b + 16;
    if (five)
        for (int l = 0; l < 32; l++) qh[l] = 0;
    for (int j = 0; j < 4; j++) {
        const float ds1 = d * static_cast<float>(sc[2 * j]), o1 = dmin * static_cast<float>(mn[2 * j]);
        const float ds2 = d * static_cast<float>(sc[2 * j + 1]), o2 = dmin * static_cast<float>(mn[2 * j + 1]);
        for (int l = 0; l < 32; l++) {
            const int lo = kq_level_dev(x[64 * j + l], ds1, o1, nmax);
            const int hi = kq_level_dev(x[64 * j + 32 + l], ds2, o2, nmax);
            qs[32 * j + l] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
            if (five) {
                qh[l] |= static_cast<uint8_t>(((lo >> 4) & 1) << (2 * j));
                qh[l] |= static_cast<uint8_t>(((hi >> 4) & 1) << (2 * j + 1));
            }
        }
    }
}

__device__ void q_q6_K_dev(const float *x, uint8_t *b) {
    float scf[16], smax = 0.f;
    for (int s = 0; s < 16; s++) {
        float a = 0.f;
        for (int i = 0; i < 16; i++) a = fmaxf(a, fabsf(x[16 * s + i]));
        scf[s] = a / 31.f;
        if (scf[s] > smax) smax = scf[s];
    }
    const uint16_t dh = f2h(smax / 127.f);
    const float d = h2f16(dh);
    int8_t sc[16];
    for (int s = 0; s < 16; s++) {
        const int v = d > 0.f ? static_cast<int>(rintf(scf[s] / d)) : 0;
        sc[s] = static_cast<int8_t>(v < 0 ? 0 : v > 127 ? 127 : v);
    }
    uint8_t *ql = b, *qh = b + 128;
    for (int n = 0; n < 2; n++) {
        for (int l = 0; l < 32; l++) {
            uint8_t q[4];
            for (int k = 0; k < 4; k++) {
                const int i = 128 * n + 32 * k + l;
                const float ds = d * static_cast<float>(sc[i / 16]);
                int v = ds > 0.f ? static_cast<int>(rintf(x[i] / ds)) : 0;
                v = v < -32 ? -32 : v > 31 ? 31 : v;
                q[k] = static_cast<uint8_t>(v + 32);
            }
            ql[64 * n + l] = static_cast<uint8_t>((q[0] & 15) | ((q[2] & 15) << 4));
            ql[64 * n + 32 + l] = static_cast<uint8_t>((q[1] & 15) | ((q[3] & 15) << 4));
            qh[32 * n + l] = static_cast<uint8_t>((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) |
                                                  ((q[3] >> 4) << 6));
        }
    }
    for (int s = 0; s < 16; s++) b[192 + s] = static_cast<uint8_t>(sc[s]);
    b[208] = dh & 0xFF;
    b[209] = dh >> 8;
}

// one thread per block; values regenerated from (seed, row*ncols + col)
__global__ void __launch_bounds__(128) k_synth_quant(int qtype, uint8_t *dst, uint64_t nrows, int ncols,
                                                     uint64_t seed, float sigma) {
    const int be = qtype == STYX_Q8_0 ? 32 : 256;
    const int bb = qtype == STYX_Q8_0 ? 34 : qtype == STYX_Q4_K ? 144 : qtype == STYX_Q5_K ? 176 : 210;
    const uint64_t bpr = static_cast<uint64_t>(ncols / be);
    const uint64_t nblk = nrows * bpr;
    float x[256];
    uint8_t ob[210];
    for (uint64_t blk = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; blk < nblk;
         blk += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t row = blk / bpr, b = blk % bpr;
        const uint64_t i0 = row * static_cast<uint64_t>(ncols) + b * be;
        for (int i = 0; i < be; i++) x[i] = synth_value(seed, i0 + i, sigma);
        switch (qtype) {
        case STYX_Q8_0: q_q8_0_dev(x, ob); break;
        case STYX_Q4_K: q_k45_dev(x, ob, false); break;
        case STYX_Q5_K: q_k45_dev(x, ob, true); break;
        default: q_q6_K_dev(x, ob); break;
        }
        uint8_t *o = dst + blk * bb;
        for (int i = 0; i < bb; i++) o[i] = ob[i];
    }
}

__global__ void k_synth_f32(float *dst, uint64_t n, uint64_t seed, uint64_t offset, float sigma) {
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = synth_value(seed, offset + i, sigma);
}

cudaError_t launch_synth_quant(int qtype, uint8_t *dst, uint64_t nrows, int ncols, uint64_t seed, float sigma,
                               cudaStream_t st) {
    k_synth_quant<<<148 * 16, 128, 0, st>>>(qtype, dst, nrows, ncols, seed, sigma);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(float *dst, uint64_t n, uint64_t seed, uint64_t offset, float sigma,
                             cudaStream_t st) {
    k_synth_f32<<<148 * 8, 256, 0, st>>>(dst, n, seed, offset, sigma);
    return cudaGetLastError();
}

}  // namespace styx
