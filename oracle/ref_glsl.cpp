// ref_glsl.cpp -- the reference's hot-path GLSL shaders, compiled as C++.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/ref_glsl.mk into
// oracle/_ref/libref_glsl.so from the shader sources in the reference tree
// (shaders/*.comp, preprocessed into oracle/_ref/*.inc by ref_glsl.sed).
// Each extern "C" driver below binds the buffers and push constants the
// way crates/model/src/moe.rs dispatches the shader and runs the whole
// dispatch grid on the CPU.
#include <cstring>

#include "ref_glsl_shim.h"

thread_local uint glsl_lid = 0;
uint glsl_wgid = 0;
uint glsl_local_size = 1;

namespace ref_matvec {
GLSL_BUILTINS
#include "matvec_strided_f32.inc"
}  // namespace ref_matvec

namespace ref_topk {
GLSL_BUILTINS
#include "topk_softmax_f32.inc"
}  // namespace ref_topk

namespace ref_reduce {
GLSL_BUILTINS
#include "moe_reduce_f32.inc"
}  // namespace ref_reduce

namespace ref_gather {
GLSL_BUILTINS
#include "gather_slabs_f32.inc"
}  // namespace ref_gather

namespace ref_attn {
GLSL_BUILTINS
#include "attn_decode_f32.inc"
}  // namespace ref_attn

namespace ref_add {
GLSL_BUILTINS
#include "add_flat_f32.inc"
}  // namespace ref_add

extern "C" {

// matvec_strided_f32 dispatched as moe.rs:1984-1996: push {ncols, stride_a},
// groups (nrows, 1, 1), 32 invocations with barriers.
void ref_matvec_strided_f32(const float *a, const float *x, float *d, uint nrows, uint ncols, uint stride_a) {
    ref_matvec::data_a = const_cast<float *>(a);
    ref_matvec::data_x = const_cast<float *>(x);
    ref_matvec::data_d = d;
    ref_matvec::p.ncols = ncols;
    ref_matvec::p.stride_a = stride_a;
    glsl_local_size = 32;
    omp_set_dynamic(0);
    for (uint wg = 0; wg < nrows; wg++) {
        glsl_wgid = wg;
#pragma omp parallel num_threads(32)
        {
            glsl_lid = static_cast<uint>(omp_get_thread_num());
            ref_matvec::main();
        }
    }
}

// topk_softmax_f32 dispatched as moe.rs:1998-2016: push {n, k, renorm},
// one invocation; ids is the layer's 64-int block.
void ref_topk_softmax_f32(const float *logits, float *weights, int *ids, const uint *remap, const uint *pmap,
                          uint n, uint k, uint renorm) {
    ref_topk::logits = const_cast<float *>(logits);
    ref_topk::weights = weights;
    ref_topk::ids = ids;
    ref_topk::remap = const_cast<uint *>(remap);
    ref_topk::pmap = const_cast<uint *>(pmap);
    ref_topk::p.n = n;
    ref_topk::p.k = k;
    ref_topk::p.renorm = renorm;
    glsl_local_size = 1;
    glsl_wgid = 0;
    glsl_lid = 0;
    ref_topk::main();
}

// moe_reduce_f32 dispatched as moe.rs:2050-2062: push {ne, k},
// groups ceil(ne/256).
void ref_moe_reduce_f32(const float *d, const float *w, float *x, uint ne, uint k) {
    ref_reduce::data_d = const_cast<float *>(d);
    ref_reduce::w = const_cast<float *>(w);
    ref_reduce::x = x;
    ref_reduce::p.ne = ne;
    ref_reduce::p.k = k;
    glsl_local_size = 256;
    for (uint wg = 0; wg < (ne + 255) / 256; wg++) {
        glsl_wgid = wg;
        for (uint l = 0; l < 256; l++) {
            glsl_lid = l;
            ref_reduce::main();
        }
    }
}

// gather_slabs_f32 recorded as moe.rs:1706-1744: push {dst_vg, dst_vu,
// dst_vd, src_vg, src_vu, src_vd, layer, k, canary} in uvec4 units, groups
// (k, 1, 1), 256 invocations.
void ref_gather_slabs_f32(const void *gate, const void *up, const void *down, void *arena_g, void *arena_u,
                          void *arena_d, const int *ids, uint dst_vg, uint dst_vu, uint dst_vd, uint src_vg,
                          uint src_vu, uint src_vd, uint layer, uint k) {
    ref_gather::gate = static_cast<uvec4 *>(const_cast<void *>(gate));
    ref_gather::up = static_cast<uvec4 *>(const_cast<void *>(up));
    ref_gather::down = static_cast<uvec4 *>(const_cast<void *>(down));
    ref_gather::arena_g = static_cast<uvec4 *>(arena_g);
    ref_gather::arena_u = static_cast<uvec4 *>(arena_u);
    ref_gather::arena_d = static_cast<uvec4 *>(arena_d);
    ref_gather::ids = const_cast<int *>(ids);
    ref_gather::p.dst_vg = dst_vg;
    ref_gather::p.dst_vu = dst_vu;
    ref_gather::p.dst_vd = dst_vd;
    ref_gather::p.src_vg = src_vg;
    ref_gather::p.src_vu = src_vu;
    ref_gather::p.src_vd = src_vd;
    ref_gather::p.layer = layer;
    ref_gather::p.k = k;
    ref_gather::p.canary = 0;
    glsl_local_size = 256;
    for (uint wg = 0; wg < k; wg++) {
        glsl_wgid = wg;
        for (uint l = 0; l < 256; l++) {
            glsl_lid = l;
            ref_gather::main();
        }
    }
}

// attn_decode_f32 dispatched as moe.rs:1946-1964: push {n_t, hd, kv_dim,
// gqa, scale}, groups (n_heads, 1, 1), 128 invocations with barriers.
void ref_attn_decode_f32(const float *q, const float *k, const float *v, float *o, uint n_heads, uint n_t, uint hd,
                         uint kv_dim, uint gqa, float scale) {
    ref_attn::data_q = const_cast<float *>(q);
    ref_attn::data_k = const_cast<float *>(k);
    ref_attn::data_v = const_cast<float *>(v);
    ref_attn::data_o = o;
    ref_attn::p.n_t = n_t;
    ref_attn::p.hd = hd;
    ref_attn::p.kv_dim = kv_dim;
    ref_attn::p.gqa = gqa;
    ref_attn::p.scale = scale;
    glsl_local_size = 128;
    omp_set_dynamic(0);
    for (uint wg = 0; wg < n_heads; wg++) {
        glsl_wgid = wg;
#pragma omp parallel num_threads(128)
        {
            glsl_lid = static_cast<uint>(omp_get_thread_num());
            ref_attn::main();
        }
    }
}

// add_flat_f32 (rec_add, moe.rs:1972): push {n}, groups ceil(n/256).
void ref_add_flat_f32(const float *a, const float *b, float *d, uint n) {
    ref_add::data_a = const_cast<float *>(a);
    ref_add::data_b = const_cast<float *>(b);
    ref_add::data_d = d;
    ref_add::p.n = n;
    glsl_local_size = 256;
    for (uint wg = 0; wg < (n + 255) / 256; wg++) {
        glsl_wgid = wg;
        for (uint l = 0; l < 256; l++) {
            glsl_lid = l;
            ref_add::main();
        }
    }
}

}  // extern "C"
