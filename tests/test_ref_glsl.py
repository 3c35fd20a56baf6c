"""Pins the oracle against the reference's own GLSL shaders compiled as C++
(oracle/_ref/libref_glsl.so, built by oracle/ref_glsl.mk from the reference
tree's shaders/*.comp).  Skipped where the reference tree is absent (the
GPU box); the oracle restatement must match bit for bit."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_DIR = os.path.join(os.path.dirname(HERE), "oracle")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libref_glsl.so")
REF_ROOT = os.environ.get("STYX_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
REF_TREE = os.path.join(REF_ROOT, "shaders")


@pytest.fixture(scope="module")
def ref():
    if os.path.isdir(REF_TREE):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR, "-f", "ref_glsl.mk", "REF=" + REF_ROOT], check=True)
    if not os.path.exists(REF_SO):
        pytest.skip("reference shaders not built (reference tree absent)")
    L = C.CDLL(REF_SO)
    vp, u = C.c_void_p, C.c_uint
    L.ref_matvec_strided_f32.argtypes = [vp, vp, vp, u, u, u]
    L.ref_topk_softmax_f32.argtypes = [vp, vp, vp, vp, vp, u, u, u]
    L.ref_moe_reduce_f32.argtypes = [vp, vp, vp, u, u]
    L.ref_gather_slabs_f32.argtypes = [vp] * 7 + [u] * 8
    L.ref_attn_decode_f32.argtypes = [vp, vp, vp, vp, u, u, u, u, u, C.c_float]
    L.ref_add_flat_f32.argtypes = [vp, vp, vp, u]
    return L


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("E,H", [(128, 2048), (32, 512), (128, 4096), (7, 96)])
def test_router_gemv_matches_reference_shader(ref, E, H):
    rng = np.random.default_rng(E + H)
    a = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    x = rng.normal(0, 1, H).astype(np.float32)
    d = np.zeros(E, np.float32)
    ref.ref_matvec_strided_f32(_p(a), _p(x), _p(d), E, H, H)
    assert np.array_equal(bits(O.matvec_strided_f32(a, x)), bits(d))


def _ref_topk(ref, logits, k, renorm, remap, pmap):
    w = np.zeros(16, np.float32)
    ids = np.full(64, -7, np.int32)
    ref.ref_topk_softmax_f32(_p(logits), _p(w), _p(ids), _p(remap), _p(pmap), logits.size, k, int(renorm))
    return w[:k], ids


@pytest.mark.parametrize("E,k", [(128, 8), (32, 4), (512, 16), (64, 1)])
@pytest.mark.parametrize("renorm", [True, False])
def test_topk_matches_reference_shader(ref, E, k, renorm):
    rng = np.random.default_rng(E * 7 + k)
    for trial in range(20):
        logits = rng.normal(0, 2, E).astype(np.float32)
        if trial % 4 == 1:                       # exact ties
            logits[rng.integers(0, E, E // 4)] = logits[0]
        if trial % 4 == 2:                       # coarse values, many ties
            logits = np.round(logits).astype(np.float32)
        remap = np.full(E, O.SKIP, np.uint32)
        pmap = np.full(E, O.SKIP, np.uint32)
        if trial % 2:
            hot = np.sort(rng.choice(E, E // 3, replace=False))
            remap[hot] = np.arange(hot.size, dtype=np.uint32)
            pm = rng.choice(E, E // 4, replace=False)
            pmap[pm] = rng.integers(0, 400, pm.size).astype(np.uint32)
        rw, rids = _ref_topk(ref, logits, k, renorm, remap, pmap)
        ow, oids = O.topk_softmax(logits, k, renorm, remap, pmap)
        assert np.array_equal(bits(ow), bits(rw))
        # the shader writes rows 0/16/32/48 only up to k; compare those
        for base in (0, 16, 32, 48):
            assert np.array_equal(oids[base:base + k], rids[base:base + k])


def test_moe_reduce_matches_reference_shader(ref):
    rng = np.random.default_rng(3)
    for ne, k in ((2048, 8), (4096, 8), (300, 5), (512, 16)):
        d = rng.normal(0, 1, k * ne).astype(np.float32)
        w = rng.random(k).astype(np.float32)
        x = rng.normal(0, 1, ne).astype(np.float32)
        xr = x.copy()
        ref.ref_moe_reduce_f32(_p(d), _p(w), _p(xr), ne, k)
        assert np.array_equal(bits(O.moe_reduce(d, w, x)), bits(xr))


def test_gather_slabs_matches_reference_shader(ref):
    rng = np.random.default_rng(4)
    E, k, layer = 9, 4, 2
    sb = [1024, 2048, 512]
    db = [2048, 2048, 1024]
    srcs = [rng.integers(0, 256, E * b, dtype=np.uint8) for b in sb]
    ids = np.array([5, -1, 0, 8], np.int32)
    a_ref = [np.zeros((layer + 1) * k * b, np.uint8) for b in db]
    a_or = [np.zeros((layer + 1) * k * b, np.uint8) for b in db]
    ref.ref_gather_slabs_f32(*[_p(s) for s in srcs], *[_p(a) for a in a_ref], _p(ids),
                             *[b // 16 for b in db], *[b // 16 for b in sb], layer, k)
    O.gather_slabs(srcs, sb, a_or, db, ids, layer, k)
    for x, y in zip(a_ref, a_or):
        assert np.array_equal(x, y)


# ------------------------------------------------------------ attention half of a decode layer
@pytest.mark.parametrize("n_heads,n_kv,hd,n_t", [(8, 2, 128, 1), (8, 2, 128, 37), (4, 4, 64, 9),
                                                 (6, 2, 256, 5), (32, 4, 128, 12), (2, 1, 96, 3)])
def test_attn_decode_matches_reference_shader(ref, n_heads, n_kv, hd, n_t):
    """attn_decode_f32.comp (one workgroup of 128 invocations per q head,
    online softmax over the cache rows) against its C restatement, bit for bit."""
    rng = np.random.default_rng(n_heads * 1000 + hd + n_t)
    kv_dim, gqa = n_kv * hd, n_heads // n_kv
    q = rng.normal(0, 1, n_heads * hd).astype(np.float32)
    k = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    v = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    got = np.zeros(n_heads * hd, np.float32)
    ref.ref_attn_decode_f32(_p(q), _p(k), _p(v), _p(got), n_heads, n_t, hd, kv_dim, gqa, float(scale))
    exp = O.attn_decode(q, k, v, n_heads, n_t, hd, kv_dim, gqa, float(scale))
    assert np.array_equal(bits(exp), bits(got))


def test_add_flat_matches_reference_shader(ref):
    rng = np.random.default_rng(5)
    a = rng.normal(0, 1, 1000).astype(np.float32)
    b = rng.normal(0, 1, 1000).astype(np.float32)
    d = np.zeros_like(a)
    ref.ref_add_flat_f32(_p(a), _p(b), _p(d), a.size)
    assert np.array_equal(bits(d), bits(a + b))
