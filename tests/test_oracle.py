"""Pins the CPU oracle against golden vectors (no GPU).

The golden vectors (tests/golden/quant_golden.npz, made by gen_golden.py)
hold llama.cpp gguf-py 0.19.0 decodes of q8_0/q4_K/q5_K/q6_K blocks and the
reference's own GPU-test cases (crates/vk-backend/tests/kernels.rs, ops2.rs)
re-created from their seeds.
"""
import numpy as np
import pytest


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["q8_0", "q4_K", "q5_K", "q6_K"])
def test_dequant_matches_gguf_py(oracle_mod, golden, name):
    O = oracle_mod
    qt = O.QTYPES[name]
    be, bb = O.BLOCK[qt]
    raw = golden[f"{name}_raw"]
    nblk = raw.size // bb
    got = O.dequantize(qt, raw, nblk * be).reshape(-1)
    assert np.array_equal(bits(got), bits(golden[f"{name}_deq"]))


def test_idmv_q4k_reference_case(oracle_mod, golden):
    """kernels.rs:150-285: 8 experts of 32x512 q4_K, ids [6,1,3,0]."""
    O = oracle_mod
    a, x = golden["idmv_a"], golden["idmv_x"]
    eb = 32 * 2 * 144
    for tag in ("ids0", "ids1"):
        y = O.mul_mat_vec_id(O.Q4_K, a, eb, 32, 512, golden[f"idmv_{tag}"], x, 1)
        assert np.array_equal(bits(y), bits(golden[f"idmv_y_{tag}"]))
    # permuting the ids moves the outputs (kernels.rs:272-279)
    y0 = O.mul_mat_vec_id(O.Q4_K, a, eb, 32, 512, golden["idmv_ids0"], x, 1)
    y1 = O.mul_mat_vec_id(O.Q4_K, a, eb, 32, 512, golden["idmv_ids1"], x, 1)
    assert np.array_equal(y1[:32], y0[96:128])
    assert np.array_equal(y1[32:64], y0[:32])


def test_matvec_q4k_q8_reference_cases(oracle_mod, golden):
    O = oracle_mod
    y = O.matvec_q(O.Q4_K, golden["mvq4_a"], 64, 512, golden["mvq4_x"])
    assert np.array_equal(bits(y), bits(golden["mvq4_y"]))
    y = O.matvec_q(O.Q8_0, golden["mvq8_a"], 128, 1024, golden["mvq8_x"])
    assert np.array_equal(bits(y), bits(golden["mvq8_y"]))


def test_swiglu_reference_case(oracle_mod, golden):
    O = oracle_mod
    y = O.swiglu(golden["swiglu_g"], golden["swiglu_u"])
    # expf (C) and numpy exp may differ by an ulp; ops2.rs:343 allows 1e-5 abs
    np.testing.assert_allclose(y, golden["swiglu_y"], rtol=2e-7, atol=1e-7)


def test_rms_norm_reference_case(oracle_mod, golden):
    O = oracle_mod
    xr = golden["rms_x"]
    for r in range(4):
        y = O.rms_norm(xr[r], None, 1e-6)
        np.testing.assert_allclose(y, golden["rms_y"][r], rtol=0, atol=1e-7)


@pytest.mark.parametrize("name,tol", [("q8_0", 0.01), ("q4_K", 0.1), ("q5_K", 0.05), ("q6_K", 0.03)])
def test_quantizer_roundtrip(oracle_mod, name, tol):
    """Test-data quantizers emit well-formed blocks close to the input."""
    O = oracle_mod
    qt = O.QTYPES[name]
    x = np.random.default_rng(7).normal(0, 0.02, size=(8, 1024)).astype(np.float32)
    y = O.dequantize(qt, O.quantize(qt, x), 1024).reshape(x.shape)
    rel = np.sqrt(np.mean((x - y) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < tol


def test_topk_serial_semantics(oracle_mod):
    """topk_softmax_f32.comp:39-51: strict '>' scan, ties to lowest index,
    ids in selection order, renormalised weights sum to 1."""
    O = oracle_mod
    logits = np.array([0.5, 2.0, 2.0, -1.0, 3.0, 2.0, 0.0, 1.0], np.float32)
    w, ids = O.topk_softmax(logits, 4, renorm=True)
    assert list(ids[:4]) == [4, 1, 2, 5]
    assert abs(float(w.sum()) - 1.0) < 1e-6
    assert w[1] == w[2] == w[3]
    # all rows: no remap/pmap -> hot/arena SKIP, gtt row = original ids
    assert all(ids[16 + s] == -1 and ids[32 + s] == -1 for s in range(4))
    assert list(ids[48:52]) == [4, 1, 2, 5]
    # -inf is never picked; fewer than k finite logits -> id -1
    l2 = np.array([-np.inf, 1.0, -np.inf, -np.inf], np.float32)
    w2, ids2 = O.topk_softmax(l2, 2, renorm=False)
    assert ids2[0] == 1 and ids2[1] == -1 and w2[1] == 0.0


def test_topk_remap_pmap_rows(oracle_mod):
    """topk_softmax_f32.comp:52-66: hot / arena / gtt rows partition the
    routed experts."""
    O = oracle_mod
    n, k = 16, 4
    logits = np.linspace(-1, 1, n).astype(np.float32)[::-1].copy()  # 0 is best
    remap = np.full(n, O.SKIP, np.uint32)
    remap[1] = 7
    pmap = np.full(n, O.SKIP, np.uint32)
    pmap[2] = 33
    w, ids = O.topk_softmax(logits, k, True, remap, pmap)
    assert list(ids[:4]) == [0, 1, 2, 3]
    assert list(ids[16:20]) == [-1, 7, -1, -1]
    assert list(ids[32:36]) == [-1, -1, 33, -1]
    assert list(ids[48:52]) == [0, -1, -1, 3]


def test_gather_slabs_semantics(oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(3)
    E, k, layer = 6, 3, 2
    sb = [64, 48, 80]
    db = [96, 64, 80]
    srcs = [rng.integers(0, 256, E * b, dtype=np.uint8) for b in sb]
    arenas = [np.zeros((layer + 1) * k * b, np.uint8) for b in db]
    ids = np.array([4, -1, 1], np.int32)
    O.gather_slabs(srcs, sb, arenas, db, ids, layer, k)
    for t in range(3):
        for s, e in enumerate(ids):
            slot = layer * k + s
            got = arenas[t][slot * db[t]: slot * db[t] + sb[t]]
            if e < 0:
                assert not got.any()
            else:
                assert np.array_equal(got, srcs[t][e * sb[t]:(e + 1) * sb[t]])
