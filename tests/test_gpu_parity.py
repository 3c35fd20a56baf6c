"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Tolerances: routing ids bit-exact wherever the top-k margin exceeds 1e-4;
hidden states within 1e-3 relative (the kernels land
near 1e-6); quantised GEMVs within 1e-4 of max|y| (the reference's own tests
allow 2e-2 for q4_K and 1e-3 for q8_0); copies and the slot-ordered reduce
bit-exact.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block, topk_margin

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def T(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def id_rows(ids64, k):
    """The written part of a 64-int id block: rows 0/16/32/48, k entries each."""
    ids64 = np.asarray(ids64)
    return np.concatenate([ids64[b:b + k] for b in (0, 16, 32, 48)])


def rel_to_max(got, exp):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


# ----------------------------------------------------- reference test cases
def test_mul_mat_vec_id_q4k_reference_case(golden):
    """crates/vk-backend/tests/kernels.rs:150-285 re-created from its seed."""
    a, x = T(golden["idmv_a"]), T(golden["idmv_x"])
    eb = 32 * 2 * 144
    outs = {}
    for tag in ("ids0", "ids1"):
        ids = T(golden[f"idmv_{tag}"])
        y = ops.mul_mat_vec_id(_lib.Q4_K, a, eb, 32, 512, ids, x, 1).cpu().numpy()
        exp = golden[f"idmv_y_{tag}"]
        rel = np.max(np.abs(y - exp) / np.maximum(np.abs(exp), 1e-3))
        assert rel < 1e-4, rel          # reference bound: 2e-2
        outs[tag] = y
    # permuting the ids moves the outputs (kernels.rs:272-279)
    np.testing.assert_allclose(outs["ids1"][:32], outs["ids0"][96:128], rtol=1e-6, atol=0)
    np.testing.assert_allclose(outs["ids1"][32:64], outs["ids0"][:32], rtol=1e-6, atol=0)


@pytest.mark.parametrize("tag,qt,nrows,ncols,bound", [("mvq4", _lib.Q4_K, 64, 512, 2e-2),
                                                      ("mvq8", _lib.Q8_0, 128, 1024, 1e-3)])
def test_matvec_reference_cases(golden, tag, qt, nrows, ncols, bound):
    """kernels.rs:353-456 (q4_K) and ops2.rs:225-292 (q8_0)."""
    a = T(golden[f"{tag}_a"])
    ids = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = ops.mul_mat_vec_id(qt, a, a.numel(), nrows, ncols, ids, T(golden[f"{tag}_x"]), 1).cpu().numpy()
    exp = golden[f"{tag}_y"]
    # the reference's own measure and bound (per-element rel, floor 1e-3)...
    rel = np.max(np.abs(y - exp) / np.maximum(np.abs(exp), 1e-3))
    assert rel < bound, rel
    # ...and against the row scale (the f32 column-order sum of the reference
    # itself carries ~1e-5 of max|y| of rounding at 1024 columns)
    assert rel_to_max(y, exp) < 5e-5


def test_swiglu_reference_case(golden):
    y = ops.swiglu(T(golden["swiglu_g"]), T(golden["swiglu_u"])).cpu().numpy()
    assert np.max(np.abs(y - golden["swiglu_y"])) < 1e-5          # ops2.rs:343


def test_rms_norm_reference_case(golden):
    y = ops.rms_norm(T(golden["rms_x"]), None, 1e-6).cpu().numpy()
    assert np.max(np.abs(y - golden["rms_y"])) < 1e-5             # kernels.rs:116


# ----------------------------------------------------------- single ops
@pytest.mark.parametrize("qname", ["q8_0", "q4_K", "q5_K", "q6_K"])
@pytest.mark.parametrize("ncols,ne11", [(512, 1), (768, 4), (2048, 1), (4096, 2)])
def test_mul_mat_vec_id_all_types(qname, ncols, ne11):
    qt = _lib.QTYPES[qname]
    if qt != _lib.Q8_0 and ncols % 256:
        pytest.skip("k-quants need 256-column rows")
    rng = np.random.default_rng(ncols + qt)
    E, nrows, k = 6, 40, 4
    w = O.quantize(qt, rng.normal(0, 0.02, (E * nrows, ncols)).astype(np.float32)).reshape(-1)
    eb = w.size // E
    x = rng.normal(0, 1, (ne11, ncols)).astype(np.float32)
    ids = np.array([3, 0, 5, 1], np.int32)
    exp = O.mul_mat_vec_id(qt, w, eb, nrows, ncols, ids, x.reshape(-1), ne11)
    y = ops.mul_mat_vec_id(qt, T(w), eb, nrows, ncols, T(ids), T(x.reshape(-1)), ne11).cpu().numpy()
    assert rel_to_max(y, exp) < 1e-5


def test_mul_mat_vec_id_skip_leaves_output():
    rng = np.random.default_rng(1)
    w = O.quantize(_lib.Q4_K, rng.normal(0, 0.02, (4 * 16, 256)).astype(np.float32)).reshape(-1)
    y = torch.full((2 * 16,), 7.0, device=DEV)
    ids = T(np.array([-1, 2], np.int32))
    ops.mul_mat_vec_id(_lib.Q4_K, T(w), w.size // 4, 16, 256, ids,
                       T(rng.normal(0, 1, 256).astype(np.float32)), 1, y=y)
    y = y.cpu().numpy()
    assert np.all(y[:16] == 7.0) and not np.all(y[16:] == 7.0)


@pytest.mark.parametrize("E,k", [(128, 8), (32, 4), (512, 16), (8, 8)])
def test_topk_softmax_random(E, k):
    rng = np.random.default_rng(E * 31 + k)
    for trial in range(5):
        logits = rng.normal(0, 2, E).astype(np.float32)
        ew, eids = O.topk_softmax(logits, k, True)
        w, ids = ops.topk_softmax(T(logits), k, True)
        assert np.array_equal(id_rows(ids.cpu().numpy(), k), id_rows(eids, k))
        np.testing.assert_allclose(w.cpu().numpy(), ew, rtol=2e-6, atol=1e-7)


def test_topk_softmax_ties_and_edges():
    logits = np.array([0.5, 2.0, 2.0, -1.0, 3.0, 2.0, 0.0, 1.0], np.float32)
    for renorm in (True, False):
        ew, eids = O.topk_softmax(logits, 4, renorm)
        w, ids = ops.topk_softmax(T(logits), 4, renorm)
        assert np.array_equal(id_rows(ids.cpu().numpy(), 4), id_rows(eids, 4))
        np.testing.assert_allclose(w.cpu().numpy(), ew, rtol=2e-6)
    l2 = np.array([-np.inf, 1.0, -np.inf, -np.inf], np.float32)
    ew, eids = O.topk_softmax(l2, 2, False)
    w, ids = ops.topk_softmax(T(l2), 2, False)
    assert np.array_equal(id_rows(ids.cpu().numpy(), 2), id_rows(eids, 2))
    np.testing.assert_allclose(w.cpu().numpy(), ew)


def test_topk_softmax_remap_pmap_rows():
    rng = np.random.default_rng(5)
    E, k = 64, 8
    logits = rng.normal(0, 1, E).astype(np.float32)
    remap = np.full(E, O.SKIP, np.uint32)
    pmap = np.full(E, O.SKIP, np.uint32)
    hot = rng.choice(E, 20, replace=False)
    remap[np.sort(hot)] = np.arange(20, dtype=np.uint32)
    pm = rng.choice(E, 10, replace=False)
    pmap[pm] = 3 * k + np.arange(10, dtype=np.uint32) % k
    ew, eids = O.topk_softmax(logits, k, True, remap, pmap)
    w, ids = ops.topk_softmax(T(logits), k, True, T(remap.view(np.int32)), T(pmap.view(np.int32)))
    assert np.array_equal(id_rows(ids.cpu().numpy(), k), id_rows(eids, k))


def test_moe_reduce_bit_exact():
    rng = np.random.default_rng(9)
    H, k = 2048, 8
    d = rng.normal(0, 1, k * H).astype(np.float32)
    w = rng.random(k).astype(np.float32)
    x = rng.normal(0, 1, H).astype(np.float32)
    exp = O.moe_reduce(d, w, x)
    got = ops.moe_reduce(T(d), T(w), T(x)).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_gather_slabs_from_pinned_host():
    """gather_slabs_f32.comp with the sources in pinned host memory (GTT)."""
    rng = np.random.default_rng(11)
    E, k, layer = 10, 4, 3
    sb = [1024, 2048, 1536]
    db = [2048, 2048, 2048]
    srcs_np = [rng.integers(0, 256, E * b, dtype=np.uint8) for b in sb]
    hbufs = [ops.HostBuffer(s.size) for s in srcs_np]
    for hb, s in zip(hbufs, srcs_np):
        hb.tensor.copy_(torch.from_numpy(s))
    srcs = [hb.tensor for hb in hbufs]
    arenas = [torch.zeros((layer + 1) * k * b, dtype=torch.uint8, device=DEV) for b in db]
    ids = np.array([7, -1, 2, 9], np.int32)
    ops.gather_slabs(srcs, sb, arenas, db, T(ids), layer, k)
    exp = [np.zeros((layer + 1) * k * b, np.uint8) for b in db]
    O.gather_slabs(srcs_np, sb, exp, db, ids, layer, k)
    for a, e in zip(arenas, exp):
        assert np.array_equal(a.cpu().numpy(), e)
    # async (copy-engine) form with host ids, same result
    arenas2 = [torch.zeros_like(a) for a in arenas]
    ops.gather_slabs_async(srcs, sb, arenas2, db, ids.tolist(), layer, k,
                           stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    for a, e in zip(arenas2, exp):
        assert np.array_equal(a.cpu().numpy(), e)


def test_synth_quant_matches_oracle_quantizer():
    """The device generator's quantiser reproduces the oracle's bytes."""
    for qt, ncols in ((_lib.Q4_K, 512), (_lib.Q5_K, 256), (_lib.Q6_K, 768), (_lib.Q8_0, 128)):
        nrows = 24
        vals = ops.synth_f32(nrows * ncols, 1234 + qt, 0, 0.02).cpu().numpy().reshape(nrows, ncols)
        exp = O.quantize(qt, vals).reshape(-1)
        got = ops.synth_quant(qt, nrows, ncols, 1234 + qt, 0.02).cpu().numpy()
        assert np.array_equal(got, exp), qt
        assert 0.015 < vals.std() < 0.025


# ------------------------------------------------------------ MoE block
def _upload_layer(c, remap=None, pmap=None, hot=None, arena=None):
    sg, su, sd = c.slabs
    lw = ops.LayerWeights(
        ffn_norm=T(c.norm), router=T(c.router),
        gate=ops.Experts(c.qts[0], T(c.gate), sg), up=ops.Experts(c.qts[1], T(c.up), su),
        down=ops.Experts(c.qts[2], T(c.down), sd),
        remap=None if remap is None else T(remap.view(np.int32)),
        pmap=None if pmap is None else T(pmap.view(np.int32)))
    return lw


def _run_block(c, lw, layer=0, nlayers=1, mode=_lib.MOE_AUTO):
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    blk.ctx.set_moe_kernels(mode)
    try:
        x = T(c.x)
        ids = torch.full((nlayers * 64,), -7, dtype=torch.int32, device=DEV)
        w = torch.zeros(c.k, dtype=torch.float32, device=DEV)
        blk.forward(x, lw, layer, ids, weights_out=w)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        blk.path = blk.ctx.last_moe_path()
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)
    return blk, x.cpu().numpy(), ids.cpu().numpy()[layer * 64:(layer + 1) * 64], w.cpu().numpy()


CASES = [
    ("cfg1-q8_0", 1, 512, 256, 32, 4, (_lib.Q8_0, _lib.Q8_0, _lib.Q8_0)),
    ("cfg2-shape-E16", 2, 2048, 768, 16, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
    ("q5K-q5K-q5K", 3, 1024, 512, 24, 6, (_lib.Q5_K, _lib.Q5_K, _lib.Q5_K)),
    ("q6K-gateup-q4K-down", 4, 1024, 256, 12, 3, (_lib.Q6_K, _lib.Q6_K, _lib.Q4_K)),
    ("mixed-gate-up", 5, 512, 256, 8, 2, (_lib.Q4_K, _lib.Q5_K, _lib.Q8_0)),
    ("k16", 6, 512, 256, 32, 16, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
    ("cfg5-shape-E6", 7, 4096, 1536, 6, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q4_K)),
]


# shapes the cluster form and the single cooperative kernel take (the others
# run three kernels)
FUSED_OK = {"cfg1-q8_0", "cfg2-shape-E16", "q5K-q5K-q5K", "k16"}
MODES = [_lib.MOE_AUTO, _lib.MOE_FUSED, _lib.MOE_SPLIT]
MODE_IDS = ["auto", "fused", "split"]


def want_path(mode, fits=True):
    """The LAST_PATH values a block call may report: auto takes the cluster
    form (6) where the device holds its k clusters at once, else the single
    kernel (1); the single kernel when asked for; three kernels (2) for the
    shapes neither takes."""
    if mode == _lib.MOE_SPLIT or not fits:
        return {2}
    return {1, 6} if mode == _lib.MOE_AUTO else {1}


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
@pytest.mark.parametrize("name,seed,H,F,E,k,qts", CASES, ids=[c[0] for c in CASES])
def test_moe_block_matches_oracle(name, seed, H, F, E, k, qts, mode):
    if mode == _lib.MOE_FUSED and name not in FUSED_OK:
        pytest.skip("the single kernel does not take this shape")
    c = make_case(seed, H, F, E, k, qts)
    ref = oracle_block(c)
    lw = _upload_layer(c)
    blk, x, ids, w = _run_block(c, lw, mode=mode)
    assert blk.path in want_path(mode, name in FUSED_OK), blk.path
    # routing: ids bit-exact when the top-k margin exceeds 1e-4
    logits = blk.view(1, E).cpu().numpy()
    assert rel_to_max(logits, ref["logits"]) < 1e-5
    if topk_margin(ref["logits"], k) > 1e-4:
        assert np.array_equal(id_rows(ids, k), id_rows(ref["ids64"], k))
    np.testing.assert_allclose(w, ref["weights"], rtol=1e-5, atol=1e-7)
    xn = blk.view(0, H).cpu().numpy()
    assert rel_to_max(xn, ref["xnorm"]) < 1e-5
    h = blk.view(2, k * F).cpu().numpy()
    assert rel_to_max(h, ref["h"]) < 1e-4
    # hidden state: 1e-3 relative (north star); achieved is far tighter
    dx = x - c.x
    dref = ref["x"] - c.x
    assert rel_to_max(x, ref["x"]) < 1e-3
    assert rel_to_max(dx, dref) < 1e-4


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
def test_moe_block_layer_chain_reuses_workspace(mode):
    """Three layers chained through one workspace, twice: the cross-CTA
    counters reset themselves and every layer matches the oracle chain."""
    cases = [make_case(40 + i, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for i in range(3)]
    lws = [_upload_layer(c) for c in cases]
    blk = ops.MoeBlock(ops.Dims(1024, 512, 32, 8), 0)
    blk.ctx.set_moe_kernels(mode)
    try:
        for rep in range(2):
            x = T(cases[0].x)
            ids = torch.zeros(3 * 64, dtype=torch.int32, device=DEV)
            xr = cases[0].x.copy()
            for layer, (c, lw) in enumerate(zip(cases, lws)):
                blk.forward(x, lw, layer, ids)
                c2 = make_case(40 + layer, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
                c2.x = xr
                xr = oracle_block(c2)["x"]
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            assert rel_to_max(x.cpu().numpy(), xr) < 1e-4
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
def test_moe_block_placement_is_invariant(mode):
    """Placement changes speed, never results (README.md:29-30): the same
    layer with experts split over a hot buffer, an arena and the full
    tensor gives bit-identical output."""
    c = make_case(21, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    ref = oracle_block(c)
    _, x_full, ids_full, _ = _run_block(c, _upload_layer(c), mode=mode)
    sel = ref["ids64"][:c.k]
    E = c.E
    hot_e = np.sort(np.concatenate([sel[:3], [e for e in range(E) if e not in sel][:5]]))
    remap = np.full(E, O.SKIP, np.uint32)
    remap[hot_e] = np.arange(len(hot_e), dtype=np.uint32)
    layer, k = 2, c.k
    pm_e = sel[3:6]
    pmap = np.full(E, O.SKIP, np.uint32)
    pmap[pm_e] = layer * k + np.arange(3, dtype=np.uint32)
    lw = _upload_layer(c, remap, pmap)
    sg, su, sd = c.slabs
    arena_slab = [sg + 256, su + 256, sd + 512]
    for t, (ex, slab, aslab, src) in enumerate(zip((lw.gate, lw.up, lw.down), (sg, su, sd), arena_slab,
                                                   (c.gate, c.up, c.down))):
        hb = np.concatenate([src[e * slab:(e + 1) * slab] for e in hot_e])
        ex.hot = T(hb)
        ar = np.zeros((layer + 1) * k * aslab, np.uint8)
        for j, e in enumerate(pm_e):
            slot = layer * k + j
            ar[slot * aslab: slot * aslab + slab] = src[e * slab:(e + 1) * slab]
        ex.arena = T(ar)
        ex.arena_slab_bytes = aslab
        # poison the full tensor where hot / arena experts live: must not be read
        full = src.copy()
        for e in list(hot_e) + list(pm_e):
            full[e * slab:(e + 1) * slab] = 0x5A
        ex.full = T(full)
    _, x_pl, ids_pl, _ = _run_block(c, lw, layer=layer, nlayers=layer + 1, mode=mode)
    assert np.array_equal(ids_pl[:k], ids_full[:k])
    assert (ids_pl[16:16 + k] != -1).sum() + (ids_pl[32:32 + k] != -1).sum() + (ids_pl[48:48 + k] != -1).sum() == k
    assert np.array_equal(x_pl.view(np.uint32), x_full.view(np.uint32))


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
@pytest.mark.parametrize("H,F,E,top,second", [
    (1024, 512, 32, [29, 3, 17, 4], [30, 11]),
    (256, 256, 512, [300, 7, 511, 149], [450, 148]),   # E > SM count: several router rows per CTA
], ids=["E32", "E512"])
def test_moe_block_routing_ties(mode, H, F, E, top, second):
    """Exactly equal logits (duplicated router rows) are taken lowest index
    first, as the reference's serial scan with strict '>' does
    (topk_softmax_f32.comp:39-46); the single-kernel block picks on one warp
    with reductions, the three-kernel block with the standalone top-k."""
    c = make_case(31, H, F, E, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    xn = O.rms_norm(c.x, c.norm, c.eps)
    base = (0.05 * np.sign(xn)).astype(np.float32)
    c.router[top] = base
    c.router[second] = 0.5 * base
    ref = oracle_block(c)
    assert list(ref["ids64"][:6]) == sorted(top) + sorted(second)
    blk, x, ids, w = _run_block(c, _upload_layer(c), mode=mode)
    assert blk.path in want_path(mode)
    logits = blk.view(1, E).cpu().numpy()
    assert np.all(logits[top] == logits[top[0]]) and np.all(logits[second] == logits[second[0]])
    assert np.array_equal(id_rows(ids, c.k), id_rows(ref["ids64"], c.k))
    np.testing.assert_allclose(w, ref["weights"], rtol=1e-5, atol=1e-7)
    assert rel_to_max(x, ref["x"]) < 1e-3


def test_moe_block_full_size_cfg2_spot_check():
    """All 128 experts of a 30B-A3B-shaped layer generated on the device;
    the selected slabs are brought back and the oracle recomputes the block."""
    H, F, E, k = 2048, 768, 128, 8
    sg = O.row_bytes(_lib.Q4_K, H) * F
    sd = O.row_bytes(_lib.Q6_K, F) * H
    gate = ops.synth_quant(_lib.Q4_K, E * F, H, 101, 0.02)
    up = ops.synth_quant(_lib.Q4_K, E * F, H, 102, 0.02)
    down = ops.synth_quant(_lib.Q6_K, E * H, F, 103, 0.02)
    rng = np.random.default_rng(104)
    router = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    norm = np.ones(H, np.float32)
    x0 = rng.normal(0, 1, H).astype(np.float32)
    lw = ops.LayerWeights(T(norm), T(router), ops.Experts(_lib.Q4_K, gate, sg),
                          ops.Experts(_lib.Q4_K, up, sg), ops.Experts(_lib.Q6_K, down, sd))
    blk = ops.MoeBlock(ops.Dims(H, F, E, k), 0)
    x = T(x0)
    ids = torch.zeros(64, dtype=torch.int32, device=DEV)
    blk.forward(x, lw, 0, ids)
    torch.cuda.synchronize()
    sel = ids[:k].cpu().numpy()
    # oracle on a compacted copy holding only the selected experts
    g = np.concatenate([gate[e * sg:(e + 1) * sg].cpu().numpy() for e in sel])
    u = np.concatenate([up[e * sg:(e + 1) * sg].cpu().numpy() for e in sel])
    d = np.concatenate([down[e * sd:(e + 1) * sd].cpu().numpy() for e in sel])
    xn = O.rms_norm(x0, norm, 1e-6)
    lg = O.matvec_strided_f32(router, xn)
    ew, eids = O.topk_softmax(lg, k, True)
    if topk_margin(lg, k) > 1e-4:
        assert np.array_equal(sel, eids[:k])
    local = np.arange(k, dtype=np.int32)
    gg = O.mul_mat_vec_id(_lib.Q4_K, g, sg, F, H, local, xn, 1)
    uu = O.mul_mat_vec_id(_lib.Q4_K, u, sg, F, H, local, xn, 1)
    hh = O.swiglu(gg, uu)
    dd = O.mul_mat_vec_id(_lib.Q6_K, d, sd, H, F, local, hh, k)
    xr = O.moe_reduce(dd, ew, x0)
    xg = x.cpu().numpy()
    assert rel_to_max(xg - x0, xr - x0) < 1e-4
    assert rel_to_max(xg, xr) < 1e-3


def test_device_error_word_is_clear():
    ops.ctx(0).check_device_error()
