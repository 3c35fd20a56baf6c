"""The cluster form of the MoE block (one thread-block cluster per selected
slot) against the single cooperative kernel: both forms run the same
arithmetic (reduction trees, digit vectors, dot products, slot-ordered
combine), so every output is bit-identical; and against the oracle through
the block matrix in test_gpu_parity.py."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block, topk_margin

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


def _layer(c, remap=None):
    sg, su, sd = c.slabs
    return ops.LayerWeights(
        ffn_norm=T(c.norm), router=T(c.router),
        gate=ops.Experts(c.qts[0], T(c.gate), sg), up=ops.Experts(c.qts[1], T(c.up), su),
        down=ops.Experts(c.qts[2], T(c.down), sd),
        remap=None if remap is None else T(remap.view(np.int32)))


def _run(blk, c, lw, mode, reps=1):
    blk.ctx.set_moe_kernels(mode)
    try:
        outs = []
        for _ in range(reps):
            x = T(c.x)
            ids = torch.full((64,), -7, dtype=torch.int32, device=DEV)
            w = torch.zeros(c.k, dtype=torch.float32, device=DEV)
            blk.forward(x, lw, 0, ids, weights_out=w)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            outs.append(dict(path=blk.ctx.last_moe_path(), x=x.cpu().numpy(), ids=ids.cpu().numpy(),
                             w=w.cpu().numpy(), logits=blk.view(1, c.E).cpu().numpy().copy(),
                             xnorm=blk.view(0, c.H).cpu().numpy().copy(),
                             h=blk.view(2, c.k * c.F).cpu().numpy().copy()))
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)
    return outs


SHAPES = [
    ("cfg2-E128", 61, 2048, 768, 128, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
    ("cfg1-q8_0", 62, 512, 256, 32, 4, (_lib.Q8_0, _lib.Q8_0, _lib.Q8_0)),
    ("q5K", 63, 1024, 512, 24, 6, (_lib.Q5_K, _lib.Q5_K, _lib.Q5_K)),
    ("k16-C8", 64, 512, 256, 32, 16, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
    ("q6K-q6K", 65, 1024, 256, 40, 8, (_lib.Q6_K, _lib.Q6_K, _lib.Q6_K)),
]


@pytest.mark.parametrize("name,seed,H,F,E,k,qts", SHAPES, ids=[s[0] for s in SHAPES])
def test_cluster_form_is_bit_identical_to_single_kernel(name, seed, H, F, E, k, qts):
    c = make_case(seed, H, F, E, k, qts)
    lw = _layer(c)
    blk = ops.MoeBlock(ops.Dims(H, F, E, k), 0)
    cl = _run(blk, c, lw, _lib.MOE_CLUSTER, reps=3)   # three launches on one workspace
    fu = _run(blk, c, lw, _lib.MOE_FUSED)[0]
    assert fu["path"] == 1
    for o in cl:
        assert o["path"] == 6
        for key in ("x", "w", "logits", "xnorm", "h"):
            assert np.array_equal(o[key].view(np.uint32), fu[key].view(np.uint32)), key
        for base in (0, 16, 32, 48):
            assert np.array_equal(o["ids"][base:base + k], fu["ids"][base:base + k])
    ref = oracle_block(c)
    if topk_margin(ref["logits"], k) > 1e-4:
        assert np.array_equal(cl[0]["ids"][:k], ref["ids64"][:k])
    assert rel_to_max(cl[0]["x"], ref["x"]) < 1e-3
    assert rel_to_max(cl[0]["x"] - c.x, ref["x"] - c.x) < 1e-4


def test_cluster_form_full_router_with_hot_experts():
    """The 30B-A3B router shape (128 experts, 8 router rows per CTA) with some
    selected experts in a hot buffer: the same bits as all-full placement."""
    c = make_case(66, 2048, 768, 128, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    sel = oracle_block(c)["ids64"][:c.k]
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    full = _run(blk, c, _layer(c), _lib.MOE_CLUSTER)[0]
    hot_e = np.sort(sel[::2])
    remap = np.full(c.E, O.SKIP, np.uint32)
    remap[hot_e] = np.arange(len(hot_e), dtype=np.uint32)
    lw = _layer(c, remap)
    for ex, src, slab in zip((lw.gate, lw.up, lw.down), (c.gate, c.up, c.down), c.slabs):
        ex.hot = T(np.concatenate([src[e * slab:(e + 1) * slab] for e in hot_e]))
        poisoned = src.copy()
        for e in hot_e:
            poisoned[e * slab:(e + 1) * slab] = 0x5A   # must not be read
        ex.full = T(poisoned)
    hot = _run(blk, c, lw, _lib.MOE_CLUSTER)[0]
    assert hot["path"] == 6
    assert np.array_equal(hot["x"].view(np.uint32), full["x"].view(np.uint32))
    assert np.array_equal(hot["ids"][:c.k], full["ids"][:c.k])
    assert (hot["ids"][16:16 + c.k] >= 0).sum() == len(hot_e)


def test_cluster_form_trace_stamps():
    """STYX_OPT_TRACE: every CTA of the k clusters records its phase stamps
    in order."""
    c = make_case(67, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    blk.ctx.set_option(_lib.OPT_TRACE, 1)
    try:
        out = _run(blk, c, _layer(c), _lib.MOE_CLUSTER)[0]
        st = blk.view(4, 256 * 32 * 2).view(torch.int64).cpu().numpy().reshape(256, 32)
    finally:
        blk.ctx.set_option(_lib.OPT_TRACE, 0)
    assert out["path"] == 6
    C = blk.ctx.get_option(_lib.OPT_MOE_LAST_CLUSTER)
    assert C in (1, 2, 4, 8, 16)
    ctas = c.k * C
    d = np.diff(st[:ctas, :13].astype(np.int64), axis=1)
    assert (st[:ctas, :13] != 0).all() and (d >= 0).all()
