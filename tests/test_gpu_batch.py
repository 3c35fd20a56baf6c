"""styx_moe_block_batch (a batch of decode tokens through one MoE layer, the
experts' matrices as grouped GEMMs on the tensor cores) against the oracle
run token by token (the reference's block, moe.rs:1974-2062): routing ids
bit-exact wherever the top-k margin exceeds 1e-4, weights within 1e-5, and
each token's update dx within 1e-3 of max|dx| (the operands are rounded to
f16); at batch 1, 8 and 64 and at the 30B and 235B-like shapes.  The result
must not depend on where an expert lives (hot buffer, or full tensor).
q8_0 is rejected by this path (its kernel stays off the GPU)."""
import dataclasses

import numpy as np
import pytest
import torch

from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block, topk_margin

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
CASES = [
    ("30B-shape-E32", 11, 2048, 768, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
    ("H1024-q5K", 12, 1024, 512, 16, 6, (_lib.Q5_K, _lib.Q5_K, _lib.Q5_K)),
    ("235B-like-E6", 14, 4096, 1536, 6, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q4_K)),
]


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _layer(c, remap=None, hot_experts=None):
    sg, su, sd = c.slabs
    if hot_experts is None:
        return ops.LayerWeights(T(c.norm), T(c.router), ops.Experts(c.qts[0], T(c.gate), sg),
                                ops.Experts(c.qts[1], T(c.up), su), ops.Experts(c.qts[2], T(c.down), sd))

    def ex(qt, src, slab):
        hot = np.concatenate([src[e * slab:(e + 1) * slab] for e in hot_experts])
        return ops.Experts(qt, T(src), slab, hot=T(hot))
    return ops.LayerWeights(T(c.norm), T(c.router), ex(c.qts[0], c.gate, sg), ex(c.qts[1], c.up, su),
                            ex(c.qts[2], c.down, sd), remap=T(remap))


def _run(c, lw, xs):
    B = xs.shape[0]
    blk = ops.MoeBatch(ops.Dims(c.H, c.F, c.E, c.k), B)
    x = T(xs)
    ids = torch.full((B * 64,), -7, dtype=torch.int32, device=DEV)
    w = torch.zeros(B * c.k, dtype=torch.float32, device=DEV)
    blk.forward(x, lw, ids, w)
    torch.cuda.synchronize()
    blk.ctx.check_device_error()
    return x.cpu().numpy(), ids.cpu().numpy().reshape(B, 64), w.cpu().numpy().reshape(B, c.k)


@pytest.mark.parametrize("B", [1, 8, 64])
@pytest.mark.parametrize("name,seed,H,F,E,k,qts", CASES, ids=[c[0] for c in CASES])
def test_batch_matches_the_oracle_token_by_token(name, seed, H, F, E, k, qts, B):
    c = make_case(seed, H, F, E, k, qts)
    xs = np.random.default_rng(seed + B).normal(0, 1, (B, H)).astype(np.float32)
    x, ids, w = _run(c, _layer(c), xs)
    for b in range(B):
        ref = oracle_block(dataclasses.replace(c, x=xs[b]))
        if topk_margin(ref["logits"], k) > 1e-4:
            assert np.array_equal(ids[b, :k], ref["ids64"][:k]), b
            np.testing.assert_allclose(w[b], ref["weights"], rtol=1e-5, atol=1e-7)
        dx, dref = x[b] - xs[b], ref["x"] - xs[b]
        assert np.max(np.abs(dx - dref)) <= 1e-3 * np.max(np.abs(dref)), b


def test_batch_placement_and_repeat_are_bit_identical():
    """Hot-buffer placement of half the experts, and a second run, give the
    same bits as the first run from the full tensors."""
    c = make_case(21, 1024, 512, 16, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    xs = np.random.default_rng(5).normal(0, 1, (16, c.H)).astype(np.float32)
    x1, ids1, _ = _run(c, _layer(c), xs)
    x2, _, _ = _run(c, _layer(c), xs)
    hot_e = list(range(0, c.E, 2))
    remap = np.full(c.E, -1, np.int32)
    remap[hot_e] = np.arange(len(hot_e), dtype=np.int32)
    x3, ids3, _ = _run(c, _layer(c, remap, hot_e), xs)
    assert np.array_equal(x1.view(np.uint32), x2.view(np.uint32))
    assert np.array_equal(x1.view(np.uint32), x3.view(np.uint32))
    assert np.array_equal(ids1[:, :8], ids3[:, :8])


def test_batch_rejects_bad_arguments():
    c = make_case(22, 512, 256, 8, 2, (_lib.Q4_K, _lib.Q5_K, _lib.Q6_K))   # gate and up differ
    blk = ops.MoeBatch(ops.Dims(c.H, c.F, c.E, c.k), 2)
    x = torch.zeros(2 * c.H, dtype=torch.float32, device=DEV)
    with pytest.raises(_lib.StyxError):
        blk.forward(x, _layer(c), torch.zeros(128, dtype=torch.int32, device=DEV),
                    torch.zeros(4, dtype=torch.float32, device=DEV))
    c8 = make_case(23, 512, 256, 8, 2, (_lib.Q8_0, _lib.Q8_0, _lib.Q8_0))   # not a batch-path format
    blk8 = ops.MoeBatch(ops.Dims(c8.H, c8.F, c8.E, c8.k), 2)
    with pytest.raises(_lib.StyxError):
        blk8.forward(torch.zeros(2 * c8.H, dtype=torch.float32, device=DEV), _layer(c8),
                     torch.zeros(128, dtype=torch.int32, device=DEV), torch.zeros(4, dtype=torch.float32, device=DEV))
    import ctypes as C
    n = C.c_uint64()
    rc = _lib.lib().styx_moe_batch_workspace_bytes(C.byref(ops.Dims(512, 256, 8, 2).struct()), 65, C.byref(n))
    assert rc == _lib.STYX_EINVAL
