"""Expert-parallel MoE block on one device with emulated ranks: rank r holds
only the experts e with e % R == r (a dense hot buffer, remap -> local slot,
no full tensor), styx_moe_block_ep writes its slot contributions, the
partials are summed as an all-reduce would, and styx_moe_combine must give
the single-device styx_moe_block bit for bit, in both kernel forms: the
single kernel (its partial-output epilogue; the H 1024 shape) and three
kernels (the H 1024 shape, and the 235B-like shape that runs gate/up as
mul_mat_vec_id dispatches, H 4096, which the single kernel does not take).
"""
import numpy as np
import pytest
import torch

from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _full_layer(c):
    sg, su, sd = c.slabs
    return ops.LayerWeights(
        ffn_norm=_t(c.norm), router=_t(c.router),
        gate=ops.Experts(c.qts[0], _t(c.gate), sg), up=ops.Experts(c.qts[1], _t(c.up), su),
        down=ops.Experts(c.qts[2], _t(c.down), sd))


def _rank_layer(c, owned):
    """This rank's weights: only its experts, densely, ascending id order."""
    sg, su, sd = c.slabs
    remap = np.full(c.E, -1, np.int32)
    remap[owned] = np.arange(len(owned), dtype=np.int32)

    def ex(qt, src, slab):
        hot = np.concatenate([src[e * slab:(e + 1) * slab] for e in owned])
        return ops.Experts(qt, None, slab, hot=_t(hot))
    return ops.LayerWeights(ffn_norm=_t(c.norm), router=_t(c.router), gate=ex(c.qts[0], c.gate, sg),
                            up=ex(c.qts[1], c.up, su), down=ex(c.qts[2], c.down, sd), remap=_t(remap))


@pytest.mark.parametrize("shape", [(1024, 512, 16, 6, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
                                   (4096, 1536, 8, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q4_K))],
                         ids=["gate_up-kernel", "235B-like"])
@pytest.mark.parametrize("R", [2, 3])
@pytest.mark.parametrize("mode", [_lib.MOE_SPLIT, _lib.MOE_FUSED, _lib.MOE_AUTO],
                         ids=["three-kernel", "single-kernel", "auto"])
def test_ep_ranks_sum_to_single_device(shape, R, mode):
    H, F, E, k, qts = shape
    if mode == _lib.MOE_FUSED and H != 1024:
        pytest.skip("the single kernel does not take this shape")
    c = make_case(51, H, F, E, k, qts)
    ref = oracle_block(c)
    blk = ops.MoeBlock(ops.Dims(H, F, E, k), 0)
    blk.ctx.set_moe_kernels(mode)
    want_path = {2} if (mode == _lib.MOE_SPLIT or H != 1024) else ({1, 6} if mode == _lib.MOE_AUTO else {1})
    try:
        x1 = _t(c.x)
        ids1 = torch.full((64,), -7, dtype=torch.int32, device=DEV)
        blk.forward(x1, _full_layer(c), 0, ids1)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        assert blk.ctx.last_moe_path() in want_path
        total = torch.zeros(k * H, dtype=torch.float32, device=DEV)
        for r in range(R):
            owned = [e for e in range(E) if e % R == r]
            lw = _rank_layer(c, owned)
            xr = _t(c.x)
            ids = torch.full((64,), -7, dtype=torch.int32, device=DEV)
            w = torch.zeros(k, dtype=torch.float32, device=DEV)
            partial = torch.full((k * H,), 7.0, dtype=torch.float32, device=DEV)
            blk.forward_ep(xr, lw, 0, ids, partial, weights_out=w)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()           # experts held elsewhere are not errors
            assert blk.ctx.last_moe_path() in want_path
            assert torch.equal(xr, _t(c.x))          # x is read, not updated
            assert torch.equal(ids[:k], ids1[:k])    # every rank routes the same
            p = partial.view(k, H).cpu().numpy()
            sel = ids[:k].cpu().numpy()
            for s in range(k):
                if sel[s] % R != r:
                    assert not p[s].any(), f"rank {r} slot {s}: expert held elsewhere must contribute 0"
            total += partial                          # the all-reduce (one non-zero per slot: exact)
        x_ep = _t(c.x)
        blk.combine(total, x_ep)
        torch.cuda.synchronize()
        a, b = x_ep.cpu().numpy(), x1.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.max(np.abs(a - ref["x"])) <= 1e-3 * np.max(np.abs(ref["x"]))
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)
