"""Residency decisions applied on the device.  Popularity pinning builds the
hot buffers from the full tensors with styx_copy (as MoeModel::load copies
hot slabs densely, moe.rs:836-858), a repin rewrites hot slots and the remap
table (Residency.apply_swaps, moe.rs:1482-1504), and the MoE block's output
stays bit-identical to the all-full placement: placement changes speed,
never results.
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


def _layer(c):
    sg, su, sd = c.slabs
    return ops.LayerWeights(
        ffn_norm=_t(c.norm), router=_t(c.router),
        gate=ops.Experts(c.qts[0], _t(c.gate), sg), up=ops.Experts(c.qts[1], _t(c.up), su),
        down=ops.Experts(c.qts[2], _t(c.down), sd))


def _run(c, lw, mode):
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    blk.ctx.set_moe_kernels(mode)
    try:
        x = _t(c.x)
        ids = torch.full((64,), -7, dtype=torch.int32, device=DEV)
        blk.forward(x, lw, 0, ids)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)
    return x.cpu().numpy(), ids.cpu().numpy()


def _build_hot(res, lw):
    """Dense hot buffers of layer 0's pinned experts, copied from the full
    tensors on the device, and the device remap table."""
    import ctypes as C
    remap, slots = res.layer(0)
    cx = ops.ctx(0).handle
    for ex in (lw.gate, lw.up, lw.down):
        ex.hot = torch.empty(max(len(slots), 1) * ex.slab_bytes, dtype=torch.uint8, device=DEV)
        for s, e in enumerate(slots):
            _lib.check(_lib.lib().styx_copy(cx, C.c_void_p(ex.full.data_ptr()), int(e) * ex.slab_bytes,
                                            C.c_void_p(ex.hot.data_ptr()), s * ex.slab_bytes, ex.slab_bytes,
                                            None))
    lw.remap = _t(remap.view(np.int32))
    torch.cuda.synchronize()
    return slots


@pytest.mark.parametrize("mode", [_lib.MOE_AUTO, _lib.MOE_SPLIT], ids=["auto", "split"])
def test_pinning_and_repin_keep_results(mode):
    c = make_case(31, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    sel = oracle_block(c)["ids64"][:c.k]
    x_full, ids_full = _run(c, _layer(c), mode)
    assert np.array_equal(ids_full[:c.k], sel)

    sg, su, sd = c.slabs
    res = ops.Residency(1, c.E, c.k, sg + su + sd)
    # histogram: half of the selected experts and six unselected ones are hot
    unsel = [e for e in range(c.E) if e not in sel][:6]
    hot_e = list(sel[: c.k // 2]) + unsel
    n = res.pin([0] * len(hot_e), hot_e, [10] * len(hot_e), len(hot_e) * (sg + su + sd))
    assert n == len(hot_e)
    lw = _layer(c)
    slots = _build_hot(res, lw)
    x_pin, ids_pin = _run(c, lw, mode)
    assert np.array_equal(x_pin.view(np.uint32), x_full.view(np.uint32))
    hot_rows = ids_pin[16:16 + c.k]
    assert (hot_rows != -1).sum() == c.k // 2          # the pinned half reads the hot buffer
    hot, cold = res.hot_cold(np.pad(ids_pin, (0, 0)))
    assert hot[0] == c.k // 2 and cold[0] == c.k - c.k // 2

    # two tokens with the same routing: the cold selected experts reach 2 hits
    # against 0 for the unselected residents, so a repin at n_past = 2 swaps
    # them in (at most 2 per layer)
    ids_host = ids_pin.copy()
    assert res.maybe_repin(ids_host, 1, 2, 2) == []
    swaps = res.maybe_repin(ids_host, 2, 2, 2)
    assert len(swaps) == 2
    assert all(old in unsel and new in sel for (_, _, old, new) in swaps)
    res.apply_swaps(swaps, [lw], [lw.remap])
    _, slots_after = res.layer(0)
    for ex in (lw.gate, lw.up, lw.down):
        hb = ex.hot.cpu().numpy()
        full = ex.full.cpu().numpy()
        for s, e in enumerate(slots_after):
            assert np.array_equal(hb[s * ex.slab_bytes:(s + 1) * ex.slab_bytes],
                                  full[int(e) * ex.slab_bytes:(int(e) + 1) * ex.slab_bytes])
    x_rep, ids_rep = _run(c, lw, mode)
    assert np.array_equal(x_rep.view(np.uint32), x_full.view(np.uint32))
    assert (ids_rep[16:16 + c.k] != -1).sum() == c.k // 2 + 2
    assert len(slots) == len(slots_after)
