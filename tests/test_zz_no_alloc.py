"""styx_moe_block_noalloc (static device scratch, no workspace) against
styx_moe_block with a caller workspace: the same inputs through both entry
points, two layers in a row, on both kernel forms.  The two run the same
kernels on the same data, so the tolerance is tight (1e-6 of max|x|).

Named to be collected last: it must pass alone in a fresh process and after
every other test (the scratch is set up by whichever call comes first).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from styx_b200 import _lib, ops
from tests.moe_case import make_case

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


def _noalloc(ctx, dims, lw_struct, layer, x, ids, w):
    _lib.check(_lib.lib().styx_moe_block_noalloc(ctx.handle, None, C.byref(dims), C.byref(lw_struct), layer,
                                                 x.data_ptr(), ids.data_ptr(), w.data_ptr()))


@pytest.mark.parametrize("mode,path", [(_lib.MOE_AUTO, (1, 6)), (_lib.MOE_FUSED, (1,)), (_lib.MOE_CLUSTER, (6,)),
                                       (_lib.MOE_SPLIT, (2,))], ids=["auto", "single-kernel", "cluster", "split"])
def test_noalloc_matches_workspace_entry(mode, path):
    c = make_case(21, 2048, 768, 16, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    lw = _layer(c)
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    st = lw.struct()
    x_ws, x_na = _t(c.x), _t(c.x)
    ids_ws = torch.full((2 * 64,), -7, dtype=torch.int32, device=DEV)
    ids_na = ids_ws.clone()
    w_ws = torch.zeros(c.k, dtype=torch.float32, device=DEV)
    w_na = torch.zeros_like(w_ws)
    blk.ctx.set_moe_kernels(mode)
    try:
        for layer in (0, 1):
            blk.forward(x_ws, lw, layer, ids_ws, weights_out=w_ws)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            _noalloc(blk.ctx, blk._dims, st, layer, x_na, ids_na, w_na)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            assert blk.ctx.last_moe_path() in path
            a, b = x_ws.cpu().numpy(), x_na.cpu().numpy()
            assert np.all(np.isfinite(b))
            assert np.max(np.abs(a - b)) <= 1e-6 * np.max(np.abs(a)), f"layer {layer}"
            np.testing.assert_array_equal(ids_ws.cpu().numpy()[: (layer + 1) * 64],
                                          ids_na.cpu().numpy()[: (layer + 1) * 64])
            np.testing.assert_allclose(w_na.cpu().numpy(), w_ws.cpu().numpy(), rtol=1e-6, atol=0)
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)


def test_noalloc_alternating_dims_match_fresh_workspaces():
    """Two shapes (other F, k and E) in turn through the one shared scratch:
    each call clears the words an earlier call with other dims left behind,
    so every result equals styx_moe_block on that shape's own workspace."""
    cases = [make_case(31, 2048, 768, 16, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
             make_case(32, 1024, 512, 32, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))]
    lws = [_layer(c) for c in cases]
    blks = [ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0) for c in cases]
    for turn in range(4):
        i = turn % 2
        c, lw, blk = cases[i], lws[i], blks[i]
        x_ws, x_na = _t(c.x), _t(c.x)
        ids_ws = torch.full((64,), -7, dtype=torch.int32, device=DEV)
        ids_na = ids_ws.clone()
        w_ws = torch.zeros(c.k, dtype=torch.float32, device=DEV)
        w_na = torch.zeros_like(w_ws)
        blk.forward(x_ws, lw, 0, ids_ws, weights_out=w_ws)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        _noalloc(blk.ctx, blk._dims, lw.struct(), 0, x_na, ids_na, w_na)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        a, b = x_ws.cpu().numpy(), x_na.cpu().numpy()
        assert np.all(np.isfinite(b))
        assert np.max(np.abs(a - b)) <= 1e-6 * np.max(np.abs(a)), f"turn {turn}"
        np.testing.assert_array_equal(ids_ws.cpu().numpy(), ids_na.cpu().numpy())


def test_noalloc_rejects_dims_above_its_scratch():
    dims = ops.Dims(16384, 2048, 64, 16).struct()
    need = C.c_uint64()
    _lib.check(_lib.lib().styx_moe_workspace_bytes(C.byref(dims), C.byref(need)))
    assert need.value > 512 * 1024
    ctx = ops.ctx(0)
    rc = _lib.lib().styx_moe_block_noalloc(ctx.handle, None, C.byref(dims), C.byref(_lib.MoeLayer()), 0,
                                           None, None, None)
    assert rc == _lib.STYX_EINVAL
    assert b"scratch" in _lib.lib().styx_last_error()
