"""Failure detection without a fault: a bounded device-side wait that runs out.

The single-kernel MoE block tags each launch from the workspace's never-reset
launch counter (launch number = counter / grid size).  Setting that counter
to half a grid splits one launch's CTAs into two launch numbers, so each half
waits for logit words and h arrivals the other half never provides.  Every
such wait gives up after about a second, records its code in the device
error word and lets the kernel finish (no fault, every access in bounds);
the host then sees STYX_ETIMEOUT, and after styx_moe_workspace_init the next
call is correct again.  The same with STYX_OPT_EXCLUSIVE (a plain launch
instead of a cooperative one).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
GEN_OFFSET = 128   # byte offset of the launch counter in the workspace's counter block


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("exclusive", [0, 1], ids=["cooperative", "exclusive"])
def test_split_launch_numbers_time_out_and_recover(exclusive):
    c = make_case(81, 1024, 512, 16, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    sg, su, sd = c.slabs
    lw = ops.LayerWeights(ffn_norm=_t(c.norm), router=_t(c.router),
                          gate=ops.Experts(c.qts[0], _t(c.gate), sg), up=ops.Experts(c.qts[1], _t(c.up), su),
                          down=ops.Experts(c.qts[2], _t(c.down), sd))
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, c.E, c.k), 0)
    blk.ctx.set_moe_kernels(_lib.MOE_FUSED)
    blk.ctx.set_option(_lib.OPT_EXCLUSIVE, exclusive)
    try:
        blk.ctx.check_device_error()          # start clean
        grid = blk.ctx.sm_count
        counters = blk.workspace[GEN_OFFSET:GEN_OFFSET + 8].view(torch.int64)
        counters.fill_(grid // 2)             # half a launch: two launch numbers in one grid
        x = _t(c.x)
        ids = torch.zeros(64, dtype=torch.int32, device=DEV)
        blk.forward(x, lw, 0, ids)
        torch.cuda.synchronize()              # returns: every wait is bounded
        assert blk.ctx.last_moe_path() == 1
        with pytest.raises(_lib.StyxError) as ei:
            blk.ctx.check_device_error()
        assert ei.value.code == _lib.STYX_ETIMEOUT
        blk.ctx.check_device_error()          # the word was cleared by the read

        # recovery: re-initialise the workspace, then the block is exact again
        _lib.check(_lib.lib().styx_moe_workspace_init(blk.ctx.handle, None, C.c_void_p(blk.workspace.data_ptr()),
                                                      blk.ws_bytes))
        torch.cuda.synchronize()
        x = _t(c.x)
        ids = torch.zeros(64, dtype=torch.int32, device=DEV)
        blk.forward(x, lw, 0, ids)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        ref = oracle_block(c)
        got = x.cpu().numpy()
        assert np.array_equal(ids.cpu().numpy()[: c.k], ref["ids64"][: c.k])
        assert np.max(np.abs(got - ref["x"])) <= 1e-3 * np.max(np.abs(ref["x"]))
    finally:
        blk.ctx.set_moe_kernels(_lib.MOE_AUTO)
        blk.ctx.set_option(_lib.OPT_EXCLUSIVE, 0)
