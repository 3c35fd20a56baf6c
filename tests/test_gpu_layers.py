"""styx_moe_blocks: consecutive layers of one token with x passed between
them as tagged words -- up to 80 layers in one persistent launch
(STYX_OPT_MOE_LAYERS 1) or one chained launch per layer (2: a layer's CTAs
start without waiting for the previous grid) -- must give exactly what one
styx_moe_block call per layer gives (0, the default), layer after layer.
"""
import dataclasses

import numpy as np
import pytest
import torch

from styx_b200 import _lib, ops
from tests.moe_case import make_case, oracle_block

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
GEN_OFFSET = 128
SEPARATE, PERSISTENT, CHAIN = 0, 1, 2
PATH = {CHAIN: 5, PERSISTENT: 4, SEPARATE: 1}


def path_ok(mode, got):
    """One call per layer takes the cluster form (6) where the device holds
    its k clusters at once, else the single kernel (1)."""
    return got in (1, 6) if mode == SEPARATE else got == PATH[mode]
MODES = pytest.mark.parametrize("mode", [CHAIN, PERSISTENT], ids=["chain", "persistent"])


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def upload(c):
    sg, su, sd = c.slabs
    return ops.LayerWeights(T(c.norm), T(c.router), ops.Experts(c.qts[0], T(c.gate), sg),
                            ops.Experts(c.qts[1], T(c.up), su), ops.Experts(c.qts[2], T(c.down), sd))


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


def run_both(cases, first_layer=0, reps=2, mode=PERSISTENT, exclusive=0):
    lws = [upload(c) for c in cases]
    c0 = cases[0]
    n, k = len(cases), c0.k
    dims = ops.Dims(c0.H, c0.F, c0.E, k)
    one, many = ops.MoeBlock(dims, 0), ops.MoeBlock(dims, 0)
    many.ctx.set_option(_lib.OPT_MOE_LAYERS, mode)   # (the blocks of a device share one context)
    total = first_layer + n
    try:
        return _run_both(cases, first_layer, reps, lws, c0, n, k, one, many, total, exclusive)
    finally:
        many.ctx.set_option(_lib.OPT_MOE_LAYERS, 0)
        many.ctx.set_option(_lib.OPT_EXCLUSIVE, 0)


def _run_both(cases, first_layer, reps, lws, c0, n, k, one, many, total, exclusive):
    for rep in range(reps):   # twice: the launch counter keeps counting on the same workspaces
        xa, xb = T(c0.x), T(c0.x)
        ia = torch.full((total * 64,), -7, dtype=torch.int32, device=DEV)
        ib = ia.clone()
        wa = torch.zeros(n * k, dtype=torch.float32, device=DEV)
        wb = torch.zeros_like(wa)
        many.ctx.set_option(_lib.OPT_EXCLUSIVE, 0)   # the reference: cooperative launches
        for i, lw in enumerate(lws):
            one.forward(xa, lw, first_layer + i, ia, weights_out=wa[i * k:(i + 1) * k])
        many.ctx.set_option(_lib.OPT_EXCLUSIVE, exclusive)
        many.forward_layers(xb, lws, first_layer, ib, weights_out=wb)
        torch.cuda.synchronize()
        one.ctx.check_device_error()
        assert np.array_equal(xa.cpu().numpy().view(np.uint32), xb.cpu().numpy().view(np.uint32)), rep
        assert np.array_equal(ia.cpu().numpy(), ib.cpu().numpy()), rep
        assert np.array_equal(wa.cpu().numpy().view(np.uint32), wb.cpu().numpy().view(np.uint32)), rep
    return many, xb, lws


@pytest.mark.parametrize("mode", [CHAIN, PERSISTENT, SEPARATE], ids=["chain", "persistent", "separate"])
def test_linked_layers_equal_one_call_per_layer_and_the_oracle(mode):
    cases = [make_case(90 + l, 1024, 512, 32, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(5)]
    many, x, _ = run_both(cases, first_layer=3, mode=mode)
    assert path_ok(mode, many.ctx.last_moe_path())
    xr = cases[0].x.copy()
    for c in cases:
        xr = oracle_block(dataclasses.replace(c, x=xr))["x"]
    assert rel_to_max(x.cpu().numpy(), xr) < 1e-4


@pytest.mark.parametrize("mode", [SEPARATE, PERSISTENT, CHAIN], ids=["separate", "persistent", "chain"])
def test_plain_launches_equal_cooperative_ones(mode):
    """STYX_OPT_EXCLUSIVE: the same kernels launched without the cooperative
    attribute give the same bits."""
    cases = [make_case(150 + l, 2048, 768, 128, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(3)]
    many, _, _ = run_both(cases, mode=mode, exclusive=1)
    assert path_ok(mode, many.ctx.last_moe_path())


@MODES
def test_more_layers_than_one_launch_holds(mode):
    # 83 small layers: persistent, two launches (80 + 3); chained, 83
    cases = [make_case(200 + l, 512, 256, 8, 2, (_lib.Q8_0, _lib.Q8_0, _lib.Q8_0), sigma=0.01)
             for l in range(83)]
    many, _, _ = run_both(cases, reps=1, mode=mode)
    assert path_ok(mode, many.ctx.last_moe_path())


@MODES
def test_mixed_formats(mode):
    # chained launches take any formats per layer; the persistent form
    # needs one set and falls back to one call per layer
    cases = [make_case(300, 1024, 512, 16, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)),
             make_case(301, 1024, 512, 16, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q4_K)),
             make_case(302, 1024, 512, 16, 4, (_lib.Q5_K, _lib.Q5_K, _lib.Q5_K))]
    many, _, _ = run_both(cases, reps=1, mode=mode)
    assert path_ok(CHAIN if mode == CHAIN else SEPARATE, many.ctx.last_moe_path())


def test_chained_layers_replayed_from_a_graph():
    """The chained launches recorded through the C ABI's graph API and
    replayed for several tokens in a row (the decode loop's form): every
    replay equals one styx_moe_block call per layer."""
    import ctypes as C
    cases = [make_case(500 + l, 2048, 768, 128, 8, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(4)]
    lws = [upload(c) for c in cases]
    dims = ops.Dims(2048, 768, 128, 8)
    one, many = ops.MoeBlock(dims, 0), ops.MoeBlock(dims, 0)
    many.ctx.set_option(_lib.OPT_MOE_LAYERS, CHAIN)
    rng = np.random.default_rng(7)
    toks = [rng.standard_normal(2048).astype(np.float32) for _ in range(5)]
    x = torch.empty(2048, dtype=torch.float32, device=DEV)
    ids = torch.zeros(4 * 64, dtype=torch.int32, device=DEV)
    stream = torch.cuda.Stream(device=DEV)
    lib, sp = _lib.lib(), C.c_void_p(stream.cuda_stream)
    with torch.cuda.stream(stream):
        x.copy_(T(toks[0]))
        many.forward_layers(x, lws, 0, ids)   # eager first (workspace warm)
    stream.synchronize()
    graph = C.c_void_p()
    _lib.check(lib.styx_graph_begin(many.ctx.handle, sp))
    with torch.cuda.stream(stream):
        many.forward_layers(x, lws, 0, ids)
    _lib.check(lib.styx_graph_end(many.ctx.handle, sp, C.byref(graph)))
    assert many.ctx.last_moe_path() == 5
    try:
        for t in toks:
            with torch.cuda.stream(stream):
                x.copy_(T(t))
            _lib.check(lib.styx_graph_launch(many.ctx.handle, graph, sp))
            stream.synchronize()
            many.ctx.check_device_error(stream)
            xa = T(t)
            ia = torch.zeros_like(ids)
            for i, lw in enumerate(lws):
                one.forward(xa, lw, i, ia)
            torch.cuda.synchronize()
            assert np.array_equal(xa.cpu().numpy().view(np.uint32), x.cpu().numpy().view(np.uint32))
            assert np.array_equal(ia.cpu().numpy(), ids.cpu().numpy())
    finally:
        _lib.check(lib.styx_graph_destroy(many.ctx.handle, graph))


@MODES
def test_split_launch_numbers_time_out_between_linked_layers_and_recover(mode):
    """As tests/test_gpu_timeout.py, for two linked layers: half a grid on the
    launch counter splits every layer's CTAs over two tags; every wait (logits,
    h, x between the layers) gives up after about a second, the error word
    says STYX_ETIMEOUT, and after styx_moe_workspace_init the call is exact."""
    cases = [make_case(400 + l, 1024, 512, 16, 4, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(2)]
    lws = [upload(c) for c in cases]
    blk = ops.MoeBlock(ops.Dims(1024, 512, 16, 4), 0)
    blk.ctx.check_device_error()
    blk.ctx.set_option(_lib.OPT_MOE_LAYERS, mode)
    blk.workspace[GEN_OFFSET:GEN_OFFSET + 8].view(torch.int64).fill_(blk.ctx.sm_count // 2)
    x = T(cases[0].x)
    ids = torch.zeros(2 * 64, dtype=torch.int32, device=DEV)
    blk.forward_layers(x, lws, 0, ids)
    torch.cuda.synchronize()
    assert blk.ctx.last_moe_path() == PATH[mode]
    with pytest.raises(_lib.StyxError) as ei:
        blk.ctx.check_device_error()
    assert ei.value.code == _lib.STYX_ETIMEOUT
    _lib.check(_lib.lib().styx_moe_workspace_init(blk.ctx.handle, None, blk.workspace.data_ptr(), blk.ws_bytes))
    x = T(cases[0].x)
    blk.forward_layers(x, lws, 0, ids)
    torch.cuda.synchronize()
    blk.ctx.check_device_error()
    xr = cases[0].x.copy()
    for c in cases:
        xr = oracle_block(dataclasses.replace(c, x=xr))["x"]
    assert rel_to_max(x.cpu().numpy(), xr) < 1e-4
    blk.ctx.set_option(_lib.OPT_MOE_LAYERS, 0)
