"""The cold tier: expert tensors held in pinned host memory (STYX_MEM_HOST,
the GTT buffers of MoeModel::load), some experts pinned in an HBM hot buffer,
some prefetched into the HBM arena with the copy engine on a side stream
(styx_gather_slabs_async, ordered by an event), the rest read in place over
the host link.  The MoE block must give the oracle's result and agree with
the all-HBM placement.
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


def _host(a):
    hb = ops.HostBuffer(a.nbytes, 0)
    hb.tensor.copy_(torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)))
    return hb


def _run(blk, c, lw, layer=0, nlayers=1):
    x = _t(c.x)
    ids = torch.full((64 * nlayers,), -7, dtype=torch.int32, device=DEV)
    blk.forward(x, lw, layer, ids)
    torch.cuda.synchronize()
    blk.ctx.check_device_error()
    return x.cpu().numpy(), ids.cpu().numpy()[64 * layer: 64 * (layer + 1)]


def test_cold_tier_in_host_memory_with_prefetch():
    c = make_case(71, 1024, 512, 16, 6, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
    ref = oracle_block(c)
    sel = [int(e) for e in ref["ids64"][: c.k]]
    sg, su, sd = c.slabs
    layer, k, E = 1, c.k, c.E
    blk = ops.MoeBlock(ops.Dims(c.H, c.F, E, k), 0)

    # all-HBM reference run
    lw_dev = ops.LayerWeights(ffn_norm=_t(c.norm), router=_t(c.router),
                              gate=ops.Experts(c.qts[0], _t(c.gate), sg), up=ops.Experts(c.qts[1], _t(c.up), su),
                              down=ops.Experts(c.qts[2], _t(c.down), sd))
    x_dev, ids_dev = _run(blk, c, lw_dev)

    # tiers: two selected + two unselected experts hot; two selected prefetched
    # into the arena; the last two selected read in place from host memory
    unsel = [e for e in range(E) if e not in sel]
    hot_e = sorted(sel[:2] + unsel[:2])
    pf_e = sel[2:4]
    hosts = [_host(c.gate), _host(c.up), _host(c.down)]
    slabs = (sg, su, sd)
    remap = np.full(E, -1, np.int32)
    remap[hot_e] = np.arange(len(hot_e))
    pmap = np.full(E, -1, np.int32)
    for j, e in enumerate(pf_e):
        pmap[e] = layer * k + j
    exps = []
    for t, (qt, src, slab) in enumerate(zip(c.qts, (c.gate, c.up, c.down), slabs)):
        hot = _t(np.concatenate([src[e * slab:(e + 1) * slab] for e in hot_e]))
        arena = torch.zeros((layer + 1) * k * slab, dtype=torch.uint8, device=DEV)
        exps.append(ops.Experts(qt, hosts[t].tensor, slab, hot=hot, arena=arena, arena_slab_bytes=slab))
    # the prefetch: host slabs -> arena slots layer*k + j on a side stream
    side = torch.cuda.Stream()
    host_ids = pf_e + [-1] * (k - len(pf_e))
    ops.gather_slabs_async([h.tensor for h in hosts], list(slabs), [ex.arena for ex in exps], list(slabs), host_ids,
                           layer, k, stream=side, n_expert=E)
    ev = torch.cuda.Event()
    ev.record(side)
    torch.cuda.current_stream().wait_event(ev)
    lw = ops.LayerWeights(ffn_norm=_t(c.norm), router=_t(c.router), gate=exps[0], up=exps[1], down=exps[2],
                          remap=_t(remap), pmap=_t(pmap))
    x_st, ids_st = _run(blk, c, lw, layer=layer, nlayers=layer + 1)
    assert blk.ctx.last_moe_path() == 3          # host-read form
    assert np.array_equal(ids_st[:k], ids_dev[:k])
    hot_rows, arena_rows, full_rows = ids_st[16:16 + k], ids_st[32:32 + k], ids_st[48:48 + k]
    assert (hot_rows != -1).sum() == 2 and (arena_rows != -1).sum() == 2 and (full_rows != -1).sum() == k - 4
    scale = np.max(np.abs(ref["x"]))
    assert np.max(np.abs(x_st - ref["x"])) <= 1e-3 * scale
    assert np.max(np.abs(x_st - x_dev)) <= 1e-5 * scale
    for h in hosts:
        h.free()


@pytest.mark.parametrize("min_hit,want_tokens", [(0.0, 5), (1.01, 2)], ids=["always", "switched-off"])
def test_streamer_prefetch_is_switched_off_when_it_does_not_pay(min_hit, want_tokens):
    """The streamer's adaptive prefetch: with a hit rate that no probe can
    reach, the prefetch runs for the probe window (2 tokens) and then stops;
    results match the all-HBM ones every token, whatever the prefetch does."""
    from styx_b200.streaming import ExpertStreamer
    L, H, F, E, k = 2, 512, 256, 16, 4
    cases = [make_case(90 + l, H, F, E, k, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(L)]
    slabs = cases[0].slabs
    hbs = []
    host = []
    for c in cases:
        trio = []
        for a in (c.gate, c.up, c.down):
            hb = _host(a)
            hbs.append(hb)
            trio.append(hb.tensor)
        host.append(tuple(trio))
    hist = (np.repeat(np.arange(L, dtype=np.int32), E), np.tile(np.arange(E, dtype=np.int32), L),
            np.tile(np.arange(E, 0, -1).astype(np.uint64), L))
    budget = 2 * L * int(sum(slabs))   # two experts of each layer in HBM
    st = ExpertStreamer(ops.Dims(H, F, E, k), L, cases[0].qts, slabs, host, hist, budget, device=0,
                        prefetch=True, prefetch_min_hit=min_hit, prefetch_probe=2)
    layers = [st.layer_weights(l, _t(cases[l].norm), _t(cases[l].router)) for l in range(L)]
    dev_layers = [ops.LayerWeights(_t(c.norm), _t(c.router), ops.Experts(c.qts[0], _t(c.gate), slabs[0]),
                                   ops.Experts(c.qts[1], _t(c.up), slabs[1]), ops.Experts(c.qts[2], _t(c.down), slabs[2]))
                  for c in cases]
    blk = ops.MoeBlock(ops.Dims(H, F, E, k), 0)
    rng = np.random.default_rng(5)
    prev = None
    try:
        for t in range(6):
            x0 = rng.normal(0, 1, H).astype(np.float32)
            st.before_token(t, prev, layers)
            x = _t(x0)
            ids = torch.zeros(L * 64, dtype=torch.int32, device=DEV)
            for l in range(L):
                st.wait_layer(l)
                blk.forward(x, layers[l], l, ids)
            prev = ids.cpu().numpy()
            st.after_token(prev)
            xr = _t(x0)
            ids_r = torch.zeros(L * 64, dtype=torch.int32, device=DEV)
            for l in range(L):
                blk.forward(xr, dev_layers[l], l, ids_r)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            a, b = x.cpu().numpy(), xr.cpu().numpy()   # host-read form against the all-HBM kernel
            assert np.max(np.abs(a - b)) <= 1e-5 * np.max(np.abs(b)), t
        hud = st.hud()
        assert hud["prefetch_tokens"] == want_tokens
        assert hud["prefetch_off_at"] == (-1 if min_hit == 0 else 3)
    finally:
        torch.cuda.synchronize()
        for hb in hbs:
            hb.free()
