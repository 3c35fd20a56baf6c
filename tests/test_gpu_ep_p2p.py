"""Expert parallelism with the exchange over NVLink peer memory (styx_ep_*:
CUDA IPC mappings of every rank's inbox, plain stores, release adds /
acquire loads of arrival counters at system scope, no library collective),
in both forms: styx_ep_moe_block (the exchange as the single kernel's
epilogue) and styx_moe_block_ep + styx_ep_combine (the exchange as a kernel
of its own).  One process per GPU (world size 2); the handles travel over a
gloo process group.  Three layers in a row (both inbox halves, a rank a call
ahead of the other) must each equal the single-device styx_moe_block bit for
bit: in the combine form, in the fused form, and alternating the two.  The
fused layers recorded once as a CUDA graph and replayed twice (the call
generation lives in device memory) must give the same bits again.  Skipped
with fewer than two GPUs.
"""
import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
LAYERS = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_dir):
    from styx_b200 import _lib, ops
    from tests.moe_case import make_case
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    ep = None
    try:
        def t(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        H, F, E, k = 1024, 512, 16, 6
        cases = [make_case(81 + l, H, F, E, k, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)) for l in range(LAYERS)]
        owned = [e for e in range(E) if e % WORLD == rank]
        remap = np.full(E, -1, np.int32)
        remap[owned] = np.arange(len(owned), dtype=np.int32)

        def ep_layer(c):
            def ex(qt, src, slab):
                return ops.Experts(qt, None, slab, hot=t(np.concatenate([src[e * slab:(e + 1) * slab] for e in owned])))
            sg, su, sd = c.slabs
            return ops.LayerWeights(ffn_norm=t(c.norm), router=t(c.router), gate=ex(c.qts[0], c.gate, sg),
                                    up=ex(c.qts[1], c.up, su), down=ex(c.qts[2], c.down, sd), remap=t(remap))
        lws = [ep_layer(c) for c in cases]
        blk = ops.MoeBlock(ops.Dims(H, F, E, k), rank)
        blk.ctx.set_option(_lib.OPT_MOE_KERNELS, 1)   # the single kernel, as the reference below
        ep = ops.EpComm(rank, WORLD, k, H, rank)
        ep.connect_with(dist)
        ids = torch.full((LAYERS * 64,), -7, dtype=torch.int32, device=dev)
        partial = torch.empty(k * H, dtype=torch.float32, device=dev)
        for name, fused in (("combine", [False] * LAYERS), ("fused", [True] * LAYERS),
                            ("mixed", [l % 2 == 0 for l in range(LAYERS)])):
            x = t(cases[0].x)
            for l, lw in enumerate(lws):   # one stream, no host sync between the layers
                if fused[l]:
                    ep.moe_block(blk, x, lw, l, ids)
                    assert blk.ctx.last_moe_path() == 1
                else:
                    blk.forward_ep(x, lw, l, ids, partial)
                    ep.combine(partial, x)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            np.save(os.path.join(out_dir, f"{name}{rank}.npy"), x.cpu().numpy())
        # the fused layers as one recorded graph, replayed twice from the same input
        lib, cx = _lib.lib(), blk.ctx.handle
        stream = torch.cuda.Stream(device=dev)
        sp = C.c_void_p(stream.cuda_stream)
        x0, xg = t(cases[0].x), torch.empty_like(x)
        graph = C.c_void_p()
        _lib.check(lib.styx_graph_begin(cx, sp))
        for l, lw in enumerate(lws):
            ep.moe_block(blk, xg, lw, l, ids, stream=stream)
        _lib.check(lib.styx_graph_end(cx, sp, C.byref(graph)))
        try:
            for rep in range(2):
                with torch.cuda.stream(stream):
                    xg.copy_(x0)
                _lib.check(lib.styx_graph_launch(cx, graph, sp))
                stream.synchronize()
                blk.ctx.check_device_error(stream)
                np.save(os.path.join(out_dir, f"graph{rank}_{rep}.npy"), xg.cpu().numpy())
        finally:
            _lib.check(lib.styx_graph_destroy(cx, graph))
        if rank == 0:   # the single-device blocks with every expert
            x1 = t(cases[0].x)
            for l, c in enumerate(cases):
                sg, su, sd = c.slabs
                full = ops.LayerWeights(ffn_norm=t(c.norm), router=t(c.router),
                                        gate=ops.Experts(c.qts[0], t(c.gate), sg),
                                        up=ops.Experts(c.qts[1], t(c.up), su),
                                        down=ops.Experts(c.qts[2], t(c.down), sd))
                blk.forward(x1, full, l, torch.full((LAYERS * 64,), -7, dtype=torch.int32, device=dev))
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, "single.npy"), x1.cpu().numpy())
        dist.barrier()
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_ep_over_peer_memory_matches_single_device(tmp_path):
    mp.start_processes(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn")
    single = np.load(tmp_path / "single.npy").view(np.uint32)
    for r in range(WORLD):
        for name in ("combine", "fused", "mixed", "graph_0", "graph_1"):
            f = tmp_path / (f"graph{r}_{name[-1]}.npy" if name.startswith("graph") else f"{name}{r}.npy")
            assert np.array_equal(np.load(f).view(np.uint32), single), (r, name)
