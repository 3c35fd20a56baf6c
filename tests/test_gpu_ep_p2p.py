"""Expert parallelism with the cross-rank sum and the combine as one kernel
over NVLink peer memory (styx_ep_*: CUDA IPC mappings of every rank's
inbox, plain stores, release / acquire flags at system scope, no library
collective).  One process per GPU (world size 2); the handles travel over a
gloo process group.  Three layers in a row (both inbox halves, and a rank a
call ahead of the other) must each equal the single-device styx_moe_block
bit for bit.  The same three layers recorded once as a CUDA graph and
replayed twice (the call generation lives in device memory, so a replay
runs with fresh generations) must give the same bits again.  Skipped with
fewer than two GPUs.
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
        ep = ops.EpComm(rank, WORLD, k, H, rank)
        ep.connect_with(dist)
        x = t(cases[0].x)
        ids = torch.full((LAYERS * 64,), -7, dtype=torch.int32, device=dev)
        partial = torch.empty(k * H, dtype=torch.float32, device=dev)
        for l, lw in enumerate(lws):   # one stream, no host sync between the layers
            blk.forward_ep(x, lw, l, ids, partial)
            ep.combine(partial, x)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x.cpu().numpy())
        # the same layers as one recorded graph, replayed twice from the same input
        lib, cx = _lib.lib(), blk.ctx.handle
        stream = torch.cuda.Stream(device=dev)
        sp = C.c_void_p(stream.cuda_stream)
        x0, xg = t(cases[0].x), torch.empty_like(x)
        graph = C.c_void_p()
        _lib.check(lib.styx_graph_begin(cx, sp))
        for l, lw in enumerate(lws):
            blk.forward_ep(xg, lw, l, ids, partial, stream=stream)
            ep.combine(partial, xg, stream=stream)
        _lib.check(lib.styx_graph_end(cx, sp, C.byref(graph)))
        try:
            for rep in range(2):
                with torch.cuda.stream(stream):
                    xg.copy_(x0)
                _lib.check(lib.styx_graph_launch(cx, graph, sp))
                stream.synchronize()
                blk.ctx.check_device_error(stream)
                np.save(os.path.join(out_dir, f"g{rank}_{rep}.npy"), xg.cpu().numpy())
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
    single = np.load(tmp_path / "single.npy")
    for r in range(WORLD):
        x = np.load(tmp_path / f"x{r}.npy")
        assert np.array_equal(x.view(np.uint32), single.view(np.uint32)), r
        for rep in range(2):
            g = np.load(tmp_path / f"g{r}_{rep}.npy")
            assert np.array_equal(g.view(np.uint32), single.view(np.uint32)), (r, rep)
