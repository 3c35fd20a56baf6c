"""Expert parallelism over NCCL: one process per GPU (world size 2), each
holding only its experts (e % 2 == rank), styx_moe_block_ep on its device,
one NCCL all-reduce of the slot buffer, styx_moe_combine; every rank's
hidden state must equal the single-device styx_moe_block bit for bit.
Skipped with fewer than two GPUs.
"""
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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_dir):
    from styx_b200 import _lib, ops
    from tests.moe_case import make_case
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(dev))
    try:
        def t(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        H, F, E, k = 1024, 512, 16, 6
        c = make_case(61, H, F, E, k, (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K))
        sg, su, sd = c.slabs
        owned = [e for e in range(E) if e % WORLD == rank]
        remap = np.full(E, -1, np.int32)
        remap[owned] = np.arange(len(owned), dtype=np.int32)

        def ex(qt, src, slab):
            return ops.Experts(qt, None, slab, hot=t(np.concatenate([src[e * slab:(e + 1) * slab] for e in owned])))
        lw = ops.LayerWeights(ffn_norm=t(c.norm), router=t(c.router), gate=ex(c.qts[0], c.gate, sg),
                              up=ex(c.qts[1], c.up, su), down=ex(c.qts[2], c.down, sd), remap=t(remap))
        blk = ops.MoeBlock(ops.Dims(H, F, E, k), rank)
        x = t(c.x)
        ids = torch.full((64,), -7, dtype=torch.int32, device=dev)
        partial = torch.empty(k * H, dtype=torch.float32, device=dev)
        blk.forward_ep(x, lw, 0, ids, partial)
        dist.all_reduce(partial, op=dist.ReduceOp.SUM)
        blk.combine(partial, x)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x.cpu().numpy())
        path = blk.ctx.last_moe_path()
        if rank == 0:   # the single-device block with every expert, in the same kernel form
            full = ops.LayerWeights(ffn_norm=t(c.norm), router=t(c.router),
                                    gate=ops.Experts(c.qts[0], t(c.gate), sg), up=ops.Experts(c.qts[1], t(c.up), su),
                                    down=ops.Experts(c.qts[2], t(c.down), sd))
            assert path in (1, 6)   # the cluster form or the single kernel, with its expert-parallel epilogue
            x1 = t(c.x)
            blk.forward(x1, full, 0, torch.full((64,), -7, dtype=torch.int32, device=dev))
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, "single.npy"), x1.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_ep_over_nccl_matches_single_device(tmp_path):
    mp.start_processes(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn")
    single = np.load(tmp_path / "single.npy")
    for r in range(WORLD):
        x = np.load(tmp_path / f"x{r}.npy")
        assert np.array_equal(x.view(np.uint32), single.view(np.uint32)), f"rank {r}"
