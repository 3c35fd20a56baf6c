"""Expert-parallel exchange on CPU ranks (torch.distributed, gloo, world size
2 and 3): every rank routes, computes w[s] * d[s] only for the slots whose
expert it owns (round-robin ownership), the slot buffers are summed with one
all-reduce, and the slot-ordered combine reproduces the single-rank MoE block
bit for bit.  The per-slot compute is the oracle here (no GPU); the device
kernels behind styx_moe_block_ep / styx_moe_combine are checked against the
single-device block in tests/test_gpu_ep.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.moe_case import make_case, oracle_block


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, seed, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = make_case(seed, 512, 256, 16, 4)
        ref = oracle_block(c)          # every rank routes: same ids, weights and per-slot d
        ids = ref["ids64"][: c.k]
        w = ref["weights"]
        d = ref["d"].reshape(c.k, c.H)
        partial = np.zeros((c.k, c.H), np.float32)
        for s in range(c.k):
            if ids[s] >= 0 and ids[s] % world == rank:          # this rank owns the expert
                partial[s] = np.float32(w[s]) * d[s]            # w[s] * d[s], one IEEE multiply each
        t = torch.from_numpy(partial)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)                # one exchange per layer
        summed = t.numpy()
        acc = np.zeros(c.H, np.float32)
        for s in range(c.k):                                    # slot order, moe_reduce_f32.comp
            acc = acc + summed[s]
        x = c.x.astype(np.float32) + acc
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x)
        np.save(os.path.join(out_dir, "ref.npy"), ref["x"])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ep_allreduce_combine_matches_single_rank(world, tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, 41, str(tmp_path)), nprocs=world, start_method="spawn")
    ref = np.load(tmp_path / "ref.npy")
    for r in range(world):
        x = np.load(tmp_path / f"x{r}.npy")
        assert np.array_equal(x.view(np.uint32), ref.view(np.uint32)), f"rank {r}"
