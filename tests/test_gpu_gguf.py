"""A model file through the loader into the MoE block: two layers written as
GGUF (the tensors and keys MoeModel::load reads, moe.rs:550-599, 1056-1078),
parsed by the library's reader, uploaded by gguf.load_moe_layers and run
through styx_moe_block; the oracle computes the same two layers from the same
bytes.  Experts on the device and, second case, in pinned host memory (the
GTT tier, read in place).
"""
import dataclasses

import numpy as np
import pytest
import torch

from styx_b200 import _lib, gguf as G, ops
from tests.moe_case import make_case, oracle_block, topk_margin

pytestmark = pytest.mark.gpu


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


@pytest.mark.parametrize("experts_in_host", [False, True], ids=["hbm", "host"])
def test_moe_layers_from_a_gguf_match_the_oracle(tmp_path, experts_in_host):
    H, F, E, k = 512, 256, 32, 4
    qts = (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K)
    cases = [make_case(60 + l, H, F, E, k, qts) for l in range(2)]
    layers = [dict(norm=c.norm, router=c.router, gate=c.gate, up=c.up, down=c.down, qtypes=c.qts) for c in cases]
    path = tmp_path / "moe.gguf"
    G.write_moe_gguf(path, "qwen3moe", H, F, E, k, cases[0].eps, layers)

    g = G.Gguf.open(path)
    dims, lws, keep = G.load_moe_layers(g, 0, experts_in_host=experts_in_host)
    assert dims == ops.Dims(H, F, E, k, True, np.float32(cases[0].eps).item())
    assert len(lws) == 2
    blk = ops.MoeBlock(dims, 0)
    x = torch.from_numpy(cases[0].x.copy()).cuda()
    ids = torch.full((2 * 64,), -7, dtype=torch.int32, device="cuda")
    for l in range(2):
        blk.forward(x, lws[l], l, ids)
    torch.cuda.synchronize()
    blk.ctx.check_device_error()
    if experts_in_host:
        assert blk.ctx.last_moe_path() == 3     # full tensors in host memory: the host-read form

    xr = cases[0].x.copy()
    ref_ids, ref_logits = [], []
    for c in cases:
        r = oracle_block(dataclasses.replace(c, x=xr))
        ref_ids.append(r["ids64"][:k])
        ref_logits.append(r["logits"])
        xr = r["x"]
    got_ids = ids.cpu().numpy().reshape(2, 64)[:, :k]
    if all(topk_margin(r, k) > 1e-4 for r in ref_logits):   # ids bit-exact where the top-k margin allows
        assert np.array_equal(got_ids, np.stack(ref_ids))
    assert rel_to_max(x.cpu().numpy(), xr) < 1e-4
    g.close()
    for hb in keep:
        hb.free()


def test_whole_model_from_a_gguf_decodes_greedy_identical(tmp_path):
    """A model file through the reader and load_decode_model into the decode
    step (single-kernel attention, head_dim 128): generate() gives the
    oracle's greedy tokens for the same bytes (generate_moe's loop)."""
    from tests.decode_case import make_model, oracle_greedy, write_gguf
    m = make_model(5, n_layers=2, H=512, n_heads=8, n_kv=2, hd=128)
    path = tmp_path / "model.gguf"
    write_gguf(m, path)
    g = G.Gguf.open(path)
    model, keep = G.load_decode_model(g, n_ctx=32)
    g.close()
    prompt, n_predict = [11, 250, 3], 8
    assert model.generate(prompt, n_predict) == oracle_greedy(m, prompt, n_predict)
    assert model.attn.last_path() == 1
    model.moe.ctx.check_device_error()


def test_c_host_decodes_like_the_oracle(tmp_path):
    """The same model file through the plain-C host (generate_moe.c: the GGUF
    reader, uploads, styx_attn_block / styx_moe_block per layer, head and
    greedy pick, all through the C ABI): the oracle's greedy tokens."""
    import subprocess

    from tests.decode_case import make_model, oracle_greedy, write_gguf
    from tests.host_c import build
    m = make_model(5, n_layers=2, H=512, n_heads=8, n_kv=2, hd=128)
    path = tmp_path / "model.gguf"
    write_gguf(m, path)
    exe = build(tmp_path)
    prompt, n_predict = [11, 250, 3], 8
    r = subprocess.run([exe, str(path), str(n_predict), ",".join(map(str, prompt)), "64"], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert [int(t) for t in r.stdout.strip().split(",")] == oracle_greedy(m, prompt, n_predict)
