"""configs[0] exactly as specified (4 layers, hidden 512, 8 Q / 2 KV heads of
64, 32 experts top-4, FFN 256, vocab 4096, every matrix q8_0, 16-id prompt
from default_rng(101), 32 greedy tokens), written as a model file and decoded
on the GPU in three placements -- experts in HBM, experts in pinned host
memory read in place, and through the plain-C host -- each against the
oracle's greedy tokens for the same bytes (the reference's own regression is
a greedy golden replayed at several placements, scripts/verify.sh:57-71)."""
import subprocess

import numpy as np
import pytest

from styx_b200 import gguf as G
from tests.decode_case import OracleDecoder, make_config1, total_cmp_argmax_last, write_gguf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg1(tmp_path_factory):
    m, prompt, n_predict = make_config1()
    path = tmp_path_factory.mktemp("cfg1") / "cfg1.gguf"
    write_gguf(m, path)
    od = OracleDecoder(m, 64)
    for t in prompt:
        lg, _, _ = od.forward_token(t)
    toks, margins = [], []
    for i in range(n_predict):
        if i:
            lg, _, _ = od.forward_token(toks[-1])
        s = np.sort(lg.astype(np.float64))[::-1]
        margins.append((s[0] - s[1]) / max(abs(s[0]), 1e-30))
        toks.append(total_cmp_argmax_last(lg))
    return m, prompt, n_predict, path, toks, margins


@pytest.mark.parametrize("experts_in_host", [False, True], ids=["experts-hbm", "experts-host"])
def test_config1_greedy_identical(cfg1, experts_in_host):
    m, prompt, n_predict, path, toks, margins = cfg1
    g = G.Gguf.open(path)
    model, keep = G.load_decode_model(g, n_ctx=64, experts_in_host=experts_in_host)
    g.close()
    got = model.generate(prompt, n_predict)
    model.moe.ctx.check_device_error()
    assert got == toks, f"first divergence at {next(i for i, (a, b) in enumerate(zip(got, toks)) if a != b)}; " \
                        f"smallest top-2 margin {min(margins):.2e}"
    for hb in keep:
        hb.free()


def test_config1_c_host_greedy_identical(cfg1, tmp_path):
    from tests.host_c import build
    m, prompt, n_predict, path, toks, margins = cfg1
    exe = build(tmp_path)
    r = subprocess.run([exe, str(path), str(n_predict), ",".join(map(str, prompt)), "64"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert [int(t) for t in r.stdout.strip().split(",")] == toks
