"""configs[2]'s shape over its full depth: 48 layers of hidden 2048, 32 Q / 4
KV heads of 128, 128 experts top-8, expert FFN 768, vocabulary 151,936, the
30B file's format mix (q4_K; v, down and the LM head q6_K).  Random weights
are generated on the device (four distinct layers, each used by 12 of the
48, so that the oracle's copy stays small), a 4-token prompt is decoded and
8 greedy tokens follow; the GPU decode step runs teacher-forced on the
oracle's tokens and must pick the same tokens, with the hidden state and
the logits within 1e-3 of their maxima (the bounds the north star sets).
The reference's own regression is a greedy golden replayed at several
placements (scripts/verify.sh:57-71)."""
import numpy as np
import pytest
import torch

from styx_b200 import ops
from styx_b200.decode import DecodeLayer, DecodeModel, DecodeParams
from tests.decode_case import Model, OracleDecoder, Q4_K, Q6_K, total_cmp_argmax_last

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
L, H, NH, NKV, HD, F, E, K, NV = 48, 2048, 32, 4, 128, 768, 128, 8, 151936
UNIQUE = 4


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


def _host(t):
    return t.cpu().numpy().copy()


@pytest.fixture(scope="module")
def model30b():
    rng = np.random.default_rng(33)
    qd, kvd = NH * HD, NKV * HD
    dev_layers, host_layers = [], []
    for u in range(UNIQUE):
        s = 5000 + 16 * u
        d = dict(wq=ops.synth_quant(Q4_K, qd, H, s, 0.02), wk=ops.synth_quant(Q4_K, kvd, H, s + 1, 0.02),
                 wv=ops.synth_quant(Q6_K, kvd, H, s + 2, 0.02), wo=ops.synth_quant(Q4_K, H, qd, s + 3, 0.02),
                 gate=ops.synth_quant(Q4_K, E * F, H, s + 4, 0.02), up=ops.synth_quant(Q4_K, E * F, H, s + 5, 0.02),
                 down=ops.synth_quant(Q6_K, E * H, F, s + 6, 0.02))
        f = dict(attn_norm=rng.uniform(0.5, 1.5, H).astype(np.float32),
                 q_norm=rng.uniform(0.5, 1.5, HD).astype(np.float32),
                 k_norm=rng.uniform(0.5, 1.5, HD).astype(np.float32),
                 ffn_norm=rng.uniform(0.5, 1.5, H).astype(np.float32),
                 router=rng.normal(0, 0.05, (E, H)).astype(np.float32))
        dev_layers.append((d, f))
        host_layers.append(dict(attn_norm=f["attn_norm"], q_norm=f["q_norm"], k_norm=f["k_norm"],
                                ffn_norm=f["ffn_norm"], router=f["router"],
                                wq=(Q4_K, _host(d["wq"])), wk=(Q4_K, _host(d["wk"])), wv=(Q6_K, _host(d["wv"])),
                                wo=(Q4_K, _host(d["wo"])), gate=_host(d["gate"]), up=_host(d["up"]),
                                down=_host(d["down"])))
    embd = ops.synth_quant(Q4_K, NV, H, 6000, 1.0)
    head = ops.synth_quant(Q6_K, NV, H, 6001, 0.05)
    out_norm = rng.uniform(0.5, 1.5, H).astype(np.float32)
    hp = dict(n_layers=L, n_embd=H, n_heads=NH, n_kv_heads=NKV, head_dim=HD, n_ff=F, n_expert=E, n_expert_used=K,
              n_vocab=NV, rms_eps=1e-6, rope_base=1_000_000.0)
    m = Model(hp, _host(embd), [host_layers[i % UNIQUE] for i in range(L)], out_norm, _host(head))
    return m, dev_layers, embd, head


def _gpu(dev_layers, embd, head, out_norm, n_ctx):
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)   # noqa: E731
    sg, sd = F * ((H // 256) * 144), H * ((F // 256) * 210)
    layers = []
    for i in range(L):
        d, f = dev_layers[i % UNIQUE]
        attn = ops.AttnWeights(T(f["attn_norm"]), ops.DenseWeight(Q4_K, d["wq"]), ops.DenseWeight(Q4_K, d["wk"]),
                               ops.DenseWeight(Q6_K, d["wv"]), ops.DenseWeight(Q4_K, d["wo"]),
                               q_norm=T(f["q_norm"]), k_norm=T(f["k_norm"]))
        moe = ops.LayerWeights(T(f["ffn_norm"]), T(f["router"]), ops.Experts(Q4_K, d["gate"], sg),
                               ops.Experts(Q4_K, d["up"], sg), ops.Experts(Q6_K, d["down"], sd))
        layers.append(DecodeLayer(attn, moe))
    p = DecodeParams(L, H, NH, NKV, HD, F, E, K, NV, 1e-6, 1_000_000.0)
    return DecodeModel(p, ops.DenseWeight(Q4_K, embd), layers, T(out_norm), ops.DenseWeight(Q6_K, head), n_ctx)


def test_48_layer_30b_shape_greedy_identical(model30b):
    m, dev_layers, embd, head = model30b
    prompt, n_predict, n_ctx = [17, 90210, 4242, 151935], 8, 16
    od = OracleDecoder(m, n_ctx)
    steps = []
    for t in prompt:
        lg, x, _ = od.forward_token(t)
    steps.append((lg, x))
    toks = [total_cmp_argmax_last(lg)]
    for _ in range(1, n_predict):
        lg, x, _ = od.forward_token(toks[-1])
        steps.append((lg, x))
        toks.append(total_cmp_argmax_last(lg))
    g = _gpu(dev_layers, embd, head, m.output_norm, n_ctx)
    for t in prompt:
        g.forward_token(t)
    got = [int(g.next.item())]
    checks = [(g.logits.cpu().numpy(), g.x.cpu().numpy())]
    for i in range(1, n_predict):
        g.forward_token(toks[i - 1])        # teacher-forced on the oracle's tokens
        got.append(int(g.next.item()))
        checks.append((g.logits.cpu().numpy(), g.x.cpu().numpy()))
    g.moe.ctx.check_device_error()
    for (lg, x), (elg, ex) in zip(checks, steps):
        assert rel_to_max(x, ex) < 1e-3
        assert rel_to_max(lg, elg) < 1e-3
    assert got == toks
