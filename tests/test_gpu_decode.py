"""The whole decode step on the GPU (styx_b200.decode: embedding row, per
layer the attention half and the MoE block, output norm, LM head, greedy
pick) against the oracle's forward_token over the same bytes: greedy tokens
identical, hidden state within 1e-3 of max|x| (the bound the north star
sets), logits within 1e-3 of max|logit|; and the two end ops on their own.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from styx_b200 import _lib, ops
from styx_b200.decode import DecodeLayer, DecodeModel, DecodeParams
from tests.decode_case import OracleDecoder, Q4_K, Q6_K, make_model, total_cmp_argmax_last

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


def gpu_model(m, n_ctx, kv_page=0):
    hp = m.hp
    H, F, E = hp["n_embd"], hp["n_ff"], hp["n_expert"]
    layers = []
    for ly in m.layers:
        attn = ops.AttnWeights(T(ly["attn_norm"]), *[ops.DenseWeight(qt, T(raw)) for qt, raw in
                                                      (ly["wq"], ly["wk"], ly["wv"], ly["wo"])],
                               q_norm=T(ly["q_norm"]), k_norm=T(ly["k_norm"]))
        moe = ops.LayerWeights(T(ly["ffn_norm"]), T(ly["router"]),
                               ops.Experts(Q4_K, T(ly["gate"]), F * O.row_bytes(Q4_K, H)),
                               ops.Experts(Q4_K, T(ly["up"]), F * O.row_bytes(Q4_K, H)),
                               ops.Experts(Q6_K, T(ly["down"]), H * O.row_bytes(Q6_K, F)))
        layers.append(DecodeLayer(attn, moe))
    p = DecodeParams(hp["n_layers"], H, hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], F, E,
                     hp["n_expert_used"], hp["n_vocab"], hp["rms_eps"], hp["rope_base"])
    return DecodeModel(p, ops.DenseWeight(Q4_K, T(m.embd)), layers, T(m.output_norm),
                       ops.DenseWeight(Q6_K, T(m.head)), n_ctx, kv_page=kv_page)


@pytest.mark.parametrize("seed,cfg", [(0, {}), (1, {}), (2, dict(hd=128, n_heads=8, n_kv=2))],
                         ids=["hd64-s0", "hd64-s1", "hd128-one-kernel-attention"])
def test_greedy_tokens_identical_to_the_oracle(seed, cfg):
    m = make_model(seed, **cfg)
    prompt, n_predict, n_ctx = [5, 17, 99], 10, 32
    # the oracle's greedy run (generate_moe's loop), keeping every step
    od = OracleDecoder(m, n_ctx)
    steps = []
    for t in prompt:
        lg, x, ids = od.forward_token(t)
    steps.append((lg, x))
    toks = [total_cmp_argmax_last(lg)]
    for _ in range(1, n_predict):
        lg, x, ids = od.forward_token(toks[-1])
        steps.append((lg, x))
        toks.append(total_cmp_argmax_last(lg))
    # the GPU, step by step on the same tokens
    g = gpu_model(m, n_ctx)
    for t in prompt:
        g.forward_token(t)
    got = [int(g.next.item())]
    checks = [(g.logits.cpu().numpy(), g.x.cpu().numpy())]
    for i in range(1, n_predict):
        g.forward_token(toks[i - 1])        # teacher-forced on the oracle's tokens
        got.append(int(g.next.item()))
        checks.append((g.logits.cpu().numpy(), g.x.cpu().numpy()))
    g.moe.ctx.check_device_error()
    assert g.attn.last_path() == (1 if m.hp["head_dim"] == 128 else 2)
    for (lg, x), (elg, ex) in zip(checks, steps):
        assert rel_to_max(x, ex) < 1e-3
        assert rel_to_max(lg, elg) < 1e-3
    assert got == toks
    # and generate() itself, free-running, gives the same sequence
    g.reset()
    assert g.generate(prompt, n_predict) == toks


@pytest.mark.parametrize("qname", ["q4_K", "q5_K", "q6_K", "q8_0"])
def test_get_rows_bit_identical_to_a_cpu_decode(qname):
    qt = _lib.QTYPES[qname]
    rng = np.random.default_rng(qt)
    nrows, ncols = 50, 512
    w = O.quantize(qt, rng.normal(0, 1, (nrows, ncols)).astype(np.float32)).reshape(-1)
    rows = np.array([0, 49, 7, 7, 23], np.int32)
    got = ops.get_rows(qt, T(w), nrows, ncols, T(rows)).cpu().numpy()
    rb = O.row_bytes(qt, ncols)
    exp = np.stack([O.dequantize(qt, w[r * rb:(r + 1) * rb], ncols).reshape(-1) for r in rows])
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_get_rows_out_of_range_is_reported():
    w = O.quantize(_lib.Q8_0, np.ones((4, 64), np.float32)).reshape(-1)
    c = ops.ctx(0)
    c.check_device_error()
    out = ops.get_rows(_lib.Q8_0, T(w), 4, 64, T(np.array([1, 4], np.int32))).cpu().numpy()
    with pytest.raises(_lib.StyxError) as ei:
        c.check_device_error()
    assert ei.value.code == _lib.STYX_EINVAL
    rb = O.row_bytes(_lib.Q8_0, 64)
    assert np.all(out[1] == 0) and np.array_equal(out[0], O.dequantize(_lib.Q8_0, w[rb:2 * rb], 64).reshape(-1))


def test_argmax_total_order_last_of_equals():
    rng = np.random.default_rng(4)
    for n in (1, 100, 151936):
        x = rng.normal(0, 1, n).astype(np.float32)
        if n > 10:
            x[[3, n // 2, n - 5]] = x.max() + 1      # three equal maxima: the last wins
        got = int(ops.argmax_f32(T(x)).item())
        assert got == total_cmp_argmax_last(x) == (n - 5 if n > 10 else 0)
    # total order details: -0.0 < +0.0, +inf below a positive NaN
    x = np.array([-0.0, 0.0, -1.0], np.float32)
    assert int(ops.argmax_f32(T(x)).item()) == 1
    x = np.array([np.inf, np.nan, 1.0], np.float32)
    assert int(ops.argmax_f32(T(x)).item()) == total_cmp_argmax_last(x) == 1


@pytest.mark.parametrize("page", [4, 7])
def test_paged_kv_cache_gives_the_same_bits(page):
    """KV caches grown page by page (moe.rs:1802-1822: reallocated one page
    larger, the filled rows copied) against caches allocated once: every
    step's hidden state, logits and greedy pick are the same bits, across
    several page boundaries."""
    m = make_model(3, hd=128, n_heads=8, n_kv=2)
    n_ctx, toks = 32, [5, 17, 99, 3, 250, 11, 42, 7, 8, 900, 1, 77, 64, 31, 2]
    flat = gpu_model(m, n_ctx)
    paged = gpu_model(m, n_ctx, kv_page=page)
    assert paged.cap == page
    for t in toks:
        flat.forward_token(t)
        paged.forward_token(t)
        torch.cuda.synchronize()
        assert np.array_equal(flat.x.cpu().numpy().view(np.uint32), paged.x.cpu().numpy().view(np.uint32))
        assert np.array_equal(flat.logits.cpu().numpy().view(np.uint32), paged.logits.cpu().numpy().view(np.uint32))
        assert int(flat.next.item()) == int(paged.next.item())
    assert paged.cap == min(n_ctx, page * -(-len(toks) // page)) and paged.kcache.shape[1] == paged.cap
    assert np.array_equal(paged.kcache.cpu().numpy(), flat.kcache[:, :paged.cap].cpu().numpy())
