"""The attention half of a decode layer on the CPU: the oracle's RoPE against
the reference test's own case (crates/vk-backend/tests/ops2.rs:413-475), and
the oracle's attention against a float64 softmax (its restatement is pinned
bit for bit to attn_decode_f32.comp in tests/test_ref_glsl.py)."""
import numpy as np
import pytest

from oracle import oracle as O


def test_rope_neox_reference_test_case():
    # ops2.rs:415-440: head_dim 128, 4 heads, 3 tokens, base 1e6, positions
    # [0, 5, 17], inputs from Lcg(0x40e0).f32()
    hd, nh, nt, base = 128, 4, 3, 1_000_000.0
    pos = np.array([0, 5, 17], np.int32)
    x, _ = O.lcg_f32(0x40E0, hd * nh * nt)
    got = O.rope_neox(x, hd, nh, nt, base, pos)
    # the test's CPU reference: theta_scale.powi(i) by repeated multiplication
    ts = float(base) ** (-2.0 / hd)
    exp = x.astype(np.float64).copy()
    for t in range(nt):
        for h in range(nh):
            b = (t * nh + h) * hd
            p = 1.0
            for i in range(hd // 2):
                th = pos[t] * p
                p *= ts
                x0, x1 = float(x[b + i]), float(x[b + i + hd // 2])
                exp[b + i] = x0 * np.cos(th) - x1 * np.sin(th)
                exp[b + i + hd // 2] = x0 * np.sin(th) + x1 * np.cos(th)
    assert np.max(np.abs(got - exp.astype(np.float32))) < 1e-4   # the reference test's bound
    assert np.max(np.abs(got - exp.astype(np.float32))) < 1e-6   # and what a double evaluation gives
    assert np.array_equal(got[: hd * nh], x[: hd * nh])          # position 0 is the identity


@pytest.mark.parametrize("n_heads,n_kv,hd,n_t", [(8, 2, 128, 50), (4, 1, 64, 7)])
def test_attn_oracle_is_softmax_attention(n_heads, n_kv, hd, n_t):
    rng = np.random.default_rng(n_t)
    kv_dim, gqa = n_kv * hd, n_heads // n_kv
    q = rng.normal(0, 1, n_heads * hd).astype(np.float32)
    k = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    v = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    got = O.attn_decode(q, k, v, n_heads, n_t, hd, kv_dim, gqa, scale)
    for h in range(n_heads):
        j = h // gqa
        s = k[:, j * hd:(j + 1) * hd].astype(np.float64) @ q[h * hd:(h + 1) * hd].astype(np.float64) * scale
        p = np.exp(s - s.max())
        o = (p / p.sum()) @ v[:, j * hd:(j + 1) * hd].astype(np.float64)
        assert np.max(np.abs(got[h * hd:(h + 1) * hd] - o)) < 1e-5


def test_oracle_attention_block_against_float64_steps():
    """The oracle's layer (or_attn_block) against the same steps written out
    in float64 numpy (moe.rs:1857-1972): RMSNorm with attn_norm, q/k/v from
    the dequantised weights, per-head q/k RMSNorm, NEOX RoPE at pos, the cache
    row, softmax attention over pos + 1 rows, o and the residual."""
    from tests.decode_case import Q4_K, Q6_K
    rng = np.random.default_rng(21)
    H, nh, nkv, hd, pos, eps, base = 512, 8, 2, 64, 5, 1e-6, 10000.0
    qd, kvd, gqa = nh * hd, nkv * hd, nh // nkv
    mats = {}
    for name, (r, c, qt) in dict(q=(qd, H, Q4_K), k=(kvd, H, Q4_K), v=(kvd, H, Q6_K), o=(H, qd, Q4_K)).items():
        raw = O.quantize(qt, rng.normal(0, 0.05, (r, c)).astype(np.float32)).reshape(-1)
        rb = O.row_bytes(qt, c)
        deq = np.stack([O.dequantize(qt, raw[i * rb:(i + 1) * rb], c).reshape(-1) for i in range(r)])
        mats[name] = (qt, raw, deq.astype(np.float64))
    an = rng.uniform(0.5, 1.5, H).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    x = rng.normal(0, 1, H).astype(np.float32)
    kc = rng.normal(0, 1, (16, kvd)).astype(np.float32)
    vc = rng.normal(0, 1, (16, kvd)).astype(np.float32)
    okc, ovc = kc.copy(), vc.copy()
    got = O.attn_block(x, an, eps, nh, nkv, hd, qn, kn, base, [(mats[n][0], mats[n][1]) for n in "qkvo"], pos,
                       okc, ovc)

    def rms(v, w):
        return v / np.sqrt(np.mean(v * v) + eps) * w

    def rope(v):
        ts = base ** (-2.0 / hd)
        out = v.copy()
        for h in range(v.size // hd):
            for i in range(hd // 2):
                th = pos * ts ** i
                a, b = v[h * hd + i], v[h * hd + i + hd // 2]
                out[h * hd + i] = a * np.cos(th) - b * np.sin(th)
                out[h * hd + i + hd // 2] = a * np.sin(th) + b * np.cos(th)
        return out
    xd = x.astype(np.float64)
    xn = rms(xd, an)
    q = mats["q"][2] @ xn
    k = mats["k"][2] @ xn
    v = mats["v"][2] @ xn
    q = np.concatenate([rms(q[h * hd:(h + 1) * hd], qn) for h in range(nh)])
    k = np.concatenate([rms(k[h * hd:(h + 1) * hd], kn) for h in range(nkv)])
    q, k = rope(q), rope(k)
    K, V = kc.astype(np.float64), vc.astype(np.float64)
    K[pos], V[pos] = k, v
    att = np.empty(qd)
    for h in range(nh):
        j = h // gqa
        s = K[:pos + 1, j * hd:(j + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(s - s.max())
        att[h * hd:(h + 1) * hd] = (p / p.sum()) @ V[:pos + 1, j * hd:(j + 1) * hd]
    exp = xd + mats["o"][2] @ att
    assert np.max(np.abs(got - exp)) / np.max(np.abs(exp)) < 1e-5
    assert np.max(np.abs(okc[pos] - k)) < 1e-5 and np.max(np.abs(ovc[pos] - v)) < 1e-5
    assert np.array_equal(okc[:pos], kc[:pos]) and np.array_equal(okc[pos + 1:], kc[pos + 1:])
