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
