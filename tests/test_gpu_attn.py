"""The attention half of a decode layer on the GPU (include/styx_attn.h)
against the CPU oracle, whose attention is pinned bit for bit to the
reference's attn_decode_f32.comp and whose RoPE is the reference test's own
CPU form (tests/test_ref_glsl.py, tests/test_attn.py).

Tolerances (float32 work in a different order than the oracle's): the
fused norm/RoPE 2e-6 of max|out|; attention 1e-5 of max|out| (the shader's
own online-softmax accumulation over 4096 rows carries ~2e-6 of rounding);
the dense GEMVs 1e-5 of max|y| (the MoE GEMVs' bound); a whole layer 1e-4
of max|x| (the MoE block's bound).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from styx_b200 import _lib, ops

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rel_to_max(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.max(np.abs(got - exp)) / max(np.max(np.abs(exp)), 1e-30))


@pytest.mark.parametrize("n_heads,n_kv,hd,n_t", [(32, 4, 128, 1), (32, 4, 128, 17), (32, 4, 128, 300),
                                                 (32, 4, 128, 4096), (64, 4, 128, 2000), (8, 8, 64, 33),
                                                 (16, 2, 256, 129), (4, 1, 96, 5)])
def test_attn_decode_matches_oracle(n_heads, n_kv, hd, n_t):
    rng = np.random.default_rng(n_heads + hd + n_t)
    kv_dim, gqa = n_kv * hd, n_heads // n_kv
    q = rng.normal(0, 1, n_heads * hd).astype(np.float32)
    k = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    v = rng.normal(0, 1, (n_t, kv_dim)).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    exp = O.attn_decode(q, k, v, n_heads, n_t, hd, kv_dim, gqa, scale)
    got = ops.attn_decode(T(q), T(k), T(v), n_t, hd, kv_dim, gqa, scale).cpu().numpy()
    assert rel_to_max(got, exp) < 1e-5


def test_attn_decode_reads_only_n_t_rows():
    # rows past n_t hold NaN: none of them may reach the output
    rng = np.random.default_rng(3)
    n_heads, n_kv, hd, n_t, n_ctx = 8, 2, 128, 40, 64
    kv_dim = n_kv * hd
    q = rng.normal(0, 1, n_heads * hd).astype(np.float32)
    k = np.full((n_ctx, kv_dim), np.nan, np.float32)
    v = np.full((n_ctx, kv_dim), np.nan, np.float32)
    k[:n_t] = rng.normal(0, 1, (n_t, kv_dim))
    v[:n_t] = rng.normal(0, 1, (n_t, kv_dim))
    got = ops.attn_decode(T(q), T(k), T(v), n_t, hd, kv_dim, 4, 0.125).cpu().numpy()
    exp = O.attn_decode(q, k[:n_t], v[:n_t], n_heads, n_t, hd, kv_dim, 4, 0.125)
    assert np.all(np.isfinite(got)) and rel_to_max(got, exp) < 1e-5


def test_rope_neox_reference_test_case():
    """crates/vk-backend/tests/ops2.rs:413-475 on the device: bound 1e-4,
    position 0 the identity."""
    hd, nh, nt, base = 128, 4, 3, 1_000_000.0
    x, _ = O.lcg_f32(0x40E0, hd * nh * nt)
    pos = np.array([0, 5, 17], np.int32)
    got = ops.rope_neox(T(x), hd, nh, nt, base, T(pos)).cpu().numpy()
    exp = O.rope_neox(x, hd, nh, nt, base, pos)
    assert np.max(np.abs(got - exp)) < 1e-6
    assert np.array_equal(got[: hd * nh], x[: hd * nh])


@pytest.mark.parametrize("n_heads,n_kv,hd,pos", [(32, 4, 128, 0), (32, 4, 128, 1234), (16, 2, 256, 77),
                                                 (8, 8, 64, 9)])
def test_qk_norm_rope_kv_matches_oracle(n_heads, n_kv, hd, pos):
    rng = np.random.default_rng(pos + hd)
    n_ctx, eps, base = 2048, 1e-6, 1_000_000.0
    kv_dim = n_kv * hd
    q = rng.normal(0, 2, n_heads * hd).astype(np.float32)
    k = rng.normal(0, 2, kv_dim).astype(np.float32)
    v = rng.normal(0, 1, kv_dim).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kc = torch.zeros(n_ctx, kv_dim, device=DEV)
    vc = torch.zeros(n_ctx, kv_dim, device=DEV)
    dq, dk = T(q), T(k)
    ops.qk_norm_rope_kv(dq, dk, T(v), T(qn), T(kn), eps, n_heads, n_kv, hd, base, T(np.array([pos], np.int32)),
                        kc, vc, n_ctx)
    eq = np.concatenate([O.rms_norm(q[h * hd:(h + 1) * hd], qn, eps) for h in range(n_heads)])
    ek = np.concatenate([O.rms_norm(k[h * hd:(h + 1) * hd], kn, eps) for h in range(n_kv)])
    eq = O.rope_neox(eq, hd, n_heads, 1, base, np.array([pos], np.int32))
    ek = O.rope_neox(ek, hd, n_kv, 1, base, np.array([pos], np.int32))
    assert rel_to_max(dq.cpu().numpy(), eq) < 2e-6
    assert rel_to_max(dk.cpu().numpy(), ek) < 2e-6
    kc, vc = kc.cpu().numpy(), vc.cpu().numpy()
    assert np.array_equal(kc[pos], dk.cpu().numpy()) and np.array_equal(vc[pos], v)
    others = np.delete(np.arange(n_ctx), pos)
    assert not kc[others].any() and not vc[others].any()


def test_qk_rope_position_outside_the_caches_is_reported():
    hd, n_ctx = 64, 16
    kc = torch.zeros(n_ctx, hd, device=DEV)
    vc = torch.zeros(n_ctx, hd, device=DEV)
    q, k, v = (torch.ones(hd, device=DEV) for _ in range(3))
    c = ops.ctx(0)
    c.check_device_error()
    ops.qk_norm_rope_kv(q, k, v, None, None, 1e-6, 1, 1, hd, 10000.0, T(np.array([n_ctx], np.int32)), kc, vc, n_ctx)
    torch.cuda.synchronize()
    with pytest.raises(_lib.StyxError) as ei:
        c.check_device_error()
    assert ei.value.code == _lib.STYX_EINVAL
    assert not kc.any() and not vc.any()


@pytest.mark.parametrize("qname,nrows,ncols", [("q4_K", 4096, 2048), ("q6_K", 512, 2048), ("q4_K", 2048, 4096),
                                               ("q8_0", 1000, 512), ("q5_K", 300, 768)])
def test_mul_mat_vec_matches_oracle(qname, nrows, ncols):
    qt = _lib.QTYPES[qname]
    rng = np.random.default_rng(nrows + ncols)
    w = O.quantize(qt, rng.normal(0, 0.02, (nrows, ncols)).astype(np.float32)).reshape(-1)
    x = rng.normal(0, 1, ncols).astype(np.float32)
    exp = O.matvec_q(qt, w, nrows, ncols, x)
    got = ops.mul_mat_vec(qt, T(w), nrows, ncols, T(x)).cpu().numpy()
    assert rel_to_max(got, exp) < 1e-5


@pytest.mark.parametrize("qname,nrows,ncols", [("q4_K", 2048, 4096), ("q6_K", 700, 2048)])
def test_mul_mat_vec_add_is_gemv_then_add(qname, nrows, ncols):
    qt = _lib.QTYPES[qname]
    rng = np.random.default_rng(nrows)
    w = T(O.quantize(qt, rng.normal(0, 0.02, (nrows, ncols)).astype(np.float32)).reshape(-1))
    x = T(rng.normal(0, 1, ncols).astype(np.float32))
    y0 = rng.normal(0, 1, nrows).astype(np.float32)
    y = T(y0)
    ops.mul_mat_vec_add(qt, w, nrows, ncols, x, y)
    sep = ops.add_f32(T(y0), ops.mul_mat_vec(qt, w, nrows, ncols, x))
    assert np.array_equal(y.cpu().numpy().view(np.uint32), sep.cpu().numpy().view(np.uint32))


def test_add_f32_in_place():
    rng = np.random.default_rng(2)
    a = rng.normal(0, 1, 5000).astype(np.float32)
    b = rng.normal(0, 1, 5000).astype(np.float32)
    da = T(a)
    ops.add_f32(da, T(b), out=da)
    assert np.array_equal(da.cpu().numpy(), a + b)


def _attn_layer(seed, H, n_heads, n_kv, hd, qts):
    rng = np.random.default_rng(seed)
    qd, kvd = n_heads * hd, n_kv * hd
    ws = []
    for (nr, nc), qt in zip([(qd, H), (kvd, H), (kvd, H), (H, qd)], qts):
        ws.append((qt, O.quantize(qt, rng.normal(0, 0.02, (nr, nc)).astype(np.float32)).reshape(-1)))
    an = rng.uniform(0.5, 1.5, H).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    return ws, an, qn, kn


# STYX_OPT_ATTN_KERNELS values and the LAST_PATH each gives for head_dim 128
AUTO, FUSED, SEPARATE, CLUSTER = 0, 1, 2, 3
PATH = {AUTO: 1, FUSED: 1, SEPARATE: 2, CLUSTER: 3}


@pytest.mark.parametrize("form", [AUTO, CLUSTER, SEPARATE], ids=["one-kernel", "cluster", "seven-kernels"])
@pytest.mark.parametrize("H,n_heads,n_kv,hd,qk", [(2048, 32, 4, 128, True), (1024, 16, 4, 128, False),
                                                 (512, 8, 2, 64, False)])
def test_attn_block_decodes_like_the_oracle(H, n_heads, n_kv, hd, qk, form):
    """Six tokens through one layer's attention half (the 30B shape: q/k/o
    q4_K, v q6_K), the caches filling up row by row; x and the caches after
    every token against the oracle's layer.  Three forms: one cooperative
    kernel (the default for head_dim 128), one launch of thread-block
    clusters and seven launches."""
    if hd != 128 and form == CLUSTER:
        pytest.skip("the one-kernel forms take head_dim 128")
    qts = (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K, _lib.Q4_K)
    ws, an, qn, kn = _attn_layer(H + hd, H, n_heads, n_kv, hd, qts)
    eps, base, n_ctx = 1e-6, 1_000_000.0, 64
    kvd = n_kv * hd
    blk = ops.AttnBlock(H, n_heads, n_kv, hd, qk, eps, base)
    blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, form)
    try:
        _decode_six(blk, H, n_heads, n_kv, hd, qk, ws, an, qn, kn, eps, base, n_ctx, kvd)
        assert blk.last_path() == (PATH[form] if hd == 128 else 2)
    finally:
        blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, 0)


def _decode_six(blk, H, n_heads, n_kv, hd, qk, ws, an, qn, kn, eps, base, n_ctx, kvd):
    w = ops.AttnWeights(T(an), *[ops.DenseWeight(qt, T(raw)) for qt, raw in ws],
                        q_norm=T(qn) if qk else None, k_norm=T(kn) if qk else None)
    kc = torch.zeros(n_ctx, kvd, device=DEV)
    vc = torch.zeros(n_ctx, kvd, device=DEV)
    okc = np.zeros((n_ctx, kvd), np.float32)
    ovc = np.zeros((n_ctx, kvd), np.float32)
    rng = np.random.default_rng(11)
    for pos in range(6):
        x0 = rng.normal(0, 1, H).astype(np.float32)
        x = T(x0)
        blk.forward(x, w, pos, T(np.array([pos], np.int32)), kc, vc, n_ctx)
        torch.cuda.synchronize()
        blk.ctx.check_device_error()
        exp = O.attn_block(x0, an, eps, n_heads, n_kv, hd, qn if qk else None, kn if qk else None, base, ws, pos,
                           okc, ovc)
        assert rel_to_max(x.cpu().numpy(), exp) < 1e-4, pos
        assert rel_to_max(kc.cpu().numpy()[: pos + 1], okc[: pos + 1]) < 1e-4
        assert rel_to_max(vc.cpu().numpy()[: pos + 1], ovc[: pos + 1]) < 1e-4
        # the oracle keeps its own caches, the kernels theirs: continue each
        # from the GPU's rows so that differences do not compound
        okc[: pos + 1] = kc.cpu().numpy()[: pos + 1]
        ovc[: pos + 1] = vc.cpu().numpy()[: pos + 1]


@pytest.mark.parametrize("pos", [300, 2047])
def test_one_kernel_attention_at_long_context(pos):
    """The single kernel with many splits (cache rows filled at random up to
    pos) against the oracle; and against the seven-kernel form."""
    H, n_heads, n_kv, hd = 2048, 32, 4, 128
    qts = (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K, _lib.Q4_K)
    ws, an, qn, kn = _attn_layer(pos, H, n_heads, n_kv, hd, qts)
    eps, base, n_ctx = 1e-6, 1_000_000.0, 2048
    kvd = n_kv * hd
    rng = np.random.default_rng(pos)
    kc0 = rng.normal(0, 1, (n_ctx, kvd)).astype(np.float32)
    vc0 = rng.normal(0, 1, (n_ctx, kvd)).astype(np.float32)
    x0 = rng.normal(0, 1, H).astype(np.float32)
    blk = ops.AttnBlock(H, n_heads, n_kv, hd, True, eps, base)
    w = ops.AttnWeights(T(an), *[ops.DenseWeight(qt, T(raw)) for qt, raw in ws], q_norm=T(qn), k_norm=T(kn))
    outs = {}
    try:
        for form in (CLUSTER, FUSED, SEPARATE):
            blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, form)
            kc, vc, x = T(kc0), T(vc0), T(x0)
            blk.forward(x, w, pos, T(np.array([pos], np.int32)), kc, vc, n_ctx)
            torch.cuda.synchronize()
            blk.ctx.check_device_error()
            assert blk.last_path() == PATH[form]
            outs[form] = (x.cpu().numpy(), kc.cpu().numpy()[pos], vc.cpu().numpy()[pos])
    finally:
        blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, 0)
    okc, ovc = kc0.copy(), vc0.copy()
    exp = O.attn_block(x0, an, eps, n_heads, n_kv, hd, qn, kn, base, ws, pos, okc, ovc)
    for form in (CLUSTER, FUSED, SEPARATE):
        x, krow, vrow = outs[form]
        assert rel_to_max(x, exp) < 1e-4, form
        assert rel_to_max(krow, okc[pos]) < 1e-4 and rel_to_max(vrow, ovc[pos]) < 1e-4
    assert rel_to_max(outs[FUSED][0], outs[SEPARATE][0]) < 1e-5
    assert rel_to_max(outs[CLUSTER][0], outs[SEPARATE][0]) < 1e-5


def test_one_kernel_attention_split_launch_numbers_time_out_and_recover():
    """As tests/test_gpu_timeout.py for the attention kernel: the workspace's
    launch counter set to half a grid splits the CTAs over two launch
    numbers; every wait gives up after about a second, STYX_ETIMEOUT is
    reported, and after styx_attn_block_workspace_init the layer is exact."""
    H, n_heads, n_kv, hd = 1024, 16, 4, 128
    qts = (_lib.Q4_K, _lib.Q4_K, _lib.Q6_K, _lib.Q4_K)
    ws, an, qn, kn = _attn_layer(7, H, n_heads, n_kv, hd, qts)
    eps, base, n_ctx, pos = 1e-6, 1_000_000.0, 16, 3
    blk = ops.AttnBlock(H, n_heads, n_kv, hd, True, eps, base)
    w = ops.AttnWeights(T(an), *[ops.DenseWeight(qt, T(raw)) for qt, raw in ws], q_norm=T(qn), k_norm=T(kn))
    kvd = n_kv * hd
    rng = np.random.default_rng(8)
    kc0 = rng.normal(0, 1, (n_ctx, kvd)).astype(np.float32)
    vc0 = rng.normal(0, 1, (n_ctx, kvd)).astype(np.float32)
    x0 = rng.normal(0, 1, H).astype(np.float32)
    blk.ctx.check_device_error()
    blk.workspace[0:8].view(torch.int64).fill_(blk.ctx.sm_count // 2)   # the launch counter
    blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, FUSED)   # the form with grid-wide waits
    try:
        x = T(x0)
        blk.forward(x, w, pos, T(np.array([pos], np.int32)), T(kc0), T(vc0), n_ctx)
        torch.cuda.synchronize()
        assert blk.last_path() == 1
    finally:
        blk.ctx.set_option(_lib.OPT_ATTN_KERNELS, 0)
    with pytest.raises(_lib.StyxError) as ei:
        blk.ctx.check_device_error()
    assert ei.value.code == _lib.STYX_ETIMEOUT
    blk.init_workspace()
    x, kc, vc = T(x0), T(kc0), T(vc0)
    blk.forward(x, w, pos, T(np.array([pos], np.int32)), kc, vc, n_ctx)
    torch.cuda.synchronize()
    blk.ctx.check_device_error()
    okc, ovc = kc0.copy(), vc0.copy()
    exp = O.attn_block(x0, an, eps, n_heads, n_kv, hd, qn, kn, base, ws, pos, okc, ovc)
    assert rel_to_max(x.cpu().numpy(), exp) < 1e-4


def test_attention_options_are_checked():
    c = ops.ctx(0)
    with pytest.raises(_lib.StyxError) as ei:
        c.set_option(_lib.OPT_ATTN_KERNELS, 4)
    assert ei.value.code == _lib.STYX_EINVAL
    with pytest.raises(_lib.StyxError):
        c.set_option(_lib.OPT_ATTN_LAST_PATH, 1)     # read only
    assert c.get_option(_lib.OPT_ATTN_KERNELS) == 0
