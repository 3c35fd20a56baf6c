"""numpy front-end for the C oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and the CPU legs of
bench.py use this module as the checker.  The product package (styx_b200)
never imports it.

Every function mirrors a function of styx_oracle.c, which restates the
reference's arithmetic (citations are in the C source).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
QTYPES = {"q8_0": Q8_0, "q4_K": Q4_K, "q5_K": Q5_K, "q6_K": Q6_K}
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
SKIP = 0xFFFFFFFF

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i, f, u64 = C.c_void_p, C.c_int, C.c_float, C.c_uint64
        sigs = {
            "or_dequant_row": (i, [i, vp, i, vp]),
            "or_quantize_row": (i, [i, vp, i, vp]),
            "or_quantize_rows": (i, [i, vp, C.c_longlong, i, vp]),
            "or_matvec_q": (None, [i, vp, i, i, vp, vp]),
            "or_mul_mat_vec_id": (None, [i, vp, C.c_size_t, i, i, vp, i, vp, i, vp]),
            "or_rms_norm": (None, [vp, vp, i, f, vp]),
            "or_matvec_strided_f32": (None, [vp, i, i, i, vp, vp]),
            "or_topk_softmax": (None, [vp, i, i, i, vp, vp, vp, vp]),
            "or_swiglu": (None, [vp, vp, i, vp]),
            "or_moe_reduce": (None, [vp, vp, i, i, vp]),
            "or_gather_slabs": (None, [vp, vp, vp, u64, u64, u64, vp, vp, vp,
                                       u64, u64, u64, vp, i, i]),
            "or_moe_block": (None, [vp, f, vp, i, i, i, i, i, i, i, i, vp, vp, vp,
                                    vp, vp, vp, vp, vp, vp, vp, vp, vp]),
            "or_moe_block_mt": (None, [vp, f, vp, i, i, i, i, i, i, i, i, vp, vp,
                                       vp, vp, i]),
            "or_rope_neox": (None, [vp, i, i, i, f, vp]),
            "or_attn_decode": (None, [vp, vp, vp, vp, i, i, i, i, i, f]),
            "or_attn_block": (None, [vp, vp, f, i, i, i, i, i, vp, vp, f, i, vp, i, vp, i, vp, i, vp, i, vp,
                                     vp]),
            "or_f16_to_f32": (f, [C.c_uint16]),
            "or_f32_to_f16": (C.c_uint16, [f]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def row_bytes(qtype: int, ncols: int) -> int:
    be, bb = BLOCK[qtype]
    assert ncols % be == 0
    return ncols // be * bb


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    """rows of float32 -> rows of quant blocks (uint8)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    rb = row_bytes(qtype, x2.shape[1])
    out = np.zeros((x2.shape[0], rb), dtype=np.uint8)
    rc = lib().or_quantize_rows(qtype, _p(x2), x2.shape[0], x2.shape[1], _p(out))
    assert rc == 0
    return out.reshape(x.shape[:-1] + (rb,))


def dequantize(qtype: int, raw: np.ndarray, ncols: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    rb = row_bytes(qtype, ncols)
    r2 = raw.reshape(-1, rb)
    out = np.zeros((r2.shape[0], ncols), dtype=np.float32)
    L = lib()
    for r in range(r2.shape[0]):
        assert L.or_dequant_row(qtype, _p(r2[r]), ncols, _p(out[r])) == 0
    return out


def matvec_q(qtype, w, nrows, ncols, x):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(nrows, dtype=np.float32)
    lib().or_matvec_q(qtype, _p(w), nrows, ncols, _p(x), _p(y))
    return y


def mul_mat_vec_id(qtype, w, expert_bytes, nrows, ncols, ids, x, ne11, y=None):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if y is None:
        y = np.zeros(len(ids) * nrows, dtype=np.float32)
    lib().or_mul_mat_vec_id(qtype, _p(w), expert_bytes, nrows, ncols, _p(ids),
                            len(ids), _p(x), ne11, _p(y))
    return y


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    lib().or_rms_norm(_p(x), _p(w), x.size, eps, _p(out))
    return out


def matvec_strided_f32(a, x):
    a = np.ascontiguousarray(a, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = np.zeros(a.shape[0], dtype=np.float32)
    lib().or_matvec_strided_f32(_p(a), a.shape[0], a.shape[1], a.shape[1], _p(x), _p(d))
    return d


def topk_softmax(logits, k, renorm=True, remap=None, pmap=None):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    w = np.zeros(16, dtype=np.float32)
    ids = np.full(64, -1, dtype=np.int32)
    remap = None if remap is None else np.ascontiguousarray(remap, dtype=np.uint32)
    pmap = None if pmap is None else np.ascontiguousarray(pmap, dtype=np.uint32)
    lib().or_topk_softmax(_p(logits), logits.size, k, int(renorm), _p(remap),
                          _p(pmap), _p(w), _p(ids))
    return w[:k].copy(), ids


def swiglu(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.zeros_like(g)
    lib().or_swiglu(_p(g), _p(u), g.size, _p(out))
    return out


def moe_reduce(d, w, x):
    d = np.ascontiguousarray(d, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.array(x, dtype=np.float32, copy=True)
    lib().or_moe_reduce(_p(d), _p(w), x.size, w.size, _p(x))
    return x


def gather_slabs(srcs, src_bytes, arenas, dst_bytes, ids, layer, k):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    lib().or_gather_slabs(*[_p(s) for s in srcs], *src_bytes, *[_p(a) for a in arenas],
                          *dst_bytes, _p(ids), layer, k)


def moe_block(x, ffn_norm, eps, router, k, renorm, qtypes, gate, up, down, F,
              remap=None, pmap=None):
    """Returns dict with x (updated), xnorm, logits, weights, ids64, h, d."""
    E, H = router.shape
    x = np.array(x, dtype=np.float32, copy=True)
    out = {
        "xnorm": np.zeros(H, np.float32), "logits": np.zeros(E, np.float32),
        "weights": np.zeros(k, np.float32), "ids64": np.full(64, -1, np.int32),
        "h": np.zeros(k * F, np.float32), "d": np.zeros(k * H, np.float32),
    }
    args = [np.ascontiguousarray(a) for a in (ffn_norm, router, gate, up, down)]
    remap = None if remap is None else np.ascontiguousarray(remap, dtype=np.uint32)
    pmap = None if pmap is None else np.ascontiguousarray(pmap, dtype=np.uint32)
    lib().or_moe_block(_p(args[0]), eps, _p(args[1]), E, H, F, k, int(renorm),
                       qtypes[0], qtypes[1], qtypes[2], _p(args[2]), _p(args[3]),
                       _p(args[4]), _p(remap), _p(pmap), _p(x), _p(out["xnorm"]),
                       _p(out["logits"]), _p(out["weights"]), _p(out["ids64"]),
                       _p(out["h"]), _p(out["d"]))
    out["x"] = x
    return out


def moe_block_mt(x, ffn_norm, eps, router, k, renorm, qtypes, gate, up, down, F,
                 nthreads):
    E, H = router.shape
    x = np.array(x, dtype=np.float32, copy=True)
    args = [np.ascontiguousarray(a) for a in (ffn_norm, router, gate, up, down)]
    lib().or_moe_block_mt(_p(args[0]), eps, _p(args[1]), E, H, F, k, int(renorm),
                          qtypes[0], qtypes[1], qtypes[2], _p(args[2]), _p(args[3]),
                          _p(args[4]), _p(x), nthreads)
    return x


# --------------------------------------------------------------- LCG inputs
def lcg_bytes(seed: int, n: int):
    """The reference tests' LCG (crates/vk-backend/tests/kernels.rs:163-167):
    s = s*1664525 + 1013904223; byte = (s >> 16) as u8.  Returns (bytes, s)."""
    out = np.empty(n, dtype=np.uint8)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = (s >> 16) & 0xFF
    return out, s


def lcg_f32(seed: int, n: int):
    """kernels.rs:174-177: v = (s >> 8) / 2^24 * 2 - 1 in f32.  Returns (v, s)."""
    out = np.empty(n, dtype=np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.float32(s >> 8) / np.float32(1 << 24)) * np.float32(2.0) - np.float32(1.0)
    return out, s


def clamp_f16_exponents(raw: np.ndarray, qtype: int) -> None:
    """kernels.rs:168-171: keep block f16 scales finite and small:
    byte = (byte & 0x83) | 0x30 on the high byte of each f16 scale."""
    bb = BLOCK[qtype][1]
    v = raw.reshape(-1, bb)
    his = {Q8_0: [1], Q4_K: [1, 3], Q5_K: [1, 3], Q6_K: [209]}[qtype]
    for h in his:
        v[:, h] = (v[:, h] & 0x83) | 0x30


# ------------------------------------------------------------ attention half of a decode layer
def rope_neox(x, head_dim, n_heads, n_tokens, freq_base, pos):
    """rope_neox_f32 in the reference test's CPU form (ops2.rs:425-440); returns a copy."""
    x = np.array(x, dtype=np.float32, copy=True)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    lib().or_rope_neox(_p(x), head_dim, n_heads, n_tokens, freq_base, _p(pos))
    return x


def attn_decode(q, kcache, vcache, n_heads, n_t, hd, kv_dim, gqa, scale):
    """shaders/attn_decode_f32.comp restated (every q head)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kcache = np.ascontiguousarray(kcache, dtype=np.float32)
    vcache = np.ascontiguousarray(vcache, dtype=np.float32)
    out = np.zeros(n_heads * hd, dtype=np.float32)
    lib().or_attn_decode(_p(q), _p(kcache), _p(vcache), _p(out), n_heads, n_t, hd, kv_dim, gqa, scale)
    return out


def attn_block(x, attn_norm, eps, n_heads, n_kv, hd, q_norm, k_norm, rope_base, weights, pos, kcache, vcache):
    """One layer's attention half (moe.rs:1857-1972); weights = [(qtype, raw)] for q, k, v, o.
    Returns the new x; kcache / vcache (numpy, [n_ctx][kv_dim]) get row pos."""
    x = np.array(x, dtype=np.float32, copy=True)
    an = np.ascontiguousarray(attn_norm, dtype=np.float32)
    qn = None if q_norm is None else np.ascontiguousarray(q_norm, dtype=np.float32)
    kn = None if k_norm is None else np.ascontiguousarray(k_norm, dtype=np.float32)
    (qq, wq), (qk, wk), (qv, wv), (qo, wo) = [(t, np.ascontiguousarray(w)) for t, w in weights]
    lib().or_attn_block(_p(x), _p(an), eps, x.size, n_heads, n_kv, hd, int(q_norm is not None), _p(qn), _p(kn),
                        rope_base, qq, _p(wq), qk, _p(wk), qv, _p(wv), qo, _p(wo), pos, _p(kcache), _p(vcache))
    return x
