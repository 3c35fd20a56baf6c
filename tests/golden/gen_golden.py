"""Generates tests/golden/quant_golden.npz.

Run in a container that has llama.cpp's gguf-py (0.19.0 here):
    python tests/golden/gen_golden.py

Contents (all float results are float32):
  * for each of q8_0 / q4_K / q5_K / q6_K: random blocks (the reference
    tests' LCG bytes with its f16-exponent clamp, crates/vk-backend/tests/
    kernels.rs:161-171) plus edge blocks, and their decoding by
    gguf.quants.dequantize -- the third-party pin for the block formats
    (q5_K and q6_K have no decoder in the reference itself);
  * the reference's own GPU-test cases, re-created from their seeds, with the
    expectation computed the way each test computes it, but with gguf-py as
    the decoder and numpy for the column-order f32 sums:
      - kernels.rs:150-285  mul_mat_vec_id_q4_k (seed 0xcafef00d, ids
        [6,1,3,0] then [0,6,1,3]),
      - kernels.rs:353-456  mul_mat_vec_q4_k    (seed 0xdeadbeef, 64x512),
      - ops2.rs:225-292     mul_mat_vec_q8_0    (seed 0x51ce, 128x1024),
      - ops2.rs:296-348     swiglu split        (seed 0x5119, 3072x2),
      - kernels.rs:41-122   rms_norm            (seed 0x12345678, 4x2048).
The oracle must reproduce the block decodes and GEMVs bit-for-bit.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import gguf  # noqa: E402
from gguf import quants  # noqa: E402

from oracle.oracle import (BLOCK, Q4_K, Q5_K, Q6_K, Q8_0, QTYPES,  # noqa: E402
                           clamp_f16_exponents, lcg_bytes, lcg_f32)

GG = {Q8_0: gguf.GGMLQuantizationType.Q8_0, Q4_K: gguf.GGMLQuantizationType.Q4_K,
      Q5_K: gguf.GGMLQuantizationType.Q5_K, Q6_K: gguf.GGMLQuantizationType.Q6_K}


def deq(qt: int, raw: np.ndarray) -> np.ndarray:
    bb = BLOCK[qt][1]
    return quants.dequantize(raw.reshape(-1, bb), GG[qt]).reshape(-1).astype(np.float32)


def seq_dot(w: np.ndarray, x: np.ndarray) -> np.float32:
    """Column-order f32 sum of rounded products, as Rust's
    iter().zip().map(|(w,v)| w*v).sum::<f32>() computes it."""
    p = (w.astype(np.float32) * x.astype(np.float32)).astype(np.float32)
    return np.add.accumulate(p, dtype=np.float32)[-1]


def main() -> None:
    out = {}
    seeds = {Q8_0: 0x51CE0001, Q4_K: 0xCAFE0001, Q5_K: 0x55AA0001, Q6_K: 0x6A6B0001}
    for name, qt in QTYPES.items():
        be, bb = BLOCK[qt]
        raw, _ = lcg_bytes(seeds[qt], 32 * bb)
        clamp_f16_exponents(raw, qt)
        edge = np.zeros((4, bb), dtype=np.uint8)
        edge[1, :] = 0xFF                      # saturated codes
        edge[2, :] = 0x5A
        edge[3, :] = np.arange(bb, dtype=np.uint8)
        clamp_f16_exponents(edge.reshape(-1), qt)  # keep f16 scales finite
        edge[0, :] = 0                          # all-zero block (d = 0)
        allraw = np.concatenate([raw, edge.reshape(-1)])
        out[f"{name}_raw"] = allraw
        out[f"{name}_deq"] = deq(qt, allraw)

    # kernels.rs:150-285 -- expert-routed q4_K matvec
    ncols, nrows, n_exp = 512, 32, 8
    bpr = ncols // 256
    eb = nrows * bpr * 144
    a, s = lcg_bytes(0xCAFEF00D, n_exp * eb)
    clamp_f16_exponents(a, Q4_K)
    x, _ = lcg_f32(s, ncols)
    wf = deq(Q4_K, a).reshape(n_exp, nrows, ncols)
    for tag, ids in (("ids0", [6, 1, 3, 0]), ("ids1", [0, 6, 1, 3])):
        y = np.array([seq_dot(wf[e, r], x) for e in ids for r in range(nrows)], dtype=np.float32)
        out[f"idmv_{tag}"] = np.array(ids, dtype=np.int32)
        out[f"idmv_y_{tag}"] = y
    out["idmv_a"], out["idmv_x"] = a, x

    # kernels.rs:353-456 -- q4_K matvec 64x512
    ncols, nrows = 512, 64
    a, s = lcg_bytes(0xDEADBEEF, nrows * (ncols // 256) * 144)
    clamp_f16_exponents(a, Q4_K)
    x, _ = lcg_f32(s, ncols)
    wf = deq(Q4_K, a).reshape(nrows, ncols)
    out["mvq4_a"], out["mvq4_x"] = a, x
    out["mvq4_y"] = np.array([seq_dot(wf[r], x) for r in range(nrows)], dtype=np.float32)

    # ops2.rs:225-292 -- q8_0 matvec 128x1024 (Lcg(0x51ce): bytes then x)
    ncols, nrows = 1024, 128
    a, s = lcg_bytes(0x51CE, nrows * (ncols // 32) * 34)
    clamp_f16_exponents(a, Q8_0)
    x, _ = lcg_f32(s, ncols)
    wf = deq(Q8_0, a).reshape(nrows, ncols)
    out["mvq8_a"], out["mvq8_x"] = a, x
    out["mvq8_y"] = np.array([seq_dot(wf[r], x) for r in range(nrows)], dtype=np.float32)

    # ops2.rs:296-348 -- swiglu split, gate = lcg*4, up = lcg
    n = 3072 * 2
    g, s = lcg_f32(0x5119, n)
    g = (g * np.float32(4.0)).astype(np.float32)
    u, _ = lcg_f32(s, n)
    out["swiglu_g"], out["swiglu_u"] = g, u
    out["swiglu_y"] = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)

    # kernels.rs:41-122 -- rms_norm 4x2048, eps 1e-6, no weight
    xr, _ = lcg_f32(0x12345678, 4 * 2048)
    xr = xr.reshape(4, 2048)
    exp = np.empty_like(xr)
    for r in range(4):
        mean = np.add.accumulate((xr[r] * xr[r]).astype(np.float32), dtype=np.float32)[-1] / np.float32(2048)
        scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(1e-6)))
        exp[r] = xr[r] * scale
    out["rms_x"], out["rms_y"] = xr, exp

    import importlib.metadata
    out["gguf_py_version"] = np.array(importlib.metadata.version("gguf"))
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "quant_golden.npz"))


if __name__ == "__main__":
    main()
