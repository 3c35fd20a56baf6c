"""Seeded MoE-layer test cases shared by the parity tests.

Weights are N(0, sigma) floats quantised by the oracle's test-data
quantiser; the same bytes go to the GPU and to the oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import oracle as O


@dataclass
class Case:
    H: int
    F: int
    E: int
    k: int
    qts: tuple          # (gate, up, down) ggml types
    x: np.ndarray       # f32[H]
    norm: np.ndarray    # f32[H]
    router: np.ndarray  # f32[E][H]
    gate: np.ndarray    # u8[E*slab_g]
    up: np.ndarray
    down: np.ndarray
    eps: float = 1e-6

    @property
    def slabs(self):
        return (O.row_bytes(self.qts[0], self.H) * self.F, O.row_bytes(self.qts[1], self.H) * self.F,
                O.row_bytes(self.qts[2], self.F) * self.H)


def make_case(seed: int, H: int, F: int, E: int, k: int, qts=(O.Q4_K, O.Q4_K, O.Q6_K), sigma=0.02,
              router_sigma=0.02) -> Case:
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, H).astype(np.float32)
    norm = (1.0 + 0.1 * rng.normal(0, 1, H)).astype(np.float32)
    router = rng.normal(0, router_sigma, (E, H)).astype(np.float32)
    g = O.quantize(qts[0], rng.normal(0, sigma, (E * F, H)).astype(np.float32)).reshape(-1)
    u = O.quantize(qts[1], rng.normal(0, sigma, (E * F, H)).astype(np.float32)).reshape(-1)
    d = O.quantize(qts[2], rng.normal(0, sigma, (E * H, F)).astype(np.float32)).reshape(-1)
    return Case(H, F, E, k, tuple(qts), x, norm, router, g, u, d)


def oracle_block(c: Case, remap=None, pmap=None):
    return O.moe_block(c.x, c.norm, c.eps, c.router, c.k, True, c.qts, c.gate, c.up, c.down, c.F,
                       remap=remap, pmap=pmap)


def topk_margin(logits: np.ndarray, k: int) -> float:
    s = np.sort(logits.astype(np.float64))[::-1]
    if k >= len(s):
        return np.inf
    return float(np.min(np.abs(np.diff(s[: k + 1]))))
