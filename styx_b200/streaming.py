"""Expert streaming under an HBM budget: the cold tier of MoeModel.

Full expert tensors live in pinned host memory (STYX_MEM_HOST, the GTT
buffers of MoeModel::load, moe.rs:856-870); popularity pinning puts the
hottest (layer, expert) slabs in per-layer HBM hot buffers (moe.rs:776-858);
an HBM arena of n_layers x k slots (moe.rs:1170-1193) receives the next
token's predicted cold experts, copied by the copy engine on a side stream
(styx_gather_slabs_async, the M7b-B prefetch of prepare_prefetch,
moe.rs:2169-2383) while the current token's earlier layers compute; a routed
expert that is neither hot nor prefetched is read in place from host memory.
Online repinning (maybe_repin, moe.rs:1450-1505) and the HUD counters
(last_hot_cold, generate_moe.rs:35-119) come from the residency module
(include/styx_residency.h).

The prefetch is adaptive.  Predicting the next token's cold experts from
the previous token's rarely hits (the reference records the same, README's
"next-token prefetch does not work" note), and every prefetched slab costs
host-link bandwidth that the in-place reads of the same token need.  So the
streamer measures the hit rate over a probe window of tokens and switches the
prefetch off when fewer than `prefetch_min_hit` of the prefetched slabs were
used; a repin (which changes what is cold) opens a new probe window.


Placement never changes results: a slot reads the same bytes from the hot
buffer, the arena or the host tensor.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import _lib, ops
from ._lib import check, lib


@dataclass
class StreamStats:
    tokens: int = 0
    hot_hits: int = 0          # routed slots served by the hot buffer
    cold_hits: int = 0         # routed slots not in the hot buffer
    prefetch_hits: int = 0     # cold slots served by the arena (prefetched)
    inplace_reads: int = 0     # cold slots read in place from host memory
    prefetched_slabs: int = 0  # expert slab triples copied by the copy engine
    repin_swaps: int = 0
    prefetch_tokens: int = 0   # tokens that issued a prefetch
    prefetch_off_at: int = -1  # token at which the probe switched the prefetch off (-1: never)
    copy_ms: float = 0.0       # side-stream copy time (first gather start -> last end)
    wait_ms: float = 0.0       # main-stream time spent waiting for those copies
    token_ms: float = 0.0
    cold_by_layer: list = field(default_factory=list)


class ExpertStreamer:
    """The cold-tier placement of an n_layers MoE stack on one device.

    host: per layer a (gate, up, down) triple of HostBuffer-backed uint8
    tensors holding all n_expert slabs; slabs: (gate, up, down) slab bytes;
    hist: (layer, expert, hits) arrays for popularity pinning; budget: bytes
    of HBM for pinned slabs (MoeModel's expert budget)."""

    def __init__(self, dims: ops.Dims, n_layers: int, qtypes, slabs, host, hist, budget: int,
                 device: int = 0, repin_interval: int = 0, repin_max: int = 2, prefetch: bool = True,
                 prefetch_min_hit: float = 0.0, prefetch_probe: int = 16):
        self.dims, self.n_layers, self.qtypes, self.slabs = dims, n_layers, tuple(qtypes), tuple(slabs)
        self.E, self.k = dims.n_expert, dims.n_expert_used
        self.dev = f"cuda:{device}"
        self.device = device
        self.host = host
        self.repin_interval, self.repin_max, self.prefetch = repin_interval, repin_max, prefetch
        # adaptive prefetch: probe window (tokens) and the hit rate that keeps it on (0: always on)
        self.prefetch_min_hit, self.prefetch_probe = prefetch_min_hit, prefetch_probe
        self._probe_left = prefetch_probe
        self._probe_slabs = self._probe_hits = 0
        self._prefetch_on = prefetch
        self.res = ops.Residency(n_layers, self.E, self.k, int(sum(slabs)))
        self.n_pinned = self.res.pin(hist[0], hist[1], hist[2], budget)
        cx = ops.ctx(device).handle
        self.hot = []      # per layer: (gate, up, down) device tensors or None
        self.remap = torch.full((n_layers, self.E), -1, dtype=torch.int32, device=self.dev)
        for l in range(n_layers):
            remap, slots = self.res.layer(l)
            self.remap[l] = torch.from_numpy(remap.view(np.int32).copy()).to(self.dev)
            trio = []
            for t in range(3):
                buf = torch.empty(max(len(slots), 1) * slabs[t], dtype=torch.uint8, device=self.dev)
                for s, e in enumerate(slots):   # the dense hot buffer (moe.rs:836-858)
                    check(lib().styx_copy(cx, C.c_void_p(host[l][t].data_ptr()), int(e) * slabs[t],
                                          C.c_void_p(buf.data_ptr()), s * slabs[t], slabs[t], None))
                trio.append(buf if len(slots) else None)
            self.hot.append(trio)
        # arena: global slot layer * k + j (moe.rs:2199-2201)
        self.arena = [torch.empty(n_layers * self.k * s, dtype=torch.uint8, device=self.dev) for s in slabs]
        self.pmap = torch.full((n_layers, self.E), -1, dtype=torch.int32, device=self.dev)
        self.side = torch.cuda.Stream(device=device)
        self.ev_layer = [torch.cuda.Event() for _ in range(n_layers)]
        self.ev_copy0, self.ev_copy1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.stats = StreamStats(cold_by_layer=[0] * n_layers)
        self._issued = False
        self._issued_pmap = False
        self._last_prefetched = 0
        self._layer_objs = {}
        torch.cuda.synchronize(device)

    def layer_weights(self, l: int, ffn_norm: torch.Tensor, router: torch.Tensor) -> ops.LayerWeights:
        """styx_moe_layer of layer l: full = host tensors, hot, arena, remap,
        pmap views (the structs keep pointers; tables change in place)."""
        ex = []
        for t in range(3):
            hot = self.hot[l][t]
            ex.append(ops.Experts(self.qtypes[t], self.host[l][t], self.slabs[t], hot=hot,
                                  arena=self.arena[t], arena_slab_bytes=self.slabs[t]))
        return ops.LayerWeights(ffn_norm, router, ex[0], ex[1], ex[2], remap=self.remap[l], pmap=self.pmap[l])

    # ---------------------------------------------------------------- per token
    def before_token(self, n_past: int, prev_ids: Optional[np.ndarray], layers: list) -> None:
        """Before forwarding token n_past: repin from the previous token's ids
        (moe.rs:1779-1785), then plan and issue this token's prefetch."""
        self._issued = False
        if prev_ids is None:
            return
        if self.repin_interval:
            swaps = self.res.maybe_repin(prev_ids, n_past, self.repin_interval, self.repin_max)
            if swaps:
                self._apply_swaps(swaps)
                self.stats.repin_swaps += len(swaps)
                if self.prefetch and self.prefetch_min_hit > 0:   # what is cold changed: probe again
                    self._prefetch_on = True
                    self._probe_left = self.prefetch_probe
                    self._probe_slabs = self._probe_hits = 0
        if not self._prefetch_on:
            if self._issued_pmap:   # the arena holds nothing this token: no slot may read it
                self.pmap.fill_(-1)
                self._issued_pmap = False
            return
        pmap, pf = self.res.prefetch_plan(prev_ids)
        self._issued_pmap = True
        self.pmap.copy_(torch.from_numpy(pmap.view(np.int32)))   # before this token's kernels (same stream)
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)          # the previous token no longer reads the arena, the pmap is in place
        self.ev_copy0.record(self.side)
        srcs = [None, None, None]
        self._last_prefetched = 0
        for l in range(self.n_layers):
            ids = pf[l, : self.k]
            n = int((ids >= 0).sum())
            if n:
                srcs = [self.host[l][t] for t in range(3)]
                ops.gather_slabs_async(srcs, list(self.slabs), self.arena, list(self.slabs), ids.tolist(), l, self.k,
                                       stream=self.side, n_expert=self.E)
                self.stats.prefetched_slabs += n
                self._last_prefetched += n
            self.ev_layer[l].record(self.side)
        self.ev_copy1.record(self.side)
        self._issued = True
        self.stats.prefetch_tokens += 1

    def wait_layer(self, l: int) -> None:
        """Order layer l's kernels after its prefetch copies."""
        if self._issued:
            torch.cuda.current_stream(self.device).wait_event(self.ev_layer[l])

    def after_token(self, ids: np.ndarray) -> None:
        """HUD counts of the token just forwarded (last_hot_cold)."""
        hot, cold = self.res.hot_cold(ids)
        self.stats.tokens += 1
        self.stats.hot_hits += int(hot.sum())
        self.stats.cold_hits += int(cold.sum())
        blk = ids.reshape(self.n_layers, 64)
        arena_rows = blk[:, 32:32 + self.k]
        full_rows = blk[:, 48:48 + self.k]
        hits = int((arena_rows >= 0).sum())
        self.stats.prefetch_hits += hits
        self.stats.inplace_reads += int((full_rows >= 0).sum())
        if self._issued and self.prefetch_min_hit > 0 and self._probe_left > 0:
            self._probe_hits += hits
            self._probe_slabs += self._last_prefetched
            self._probe_left -= 1
            if self._probe_left == 0 and self._probe_hits < self.prefetch_min_hit * max(self._probe_slabs, 1):
                self._prefetch_on = False
                self.stats.prefetch_off_at = self.stats.tokens
        for l in range(self.n_layers):
            self.stats.cold_by_layer[l] += int(cold[l])
        if self._issued:
            self.side.synchronize()
            self.stats.copy_ms += self.ev_copy0.elapsed_time(self.ev_copy1)

    def _apply_swaps(self, swaps) -> None:
        cx = ops.ctx(self.device).handle
        st = ops._stream()
        for (l, slot, _old, new) in swaps:
            for t in range(3):
                check(lib().styx_copy(cx, C.c_void_p(self.host[l][t].data_ptr()), new * self.slabs[t],
                                      C.c_void_p(self.hot[l][t].data_ptr()), slot * self.slabs[t], self.slabs[t], st))
            remap, _ = self.res.layer(l)
            self.remap[l].copy_(torch.from_numpy(remap.view(np.int32).copy()))

    def hud(self) -> dict:
        """generate_moe's HUD figures (generate_moe.rs:87-119)."""
        s = self.stats
        tot = max(s.hot_hits + s.cold_hits, 1)
        slab3 = int(sum(self.slabs))
        per_tok = max(s.tokens, 1)
        glyphs = "".join("." if c == 0 else str(min(9, int(10 * c / (per_tok * self.k)))) for c in s.cold_by_layer)
        return {"hot_pct": 100.0 * s.hot_hits / tot, "cold_pct": 100.0 * s.cold_hits / tot,
                "hot_hits": s.hot_hits, "cold_hits": s.cold_hits,
                "prefetch_hits": s.prefetch_hits, "inplace_reads": s.inplace_reads,
                "prefetched_MiB_per_tok": s.prefetched_slabs * slab3 / per_tok / 2 ** 20,
                "inplace_MiB_per_tok": s.inplace_reads * slab3 / per_tok / 2 ** 20,
                "repin_swaps": s.repin_swaps, "cold_by_layer": glyphs, "pinned_slabs": self.n_pinned,
                "prefetch_tokens": s.prefetch_tokens, "prefetch_off_at": s.prefetch_off_at}
