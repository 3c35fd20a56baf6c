"""TEST INFRASTRUCTURE ONLY -- CPU restatement of MoeModel's expert placement
(crates/model/src/moe.rs), the checker for libstyx_moe.so's residency module
(include/styx_residency.h).  Nothing in the product imports this file.

Plain Python over small lists, written from the reference's Rust:
  budget          moe.rs:741-753
  arena bytes     moe.rs:727-740
  pinning         moe.rs:776-813 (rank by hits, spend the budget), hot_order
                  moe.rs:825-835 (ascending ids), remap moe.rs:984-995
  maybe_repin     moe.rs:1450-1505
  last_hot_cold   moe.rs:1512-1521
  prepare_prefetch moe.rs:2169-2213 (the plan; the async gather is not here)

The reference ranks with Rust's unstable sorts, which leave equal hit counts
in an unspecified order.  This restatement fixes one: equal counts keep input
order when pinning, slot order for residents and ascending expert id for
outsiders when repinning (Python's sort is stable).
"""
from __future__ import annotations

SKIP = 0xFFFFFFFF
IDS_PER_LAYER = 64
U64_MAX = (1 << 64) - 1


def expert_budget(device_vram, headroom, pinned, kv_max, arena, explicit=None, all_vram=False):
    """moe.rs:741-753: u64::MAX for MOE_EXPERTS_VRAM, the explicit figure, or
    device_vram.saturating_sub(headroom + pinned + kv + arena)."""
    if all_vram:
        return U64_MAX
    if explicit is not None:
        return explicit
    res = min(headroom + pinned + kv_max + arena, U64_MAX)
    return max(device_vram - res, 0)


def arena_bytes(n_layers, k, max_slab):
    """moe.rs:727-740: n_layers * k * (max gate + max up + max down slab)."""
    return n_layers * k * sum(max_slab)


def parse_hist_csv(text):
    """MOE_EXPERT_HIST text -> [(hits, layer, expert)] (moe.rs:781-792):
    skip the first line; a line contributes only if its first three comma
    fields parse as unsigned integers."""
    out = []
    lines = text.split("\n")
    if lines and lines[-1] == "":
        lines = lines[:-1]
    for line in lines[1:]:
        if line.endswith("\r"):
            line = line[:-1]
        f = line.split(",")
        # Rust's unsigned FromStr: ASCII digits with at most one leading '+'
        f3 = [x[1:] if x.startswith("+") else x for x in f[:3]]
        if len(f) < 3 or not all(x.isdigit() and x.isascii() for x in f3):
            continue
        layer, expert, hits = int(f3[0]), int(f3[1]), int(f3[2])
        if hits > U64_MAX or expert > 0xFFFFFFFF:
            continue
        out.append((hits, layer, expert))
    return out


class Residency:
    def __init__(self, n_layers, n_expert, k, cost):
        self.n_layers, self.n_expert, self.k, self.cost = n_layers, n_expert, k, cost
        self.remap = [[SKIP] * n_expert for _ in range(n_layers)]
        self.slot_experts = [[] for _ in range(n_layers)]
        self.hits = [[0] * n_expert for _ in range(n_layers)]

    # moe.rs:793-810, 825-835, 984-995
    def pin(self, entries, budget):
        """entries: [(hits, layer, expert)] in input order; returns #pinned."""
        ranked = sorted(entries, key=lambda t: -t[0])
        sets = [set() for _ in range(self.n_layers)]
        left = budget
        for _hits, l, e in ranked:
            if left < self.cost:
                break
            left -= self.cost
            sets[l].add(e)
        for l in range(self.n_layers):
            order = sorted(sets[l])
            self.remap[l] = [SKIP] * self.n_expert
            for i, e in enumerate(order):
                self.remap[l][e] = i
            self.slot_experts[l] = list(order)
            self.hits[l] = [0] * self.n_expert
        return sum(len(s) for s in sets)

    def _routed(self, ids, l, s):
        e = ids[l * IDS_PER_LAYER + s]
        return e if 0 <= e < self.n_expert else None

    # moe.rs:1450-1505
    def maybe_repin(self, ids, n_past, interval, repin_max):
        if interval == 0:
            return []
        for l in range(self.n_layers):
            for s in range(self.k):
                e = self._routed(ids, l, s)
                if e is not None:
                    self.hits[l][e] += 1
        if n_past % interval != 0:
            return []
        swaps = []
        for l in range(self.n_layers):
            slots = self.slot_experts[l]
            h = self.hits[l]
            if not slots:
                continue
            res = sorted(range(len(slots)), key=lambda s: h[slots[s]])
            out = sorted((e for e in range(self.n_expert) if self.remap[l][e] == SKIP), key=lambda e: -h[e])
            for slot, new in list(zip(res, out))[:repin_max]:
                old = slots[slot]
                if h[new] < 2 * max(h[old], 1):
                    break
                self.remap[l][old] = SKIP
                self.remap[l][new] = slot
                slots[slot] = new
                swaps.append((l, slot, old, new))
        return swaps

    # moe.rs:1512-1521
    def hot_cold(self, ids):
        hot, cold = [], []
        for l in range(self.n_layers):
            h = sum(1 for s in range(self.k)
                    if self._routed(ids, l, s) is not None and self.remap[l][self._routed(ids, l, s)] != SKIP)
            hot.append(h)
            cold.append(self.k - h)
        return hot, cold

    # moe.rs:2169-2213
    def prefetch_plan(self, ids):
        pmap = [[SKIP] * self.n_expert for _ in range(self.n_layers)]
        pf = [[-1] * IDS_PER_LAYER for _ in range(self.n_layers)]
        for l in range(self.n_layers):
            n_pf = 0
            for s in range(self.k):
                e = self._routed(ids, l, s)
                if e is None or self.remap[l][e] != SKIP or pmap[l][e] != SKIP:
                    continue
                pmap[l][e] = l * self.k + n_pf
                pf[l][n_pf] = e
                n_pf += 1
        return pmap, pf
