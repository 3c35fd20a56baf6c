"""Expert residency planning (include/styx_residency.h, C++ in libstyx_moe.so)
against the CPU restatement of MoeModel's placement (oracle/residency.py):
budget, popularity pinning, remap tables, online repin, HUD counts and the
prefetch plan.  Host logic only: these run without a GPU.

Pinned to the reference's own routing histogram through
tests/golden/residency_golden.json (tests/golden/gen_residency_golden.py);
when the reference tree is present the golden is re-derived from its CSV.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import residency as R
from styx_b200 import _lib, ops

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "residency_golden.json")
REF_ROOT = os.environ.get("STYX_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")
REF_HIST = os.path.join(REF_ROOT, "tests", "golden", "route_hist_30b.csv")
COST_30B = 884736 + 884736 + 1290240


def ids_buffer(rows, n_layers, k):
    """n_layers x 64 int32 with rows[l] in the first k entries (row 0)."""
    a = np.full((n_layers, 64), -7, np.int32)
    for l, r in enumerate(rows):
        a[l, :k] = r
    return a


def random_ids(rng, n_layers, n_expert, k, p_skip=0.0, zipf=False):
    rows = []
    for _ in range(n_layers):
        if zipf:
            w = 1.0 / np.arange(1, n_expert + 1) ** 1.1
            r = rng.choice(n_expert, size=k, replace=False, p=w / w.sum())
        else:
            r = rng.choice(n_expert, size=k, replace=False)
        r = r.astype(np.int32)
        r[rng.random(k) < p_skip] = -1
        rows.append(r)
    return ids_buffer(rows, n_layers, k)


@pytest.mark.parametrize("args", [
    (192 << 30, 1 << 30, 4 << 30, 2 << 30, 1 << 30, None, False),
    (8 << 30, 1 << 30, 6 << 30, 2 << 30, 1 << 30, None, False),      # saturates at 0
    (192 << 30, 0, 0, 0, 0, 6144 << 20, False),
    (192 << 30, 0, 0, 0, 0, 0, False),                                # explicit 0 = nothing pinned
    (192 << 30, 1 << 30, 0, 0, 0, None, True),
    ((1 << 64) - 1, (1 << 63), (1 << 63), 5, 0, None, False),       # reservations overflow: saturate
])
def test_budget_matches_oracle(args):
    vram, head, pinned, kv, arena, explicit, all_vram = args
    assert ops.expert_budget(vram, head, pinned, kv, arena, explicit, all_vram) == \
        R.expert_budget(vram, head, pinned, kv, arena, explicit, all_vram)


def test_arena_bytes():
    assert ops.arena_bytes(48, 8, (884736, 884736, 1290240)) == R.arena_bytes(48, 8, (884736, 884736, 1290240))
    assert ops.arena_bytes(48, 8, (884736, 884736, 1290240)) == 48 * 8 * 3059712


@pytest.mark.parametrize("seed", range(6))
def test_pin_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    L, E, k, cost = 6, 32, 4, 1000
    n = int(rng.integers(0, L * E + 20))
    layer = rng.integers(0, L, n).astype(np.int32)
    expert = rng.integers(0, E, n).astype(np.int32)    # repeats allowed: the reference pins a set
    hits = rng.integers(0, 6, n).astype(np.uint64)     # many ties
    budget = int(rng.integers(0, n + 3)) * cost + int(rng.integers(0, cost))
    got = ops.Residency(L, E, k, cost)
    exp = R.Residency(L, E, k, cost)
    assert got.pin(layer, expert, hits, budget) == exp.pin(list(zip(hits.tolist(), layer.tolist(),
                                                                    expert.tolist())), budget)
    for l in range(L):
        remap, slots = got.layer(l)
        assert remap.tolist() == exp.remap[l]
        assert slots.tolist() == exp.slot_experts[l]


def test_pin_csv_parsing_matches_oracle():
    text = ("layer,expert,hits\n"
            "0,3,10\r\n"          # CRLF line end
            "0,+4,9\n"            # Rust's unsigned parse takes one leading '+'
            "1,5,x\n"             # does not parse: skipped
            "\n"                  # empty line: skipped
            "1,6\n"               # too few fields: skipped
            "1,7,8,extra\n"       # extra fields ignored
            "2,1,-3\n"            # sign: skipped
            " 2,2,5\n"            # whitespace: skipped
            "2,3,99999999999999999999999\n"   # u64 overflow: skipped
            "2,0,7")              # no final newline
    for budget in (0, 1000, 3000, 10 ** 6):
        got = ops.Residency(3, 8, 2, 1000)
        exp = R.Residency(3, 8, 2, 1000)
        assert got.pin_csv(text, budget) == exp.pin(R.parse_hist_csv(text), budget)
        for l in range(3):
            remap, slots = got.layer(l)
            assert remap.tolist() == exp.remap[l] and slots.tolist() == exp.slot_experts[l]
    r = ops.Residency(3, 8, 2, 1000)
    assert r.pin_csv("layer,expert,hits\n", 10 ** 9) == 0
    assert r.pin_csv("", 10 ** 9) == 0


def test_pin_rejects_out_of_range():
    r = ops.Residency(2, 8, 2, 10)
    with pytest.raises(_lib.StyxError):
        r.pin([2], [0], [1], 100)
    with pytest.raises(_lib.StyxError):
        r.pin_csv("h\n0,8,1\n", 100)


def test_pin_reference_histogram_golden():
    g = json.load(open(GOLDEN))
    text = None
    if os.path.exists(REF_HIST):
        text = open(REF_HIST).read()
        assert hashlib.sha256(text.encode()).hexdigest() == g["sha256"]
    for mib, rec in g["budgets"].items():
        r = ops.Residency(48, 128, 8, g["cost_per_expert"])
        if text is not None:
            n = r.pin_csv(text, int(mib) << 20)
        else:
            # the golden's own hot sets, re-pinned through the array entry point
            ent = [(l, e) for l in range(48) for e in rec["hot"][l]]
            n = r.pin([x[0] for x in ent], [x[1] for x in ent], [1] * len(ent), len(ent) * g["cost_per_expert"])
        assert n == rec["n_pinned"]
        for l in range(48):
            assert r.layer(l)[1].tolist() == rec["hot"][l]
    # the reference's verify script pins about 2,105 slabs at 6 GiB
    assert g["budgets"]["6144"]["n_pinned"] == 6442450944 // COST_30B


@pytest.mark.parametrize("seed,interval,rmax", [(0, 1, 2), (1, 3, 2), (2, 4, 1), (3, 2, 8), (4, 0, 2)])
def test_repin_sequence_matches_oracle(seed, interval, rmax):
    rng = np.random.default_rng(seed)
    L, E, k, cost = 4, 24, 4, 1
    got = ops.Residency(L, E, k, cost)
    exp = R.Residency(L, E, k, cost)
    # pin a cold set so the Zipf stream has profitable swaps
    ent = [(l, e) for l in range(L) for e in range(E - 6, E)]
    got.pin([x[0] for x in ent], [x[1] for x in ent], [1] * len(ent), 10 ** 9)
    exp.pin([(1, l, e) for l, e in ent], 10 ** 9)
    n_swaps = 0
    for n_past in range(1, 60):
        ids = random_ids(rng, L, E, k, p_skip=0.05, zipf=True)
        s_got = got.maybe_repin(ids, n_past, interval, rmax)
        s_exp = exp.maybe_repin(ids.reshape(-1).tolist(), n_past, interval, rmax)
        assert s_got == s_exp
        n_swaps += len(s_got)
        for l in range(L):
            remap, slots = got.layer(l)
            assert remap.tolist() == exp.remap[l] and slots.tolist() == exp.slot_experts[l]
            assert got.hits(l).tolist() == exp.hits[l]
    if interval:
        assert n_swaps > 0
    else:
        assert n_swaps == 0


def test_repin_hysteresis_and_cap():
    r = ops.Residency(1, 8, 2, 1)
    r.pin([0, 0], [0, 1], [5, 5], 2)          # experts 0, 1 hot
    ids = ids_buffer([[2, 3]], 1, 2)
    assert r.maybe_repin(ids, 1, 2, 2) == []  # not a repin token
    # expert 2 and 3 have 2 hits each, residents 0: 2 >= 2*max(0,1) -> swap both
    assert r.maybe_repin(ids, 2, 2, 2) == [(0, 0, 0, 2), (0, 1, 1, 3)]
    # cap smaller than the swaps: error, tables untouched afterwards
    r2 = ops.Residency(1, 8, 2, 1)
    r2.pin([0, 0], [0, 1], [5, 5], 2)
    assert r2.maybe_repin(ids, 1, 2, 2) == []   # first token counted, no repin yet
    buf = (_lib.RepinSwap * 1)()
    import ctypes as C
    n = C.c_int()
    a = np.ascontiguousarray(ids_buffer([[2, 3]], 1, 2).reshape(-1))
    rc = _lib.lib().styx_residency_maybe_repin(r2.handle, a.ctypes.data, 2, 2, 2, buf, 1, C.byref(n))
    assert rc == _lib.STYX_EINVAL


@pytest.mark.parametrize("seed", range(4))
def test_hot_cold_and_prefetch_match_oracle(seed):
    rng = np.random.default_rng(100 + seed)
    L, E, k = 5, 16, 6
    got = ops.Residency(L, E, k, 1)
    exp = R.Residency(L, E, k, 1)
    n = 3 * L
    layer = rng.integers(0, L, n).astype(np.int32)
    expert = rng.integers(0, E, n).astype(np.int32)
    hits = rng.integers(1, 9, n).astype(np.uint64)
    got.pin(layer, expert, hits, n)
    exp.pin(list(zip(hits.tolist(), layer.tolist(), expert.tolist())), n)
    ids = random_ids(rng, L, E, k, p_skip=0.1)
    ids[1, 2] = ids[1, 1]   # a duplicate routed id in one layer
    hot, cold = got.hot_cold(ids)
    eh, ec = exp.hot_cold(ids.reshape(-1).tolist())
    assert hot.tolist() == eh and cold.tolist() == ec
    assert int(hot.sum() + cold.sum()) == L * k        # the HUD identity (verify.sh:73-83)
    pmap, pf = got.prefetch_plan(ids)
    epmap, epf = exp.prefetch_plan(ids.reshape(-1).tolist())
    assert pmap.tolist() == epmap
    assert pf[:, :k].tolist() == [row[:k] for row in epf]
    # every planned slot is this layer's block of the arena, and never a hot expert
    for l in range(L):
        slots = pmap[l][pmap[l] != _lib.SKIP]
        assert all(l * k <= s < (l + 1) * k for s in slots)
        remap, _ = got.layer(l)
        assert all(remap[e] == _lib.SKIP for e in pf[l, :k] if e >= 0)
