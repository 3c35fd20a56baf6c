"""Writes tests/golden/residency_golden.json from the reference's own routing
histogram (tests/golden/route_hist_30b.csv in the reference project, the
fixture its verify script pins with MOE_EXPERT_HIST and a 6 GiB budget).

The placement comes from the oracle restatement (oracle/residency.py) at the
30B-A3B cost per expert (gate 884,736 + up 884,736 + down 1,290,240 bytes)
and budgets of 0, 1, 6 and 12 GiB.  The histogram itself is not copied: the
file records its SHA-256, the per-budget pinned counts and the per-layer hot
sets.  Run from the repository root where the reference is present:

    python tests/golden/gen_residency_golden.py <reference root>
"""
import hashlib
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import residency as R  # noqa: E402

COST = 884736 + 884736 + 1290240
BUDGETS_MIB = [0, 1024, 6144, 12288]


def main() -> int:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STYX_REFERENCE_ROOT", "")
    path = os.path.join(ref, "tests", "golden", "route_hist_30b.csv")
    text = open(path).read()
    entries = R.parse_hist_csv(text)
    out = {"source": "tests/golden/route_hist_30b.csv (reference project)",
           "sha256": hashlib.sha256(text.encode()).hexdigest(),
           "n_layers": 48, "n_expert": 128, "k": 8, "cost_per_expert": COST,
           "n_entries": len(entries), "total_hits": sum(e[0] for e in entries), "budgets": {}}
    for mib in BUDGETS_MIB:
        r = R.Residency(48, 128, 8, COST)
        n = r.pin(entries, mib << 20)
        out["budgets"][str(mib)] = {"n_pinned": n, "hot": [r.slot_experts[l] for l in range(48)]}
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "residency_golden.json")
    with open(dst, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(dst, {k: v["n_pinned"] for k, v in out["budgets"].items()})
    return 0


if __name__ == "__main__":
    sys.exit(main())
