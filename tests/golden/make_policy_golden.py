"""Generates tests/golden/policy_replay.json: cache-policy hit counts computed
by the reference's own compiled policy code (src/cache, built unchanged into
oracle/_ref/libref.so by `make -C oracle ref`) on seeded synthetic routing
traces.  The traces are regenerated from their seeds by `traces()`, so the
fixture holds only the seeds and the counts.

    python tests/golden/make_policy_golden.py      # needs oracle/_ref
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "policy_replay.json"

LRU_BUDGETS = [1, 2, 4, 8, 16, 32]
OS_CAPACITIES = [8, 32, 64, 128]
PIN_BUDGETS = [4, 8, 16]


def _zipf_trace(seed, n_layers, n_expert, k, n_tok, s):
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, n_expert + 1, dtype=np.float64)
    p = ranks ** -s
    p /= p.sum()
    perms = [rng.permutation(n_expert) for _ in range(n_layers)]
    recs = []
    for t in range(n_tok):
        for l in range(n_layers):
            pick = rng.choice(n_expert, size=k, replace=False, p=p)
            recs.append((t, l, [int(perms[l][i]) for i in pick]))
    return recs


def _phased_trace(seed, n_layers, n_expert, k, n_tok, phase):
    rng = np.random.default_rng(seed)
    recs = []
    for t in range(n_tok):
        hot = np.random.default_rng(seed * 1000 + t // phase).permutation(n_expert)[: 2 * k]
        for l in range(n_layers):
            recs.append((t, l, [int(x) for x in rng.choice(hot, size=k, replace=False)]))
    return recs


def traces() -> dict:
    """name -> (n_layers, n_expert, records [(token, layer, experts)])."""
    return {
        "zipf_l4_e64_k8": (4, 64, _zipf_trace(11, 4, 64, 8, 300, 1.1)),
        "uniform_l2_e16_k4": (2, 16, _zipf_trace(12, 2, 16, 4, 200, 0.0)),
        "phased_l3_e32_k8": (3, 32, _phased_trace(13, 3, 32, 8, 240, 60)),
    }


def pin_has_tie(recs, n_layers, pin) -> bool:
    """True when some layer's pin-th and (pin+1)-th usage counts are equal:
    the reference breaks such ties by hash-map order, this build by expert id."""
    for l in range(n_layers):
        c = {}
        for _, ll, ex in recs:
            if ll == l:
                for e in ex:
                    c[e] = c.get(e, 0) + 1
        v = sorted(c.values(), reverse=True)
        if pin < len(v) and pin > 0 and v[pin - 1] == v[pin]:
            return True
    return False


def main() -> int:
    sys.path.insert(0, str(ROOT))
    import oracle

    if not oracle.ref_available():
        print("oracle/_ref/libref.so is missing: run `make -C oracle ref`", file=sys.stderr)
        return 1
    out = {"source": "reference src/cache compiled unchanged (oracle/_ref/libref.so)", "traces": {}}
    for name, (L, E, recs) in traces().items():
        flat = [(l, ex) for _, l, ex in recs]
        entry = {"n_layers": L, "n_expert": E, "n_records": len(recs), "lru": {}, "os": {}, "learned_pin": {}}
        for b in LRU_BUDGETS:
            entry["lru"][str(b)] = oracle.replay(0, flat, L, E, b, use_ref=True)[0]
        for c in OS_CAPACITIES:
            entry["os"][str(c)] = oracle.replay(1, flat, L, E, c, use_ref=True)[0]
        for b in PIN_BUDGETS:
            pin = int(math.ceil(0.75 * b))
            if pin_has_tie(recs, L, pin):
                continue
            entry["learned_pin"][f"{pin},{b - pin}"] = oracle.replay(2, flat, L, E, pin, b - pin, use_ref=True)[0]
        entry["accesses"] = oracle.replay(0, flat, L, E, 1, use_ref=True)[1]
        out["traces"][name] = entry
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
