"""Model-free cache-policy curves over a routing trace (trace_replay_main.cc):
read one trace file and compare the three policies' hit rates over several
per-layer budgets, or sweep the pin/LRU split of learned pin at one budget.
Seconds of host work; no model and no GPU.

    python -m nuthatch_b200.trace_replay [--text] trace [budget ...]   (default 4 8 12 16 24 32)
    python -m nuthatch_b200.trace_replay [--text] trace pin budget

--text reads the text form (one "<layer> e0 e1 ..." line per record), else
the binary form (routing_trace.cc).  The numeric rows have the reference
tool's formats; its header lines are given here in English.  Budgets must be
non-negative integers (the reference's atoi takes anything).
"""
from __future__ import annotations

import sys
from typing import Sequence

from . import ReadRoutingTrace, ReadRoutingTraceText, RoutingTrace, SweepBudgets, SweepPinRatio

DEFAULT_BUDGETS = (4, 8, 12, 16, 24, 32)


def _budget(s: str) -> int | None:
    return int(s) if s.isdigit() else None


def main(argv: Sequence[str]) -> int:
    a = 1
    text = len(argv) > a and argv[a] == "--text"
    if text:
        a += 1
    usage = f"usage: {argv[0]} [--text] trace [budget ...] | trace pin B"
    if len(argv) <= a:
        print(usage, file=sys.stderr)
        return 1
    path = argv[a]
    a += 1
    t = RoutingTrace()
    if not (ReadRoutingTraceText(path, t) if text else ReadRoutingTrace(path, t)):
        print(f"read trace failed: {path}", file=sys.stderr)
        return 1
    print(f"trace: {len(t.records)} records, {t.n_layers} layers, {t.n_expert} experts/layer")

    if len(argv) >= a + 2 and argv[a] == "pin":
        budget = _budget(argv[a + 1])
        if budget is None:
            print(usage, file=sys.stderr)
            return 1
        print(f"\nfixed budget {budget}/layer, pin/lru split:")
        print("  pin  lru   learned")
        for pin, lru, learned in SweepPinRatio(t, budget):
            print(f"{pin:5d} {lru:4d}   {100.0 * learned:6.1f}%")
        return 0

    budgets = [_budget(s) for s in argv[a:]]
    if any(b is None for b in budgets):
        print(usage, file=sys.stderr)
        return 1
    if not budgets:
        budgets = list(DEFAULT_BUDGETS)
    print("\nbudget/L   learned     lru       os      learned-lru")
    for budget, learned, lru, os_ in SweepBudgets(t, budgets):
        print(f"{budget:6d}    {100.0 * learned:6.1f}%   {100.0 * lru:6.1f}%   {100.0 * os_:6.1f}%    "
              f"{100.0 * (learned - lru):+.1f} pp")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
