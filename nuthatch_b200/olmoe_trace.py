"""Routing trace of real generation and the three cache policies replayed on
it (olmoe_trace_main.cc): decode the prompt on the GPU with the routing
trace, then replay learned pin (about 3/4 of the budget pinned to the
hottest experts, the rest LRU), per-layer LRU and one global LRU of the same
total size (the OS page cache), and print their hit rates.

    python -m nuthatch_b200.olmoe_trace model.gguf n_predict budget_per_layer prompt...

NUTHATCH_TRACE_OUT=path also writes the trace (binary format).
"""
from __future__ import annotations

import os
import sys
from typing import Sequence

from . import (BuildUsage, GreedyGenerateCachedTrace, LearnedPinPolicy, LruPolicy, OlmoeModel, OsPageCachePolicy,
               Replay, RoutingTrace, Tokenizer, WriteRoutingTrace)
from ._cli import atoi, emit, norm_topk_from_env, prompt_text


def main(argv: Sequence[str]) -> int:
    if len(argv) < 5:
        print(f"usage: {argv[0]} model.gguf n_predict budget_per_layer prompt...", file=sys.stderr)
        return 1
    model = OlmoeModel.Load(argv[1])
    tok = Tokenizer.Load(argv[1])
    if model is None or tok is None:
        print(f"load failed: {argv[1]}", file=sys.stderr)
        return 1
    n_predict = atoi(argv[2])
    budget = atoi(argv[3]) & 0xFFFFFFFF
    ids = tok.Encode(prompt_text(argv, 4))
    tr = RoutingTrace()
    gen = GreedyGenerateCachedTrace(model, ids, n_predict, norm_topk_from_env(), tr)
    emit(b"text: " + tok.DecodeBytes(ids + gen))
    emit(f"trace: {len(tr.records)} records over {tr.n_layers} layers, {tr.n_expert} experts/layer, "
         f"budget={budget}/layer")
    out = os.environ.get("NUTHATCH_TRACE_OUT")
    if out is not None:
        emit(f"trace written: {out} ({'ok' if WriteRoutingTrace(tr, out) else 'FAILED'})")
    pin = (budget * 3 + 3) // 4 if budget > 1 else 1
    lru_slots = budget - pin if budget > pin else 0
    usage = BuildUsage(tr, tr.n_expert)
    stats = [("learned", Replay(tr, LearnedPinPolicy(tr.n_layers, pin, lru_slots, usage))),
             ("lru", Replay(tr, LruPolicy(tr.n_layers, budget))),
             ("os-page", Replay(tr, OsPageCachePolicy(budget * tr.n_layers)))]
    emit()
    emit("           hit-rate   hits/accesses   (miss = disk read)")
    for name, s in stats:
        emit(f"{name:<10s}  {100.0 * s.hit_rate():6.1f}%   {s.hits}/{s.accesses}")
    learned, lru, os_page = (s.hit_rate() for _, s in stats)
    emit()
    emit(f"learned vs lru:  {100.0 * (learned - lru):+.1f} pp   vs os: {100.0 * (learned - os_page):+.1f} pp")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
