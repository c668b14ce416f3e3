"""Text in, text out (olmoe_generate_main.cc): tokenize the prompt with the
model file's own vocabulary, decode greedily on the GPU, print the ids, the
text and the speed.

    python -m nuthatch_b200.olmoe_generate model.gguf n_predict prompt text ...

NUTHATCH_NO_KV_CACHE=1 recomputes the whole sequence every step
(GreedyGenerate) instead of the KV-cached decode; NUTHATCH_NORM_TOPK=1
renormalises the top-k weights.
"""
from __future__ import annotations

import os
import sys
import time
from typing import Sequence

from . import GreedyGenerate, GreedyGenerateCached, OlmoeModel, Tokenizer
from ._cli import atoi, emit, norm_topk_from_env, prompt_text


def main(argv: Sequence[str]) -> int:
    if len(argv) < 4:
        print(f"usage: {argv[0]} model.gguf n_predict prompt text ...", file=sys.stderr)
        return 1
    model = OlmoeModel.Load(argv[1])
    tok = Tokenizer.Load(argv[1])
    if model is None or tok is None:
        print(f"load failed: {argv[1]}", file=sys.stderr)
        return 1
    n_predict = atoi(argv[2])
    ids = tok.Encode(prompt_text(argv, 3))
    norm_topk = norm_topk_from_env()
    emit("prompt ids:" + "".join(f" {t}" for t in ids))
    use_cache = os.environ.get("NUTHATCH_NO_KV_CACHE", "")[:1] != "1"
    t0 = time.perf_counter()
    gen = (GreedyGenerateCached if use_cache else GreedyGenerate)(model, ids, n_predict, norm_topk)
    ms = (time.perf_counter() - t0) * 1000.0
    emit("generated ids:" + "".join(f" {t}" for t in gen))
    emit(b"text: " + tok.DecodeBytes(ids + gen))
    rate = 1000.0 * n_predict / ms if ms > 0 else float("inf")
    emit(f"[{'kv-cache' if use_cache else 'no-cache'}] {n_predict} tokens in {ms:.0f} ms ({rate:.1f} tok/s)")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
