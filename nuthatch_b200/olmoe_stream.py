"""Streaming text generation (olmoe_stream_main.cc): the experts stay on disk
and stream through `capacity` HBM slots per layer (LRU), read through pinned
bounce buffers; the non-expert weights are resident.  Prints the text and
the process's peak resident host memory.

    python -m nuthatch_b200.olmoe_stream model.gguf n_predict capacity prompt ...
"""
from __future__ import annotations

import resource
import sys
from typing import Sequence

from . import StreamingGenerate, StreamingModel, Tokenizer
from ._cli import atoi, emit, norm_topk_from_env, prompt_text


def peak_rss_mb() -> float:
    return resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 1024.0  # Linux reports KiB


def main(argv: Sequence[str]) -> int:
    if len(argv) < 5:
        print(f"usage: {argv[0]} model.gguf n_predict capacity prompt...", file=sys.stderr)
        return 1
    model = StreamingModel.Load(argv[1], pinned_store=False)
    tok = Tokenizer.Load(argv[1])
    if model is None or tok is None:
        print(f"load failed: {argv[1]}", file=sys.stderr)
        return 1
    n_predict = atoi(argv[2])
    capacity = atoi(argv[3])
    ids = tok.Encode(prompt_text(argv, 4))
    gen = StreamingGenerate(model, ids, n_predict, norm_topk_from_env(), capacity)
    emit(b"text: " + tok.DecodeBytes(ids + gen))
    emit(f"peak RSS: {peak_rss_mb():.0f} MB (capacity={capacity} experts/layer, non-expert weights resident)")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
