"""Debugging tool (olmoe_forward_main.cc:17-65): load an OLMoE GGUF, run the
forward over the given token ids and print the top-5 next-token logits of the
last position, to see on a real model that the forward gives a peaked
distribution rather than noise.

    python -m nuthatch_b200.olmoe_forward model.gguf tok0 [tok1 ...]

The forward runs on the GPU as one step of GreedyGenerate (generate.cc:10-53,
a fresh KV cache every call): positions 0..T-2 in one prompt pass, then the
last position, whose logits are printed.  They equal the last row of the
reference's full-sequence BuildForward (forward.cc:8-43), which the oracle's
forward restates.  Ties in the top 5 go to the lower id (the reference's
partial_sort leaves their order unspecified).
"""
from __future__ import annotations

import sys
from typing import Sequence

import numpy as np

from . import OlmoeModel, generate_ex


def last_logits(model: OlmoeModel, toks: Sequence[int], norm_topk: bool = False) -> np.ndarray:
    """Logits [n_vocab] after the last of `toks` (positions 0..T-1)."""
    if len(toks) == 0:
        raise ValueError("at least one token id is needed")
    return generate_ex(model, list(toks), 1, norm_topk, logits=True)["logits"][0]


def top_k(logits: np.ndarray, k: int = 5) -> list[tuple[int, float]]:
    """The k largest logits as (id, logit), largest first, ties to the lower id."""
    order = np.argsort(-logits, kind="stable")[:k]
    return [(int(i), float(logits[i])) for i in order]


def main(argv: Sequence[str]) -> int:
    if len(argv) < 3:
        print(f"usage: {argv[0]} model.gguf tok0 [tok1 ...]", file=sys.stderr)
        return 1
    model = OlmoeModel.Load(argv[1])
    if model is None:
        print(f"load failed: {argv[1]}", file=sys.stderr)
        return 1
    cfg = model.config()
    print(f"loaded: layers={cfg.n_layers} n_embd={cfg.n_embd} n_expert={cfg.n_expert_used}/{cfg.n_expert} "
          f"vocab={cfg.n_vocab}")
    toks = [int(t) for t in argv[2:]]
    best = top_k(last_logits(model, toks))
    print(f"top-5 next-token logits (after pos {len(toks) - 1}):")
    for i, v in best:
        print(f"  tok {i:<6d} logit {v:.4f}")
    model.close()
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
