"""Batched greedy decode (GreedyGenerateCachedBatch) against the batch-1 path
and the oracle: every sequence's ids are identical to decoding it alone
(the per-token arithmetic is the same), with CUDA graphs and without."""
from __future__ import annotations

import numpy as np
import pytest

import nuthatch_b200 as nh
import oracle
from nuthatch_b200 import synth

pytestmark = pytest.mark.gpu


def _prompts(n_seq, n_prompt, n_vocab, seed):
    return np.random.default_rng(seed).integers(0, n_vocab, (n_seq, n_prompt)).tolist()


@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict", [
    ("MINI", 3, 8, 6),          # MHA, 16 experts top-4
    ("MINI_GQA", 5, 5, 5),      # GQA, every expert selected (top-8 of 8)
    ("MINI", 2, 70, 4),         # contexts past one 64-position split
])
def test_batch_matches_single_sequence_and_oracle(gpu, synth_dir, spec_name, n_seq, n_prompt, n_predict):
    path = str(synth.cached(getattr(synth, spec_name), synth_dir))
    m = nh.OlmoeModel.Load(path)
    cfg = m.config()
    prompts = _prompts(n_seq, n_prompt, cfg.n_vocab, 100 + n_seq)
    got = nh.generate_batch_ex(m, prompts, n_predict, False)
    eager = nh.generate_batch_ex(m, prompts, n_predict, False, use_graph=False)
    assert got["tokens"] == eager["tokens"]
    om = oracle.OracleModel(path)
    for b in range(n_seq):
        single = nh.GreedyGenerateCached(m, prompts[b], n_predict, False)
        assert got["tokens"][b] == single, (b, got["tokens"][b], single)
        assert got["tokens"][b] == om.generate(prompts[b], n_predict, mode=0)["tokens"]
    om.close()


def test_batch_full_olmoe_matches_single_sequence(gpu, synth_dir):
    path = str(synth.cached(synth.OLMOE_1B7B, synth_dir))
    m = nh.OlmoeModel.Load(path)
    prompts = _prompts(4, 8, m.config().n_vocab, 7)
    got = nh.GreedyGenerateCachedBatch(m, prompts, 6, False)
    for b in range(4):
        assert got[b] == nh.GreedyGenerateCached(m, prompts[b], 6, False), b


def test_batch_rejects_ragged_prompts(gpu, synth_dir):
    m = nh.OlmoeModel.Load(str(synth.cached(synth.MINI, synth_dir)))
    with pytest.raises(ValueError):
        nh.generate_batch_ex(m, [[1, 2, 3], [4, 5]], 2, False)


@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict", [
    ("MINI", 3, 200, 4),        # two chunks of 170 + 29 positions
    ("MINI_GQA", 64, 20, 3),    # 8 positions x 64 sequences per chunk, a ragged last chunk
    ("MINI", 520, 3, 2),        # more sequences than one chunk's rows: one position per chunk
    ("OLMOE_1B7B", 8, 150, 4),  # configuration 4's shape, cut short: 512-row chunks on the tensor cores
])
def test_batched_prefill_matches_position_by_position(gpu, synth_dir, monkeypatch, spec_name, n_seq, n_prompt,
                                                      n_predict):
    """The chunked prompt prefill (positions 0..P-2 of every sequence as rows
    of the batched kernels) gives the same ids as running the prompt one
    position per step (NH_BATCH_PREFILL=0)."""
    path = str(synth.cached(getattr(synth, spec_name), synth_dir))
    m = nh.OlmoeModel.Load(path)
    prompts = _prompts(n_seq, n_prompt, m.config().n_vocab, 300 + n_seq)
    got = nh.generate_batch_ex(m, prompts, n_predict, False)
    assert got["prefill_ms"] > 0
    monkeypatch.setenv("NH_BATCH_PREFILL", "0")
    ref = nh.generate_batch_ex(m, prompts, n_predict, False)
    monkeypatch.delenv("NH_BATCH_PREFILL")
    assert ref["prefill_ms"] == 0
    assert got["tokens"] == ref["tokens"]
    for b in (0, n_seq - 1):
        assert got["tokens"][b] == nh.GreedyGenerateCached(m, prompts[b], n_predict, False), b
    m.close()
