"""The benchmark configurations at their stated sizes, against the oracle and
the reference's own compiled cache policies (oracle/_ref).

* Configuration 2 (streaming): the router-skewed OLMoE-1B-7B-shaped GGUF,
  prompt 64, 256 greedy ids, slot budget 16 of 64 experts per layer, LRU
  (the reference's ExpertSlotCache, expert_slot_cache.cc:59-72) and learned
  pin (pin = ceil(3/4 x 16) = 12, usage histogram from a resident run on a
  different prompt, olmoe_trace_main.cc:61-71).  Ids equal the oracle's
  StreamingGenerate; per-layer hits and misses equal the oracle's; the hit
  counts equal a replay of the GPU's own routing trace through the
  reference's compiled LruPolicy / LearnedPinPolicy
  (streaming_forward.cc:228-253, expert_slot_cache.cc:83-104).
* Configuration 3 (batched decode, 64 sequences): the 64-sequence batch at
  2048-token contexts against decoding sequences alone (first and last), and
  a 64-sequence batch at 512-token contexts against the oracle on a seeded
  subset of two sequences.  Subset stated: the oracle restatement runs at
  about 5-10 positions/s on the host, so the 2048-token contexts are pinned
  through the single-sequence path (itself pinned to the oracle by the
  prefill and decode tests), not by the oracle directly.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import nuthatch_b200 as nh
import oracle
from nuthatch_b200 import synth

pytestmark = pytest.mark.gpu


def _pin_cut_has_tie(usage: np.ndarray, pin: int) -> bool:
    """Whether some layer's pin-th and (pin+1)-th counts are equal (the
    reference breaks such ties by hash-map order)."""
    for row in usage:
        c = np.sort(row)[::-1]
        if pin < len(c) and c[pin - 1] == c[pin]:
            return True
    return False


@pytest.fixture(scope="module")
def skew_setup(synth_dir):
    path = synth.cached(synth.OLMOE_1B7B_SKEW, synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    cfg = m.config()
    cal = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(m, np.random.default_rng(70).integers(0, cfg.n_vocab, 64).tolist(), 64, False, cal)
    usage = nh.BuildUsage(cal, cfg.n_expert).counts
    m.close()
    oracle.set_threads(min(32, os.cpu_count() or 8))
    return path, cfg, usage


@pytest.mark.parametrize("policy", ["lru", "learned_pin"])
def test_config2_streaming_budget16_matches_oracle_and_reference_policies(gpu, skew_setup, policy):
    path, cfg, usage = skew_setup
    budget, pin = 16, 12
    prompt = np.random.default_rng(80).integers(0, cfg.n_vocab, 64).tolist()
    sm = nh.StreamingModel.Load(str(path))
    s = nh.streaming_generate_ex(sm, prompt, 256, False, budget, policy=policy, pin_slots=pin if policy != "lru" else 0,
                                 usage=usage if policy != "lru" else None, trace=True)
    sm.close()
    om = oracle.OracleModel(str(path))
    ora = om.stream_generate(prompt, 256, False, budget, policy=0 if policy == "lru" else 1,
                             pin_slots=pin if policy != "lru" else 0, usage=usage if policy != "lru" else None)
    assert s["tokens"] == ora["tokens"]
    assert np.array_equal(s["hits"], ora["hits"]) and np.array_equal(s["misses"], ora["misses"])
    # The reference's own compiled policy over the GPU's routing, layer by layer.
    L = cfg.n_layers
    recs = [(l, s["sel"][t, l].tolist()) for t in range(s["sel"].shape[0]) for l in range(L)]
    if oracle.ref_available():
        if policy == "lru":
            hits, acc = oracle.replay(0, recs, L, cfg.n_expert, budget, use_ref=True)
        else:
            if _pin_cut_has_tie(usage, pin):
                pytest.skip("calibration counts tie at the pin cut (the reference orders ties by hash map)")
            hits, acc = oracle.ref_replay_pin_usage(recs, L, cfg.n_expert, pin, budget - pin, usage)
        assert hits == int(s["hits"].sum()) and acc == int(s["hits"].sum() + s["misses"].sum())
        for l in (0, L // 2, L - 1):
            mine = [r for r in recs if r[0] == l]
            if policy == "lru":
                h, _ = oracle.replay(0, mine, L, cfg.n_expert, budget, use_ref=True)
            else:
                h, _ = oracle.ref_replay_pin_usage(mine, L, cfg.n_expert, pin, budget - pin, usage)
            assert h == int(s["hits"][l]), l


@pytest.fixture(scope="module")
def olmoe(synth_dir):
    path = synth.cached(synth.OLMOE_1B7B, synth_dir)
    return path, nh.OlmoeModel.Load(str(path))


def test_config3_batch64_2048_context_matches_single_sequence(gpu, olmoe):
    path, m = olmoe
    cfg = m.config()
    prompts = np.random.default_rng(3).integers(0, cfg.n_vocab, (64, 2048)).tolist()
    r = nh.generate_batch_ex(m, prompts, 16, False)
    for b in (0, 63):
        assert r["tokens"][b] == nh.GreedyGenerateCached(m, prompts[b], 16, False), b


def test_config3_batch64_matches_oracle_on_a_subset(gpu, olmoe):
    path, m = olmoe
    cfg = m.config()
    prompts = np.random.default_rng(13).integers(0, cfg.n_vocab, (64, 512)).tolist()
    r = nh.generate_batch_ex(m, prompts, 8, False)
    om = oracle.OracleModel(str(path))
    oracle.set_threads(min(32, os.cpu_count() or 8))
    for b in (0, 37):
        ora = om.generate(prompts[b], 8, mode=2)
        assert r["tokens"][b] == ora["tokens"], b
