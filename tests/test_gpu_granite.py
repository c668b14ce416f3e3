"""Configuration 5's model shape (Granite-3-MoE-shaped: 24 layers, n_embd 1024,
16 query heads x 64 with 8 KV heads, 32 experts top-8, expert FFN 512,
vocab 49155, emitted as an OLMoE GGUF with q/k-norm weights of 1) and its
batched streaming form.

* Resident batch-1 decode and streaming at a budget of 8 of 32 experts per
  layer (LRU and learned pin) against the oracle; streaming hit counts
  against the reference's compiled policies over the GPU's own routing.
* Batched streaming (StreamingGenerateBatch): when a step's batch (or a
  chunk of the prompt) selects more distinct experts than the slot pool
  holds (a precondition violation for the reference,
  expert_slot_cache.h:21) each layer runs in waves; every
  sequence's ids equal the resident batched decode, on the mini model and on
  the Granite shape, with LRU and learned-pin pools.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import nuthatch_b200 as nh
import oracle
from nuthatch_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def granite(synth_dir):
    path = synth.cached(synth.GRANITE_MOE, synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    assert m is not None
    c = m.config()
    assert (c.n_layers, c.n_embd, c.n_head, c.n_head_kv, c.n_expert, c.n_expert_used, c.n_ff, c.n_vocab) == (
        24, 1024, 16, 8, 32, 8, 512, 49155)
    oracle.set_threads(min(32, os.cpu_count() or 8))
    return path, m


def test_granite_resident_decode_matches_oracle(gpu, granite):
    path, m = granite
    prompt = np.random.default_rng(50).integers(0, 49155, 12).tolist()
    g = nh.generate_ex(m, prompt, 12, False, hidden=True)
    ora = oracle.OracleModel(str(path)).generate(prompt, 12, mode=0, hidden=True)
    assert g["tokens"] == ora["tokens"]
    assert np.array_equal(g["hidden"], ora["hidden"])


@pytest.mark.parametrize("policy", ["lru", "learned_pin"])
def test_granite_streaming_budget8_matches_oracle(gpu, granite, policy):
    path, m = granite
    cfg = m.config()
    cal = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(m, np.random.default_rng(51).integers(0, cfg.n_vocab, 16).tolist(), 16, False, cal)
    usage = nh.BuildUsage(cal, cfg.n_expert).counts
    prompt = np.random.default_rng(52).integers(0, cfg.n_vocab, 10).tolist()
    pin = 6  # ceil(3/4 x 8)
    sm = nh.StreamingModel.Load(str(path))
    kw = dict(policy="learned_pin", pin_slots=pin, usage=usage) if policy == "learned_pin" else {}
    s = nh.streaming_generate_ex(sm, prompt, 14, False, 8, trace=True, **kw)
    sm.close()
    ora = oracle.OracleModel(str(path)).stream_generate(prompt, 14, False, 8, policy=1 if kw else 0,
                                                        pin_slots=pin if kw else 0, usage=usage if kw else None)
    assert s["tokens"] == ora["tokens"] == nh.GreedyGenerateCached(m, prompt, 14, False)
    assert np.array_equal(s["hits"], ora["hits"]) and np.array_equal(s["misses"], ora["misses"])
    if oracle.ref_available():
        L = cfg.n_layers
        recs = [(l, s["sel"][t, l].tolist()) for t in range(s["sel"].shape[0]) for l in range(L)]
        if policy == "lru":
            hits, _ = oracle.replay(0, recs, L, cfg.n_expert, 8, use_ref=True)
        else:
            cut = np.sort(usage, axis=1)[:, ::-1]
            if np.any(cut[:, pin - 1] == cut[:, pin]):
                pytest.skip("calibration counts tie at the pin cut (the reference orders ties by hash map)")
            hits, _ = oracle.ref_replay_pin_usage(recs, L, cfg.n_expert, pin, 8 - pin, usage)
        assert hits == int(s["hits"].sum())


@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict,capacity,policy", [
    ("MINI", 6, 5, 6, 4, "lru"),            # 16 experts top-4: several waves per layer
    ("MINI", 6, 5, 6, 4, "learned_pin"),    # pinned experts join the first wave
    ("GRANITE_MOE", 8, 6, 5, 8, "lru"),     # configuration 5's pool: 8 of 32 experts
    ("GRANITE_MOE", 8, 6, 5, 8, "learned_pin"),
])
def test_batched_streaming_waves_match_resident_batch(gpu, synth_dir, spec_name, n_seq, n_prompt, n_predict,
                                                      capacity, policy):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    cfg = m.config()
    prompts = np.random.default_rng(60 + n_seq).integers(0, cfg.n_vocab, (n_seq, n_prompt)).tolist()
    ref = nh.generate_batch_ex(m, prompts, n_predict, False)["tokens"]
    kw = {}
    if policy == "learned_pin":
        cal = nh.RoutingTrace()
        nh.GreedyGenerateCachedTrace(m, prompts[0], 8, False, cal)
        kw = dict(policy="learned_pin", pin_slots=(capacity * 3 + 3) // 4,
                  usage=nh.BuildUsage(cal, cfg.n_expert).counts)
    m.close()
    sm = nh.StreamingModel.Load(str(path))
    r = nh.streaming_generate_batch_ex(sm, prompts, n_predict, False, capacity, **kw)
    sm.close()
    assert r["tokens"] == ref
    # Passes over the layers: the prompt's 512-row chunks (positions 0..P-2 of
    # every sequence), then one per decoded id.
    chunk = min(n_prompt - 1, 512 // n_seq)
    passes = -(-(n_prompt - 1) // chunk) + n_predict
    assert r["waves"] > passes * cfg.n_layers  # more distinct experts than slots: more than one wave per layer
    assert int((r["hits"] + r["misses"]).sum()) > 0 and r["h2d_bytes"] > 0
