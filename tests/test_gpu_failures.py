"""Failure handling on the host side (no GPU fault is provoked: the failures
are made by the host, as a failing disk read or a truncated file would).

* ExpertSlotCache with a reader whose reads start failing mid-batch (the
  reader's host-side fault injection): Ensure reports the error, the expert
  whose fill failed is mapped to no slot, the one filled before the failure
  stays resident, and a later Ensure of the failed id misses and fills it
  with the right bytes.  (The reference ignores a failed read and maps the
  slot regardless, expert_slot_cache.cc:96.)
* Streaming straight from disk (no pinned host store) through the slot
  cache's ring of bounce buffers: ids equal the resident decode.
* GGUF files cut short in the header or in the tensor data: probing and
  loading return an error / nullptr instead of a model.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import nuthatch_b200 as nh
from nuthatch_b200 import synth
from nuthatch_b200._lib import NhConfig, lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mini(synth_dir):
    return synth.cached(synth.MINI, synth_dir)


def _cfg(path):
    m = nh.OlmoeModel.Load(str(path))
    c = m.config()
    m.close()
    return c


def test_slot_cache_failed_fill_leaves_no_mapping(gpu, mini):
    cfg = _cfg(mini)
    rd = nh.ExpertReader.Open(str(mini))
    cache = nh.ExpertSlotCache.Create(cfg, 0, 4, rd)
    assert cache is not None
    # Expert 1's three tensors read; the first read of expert 2 fails.
    rd.FailReadsAfter(3)
    with pytest.raises(nh.NhError):
        cache.Ensure([1, 2])
    assert cache.misses() == 2 and cache.hits() == 0
    rd.FailReadsAfter(-1)
    # Expert 1 was filled before the failure: resident, a hit.
    s1 = cache.Ensure([1])[1]
    assert cache.hits() == 1
    # Expert 2 was never mapped: a miss, filled now with the right bytes.
    s2 = cache.Ensure([2])[2]
    assert cache.misses() == 3
    for which, name in enumerate(("blk.0.ffn_gate_exps.weight", "blk.0.ffn_up_exps.weight",
                                  "blk.0.ffn_down_exps.weight")):
        want = rd.ReadExpert(name, 2)
        assert cache.slot_bytes(which, s2, len(want)) == want, name
        assert cache.slot_bytes(which, s1, len(want)) == rd.ReadExpert(name, 1), name


def test_disk_backed_streaming_matches_resident(gpu, mini):
    """Streaming without the pinned host store: every miss reads the expert
    from disk into one of the slot cache's pinned bounce buffers (a ring of
    three, each reused only after its copies finished) and copies it to its
    slot; the ids equal the resident decode."""
    prompt = np.random.default_rng(31).integers(0, 1000, 9).tolist()
    m = nh.OlmoeModel.Load(str(mini))
    ref = nh.GreedyGenerateCached(m, prompt, 10, False)
    m.close()
    sm = nh.StreamingModel.Load(str(mini), pinned_store=False)
    for cap in (4, 6):
        r = nh.streaming_generate_ex(sm, prompt, 10, False, cap)
        assert r["tokens"] == ref, cap
        assert int(r["misses"].sum()) > 0 and r["h2d_bytes"] > 0
    sm.close()


def test_truncated_gguf_is_refused(gpu, mini, tmp_path):
    raw = mini.read_bytes()
    c = NhConfig()
    for frac, what in ((0.0005, "header"), (0.6, "tensor data")):
        cut = tmp_path / f"cut_{what.replace(' ', '_')}.gguf"
        cut.write_bytes(raw[:max(16, int(len(raw) * frac))])
        if what == "header":
            assert lib().nh_gguf_probe(str(cut).encode(), C.byref(c)) < 0
        assert nh.OlmoeModel.Load(str(cut)) is None, what
        assert nh.StreamingModel.Load(str(cut)) is None, what
    # The intact file still loads.
    m = nh.OlmoeModel.Load(str(mini))
    assert m is not None
    m.close()
