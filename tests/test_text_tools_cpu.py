"""The text tools (olmoe_generate / olmoe_stream / olmoe_trace, the
reference's *_main.cc programs) on CPU: argument handling, the environment
switches and the output lines, with the real tokenizer on a GGUF vocabulary
and the GPU decode replaced by fakes (the decode itself is tested on the
GPU through the same API calls)."""
from __future__ import annotations

import re

import numpy as np
import pytest

import nuthatch_b200 as nh
from nuthatch_b200 import _cli, olmoe_generate, olmoe_stream, olmoe_trace

VOCAB = ["h", "e", "l", "o", "Ġ", "w", "r", "d", "he", "ll", "hell", "hello", "Ġw", "or", "Ġwor", "Ġworld", "!"]
MERGES = ["h e", "l l", "he ll", "hell o", "Ġ w", "o r", "Ġw or", "Ġwor l", "Ġworl d"]


@pytest.fixture()
def model_file(tmp_path):
    import gguf

    vocab = VOCAB + ["Ġworl"]
    path = tmp_path / "m.gguf"
    w = gguf.GGUFWriter(str(path), "olmoe")
    w.add_token_list(vocab)
    w.add_token_merges(MERGES)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return str(path)


class _Model:
    def close(self):
        pass


def test_atoi_follows_c():
    assert [_cli.atoi(s) for s in ("12", " 7x", "-3", "+4", "x", "", "  ", "0009")] == [12, 7, -3, 4, 0, 0, 0, 9]


def test_generate_prints_ids_text_and_rate(model_file, monkeypatch, capsys):
    calls = []

    def fake(model, ids, n, norm_topk):
        calls.append(("cached", ids, n, norm_topk))
        return [16, 15]  # "!" " world"

    monkeypatch.setattr(olmoe_generate.OlmoeModel, "Load", staticmethod(lambda p: _Model()))
    monkeypatch.setattr(olmoe_generate, "GreedyGenerateCached", fake)
    monkeypatch.setattr(olmoe_generate, "GreedyGenerate", lambda *a: calls.append(("full",) + a[1:]) or [16, 16])
    monkeypatch.delenv("NUTHATCH_NO_KV_CACHE", raising=False)
    monkeypatch.setenv("NUTHATCH_NORM_TOPK", "1")
    assert olmoe_generate.main(["olmoe_generate", model_file, "2", "hello", "world"]) == 0
    out = capsys.readouterr().out.splitlines()
    tok = nh.Tokenizer.Load(model_file)
    ids = tok.Encode("hello world")
    assert ids == [11, 15]
    assert calls == [("cached", ids, 2, True)]
    assert out[0] == "prompt ids: 11 15" and out[1] == "generated ids: 16 15"
    assert out[2] == "text: hello world! world"
    assert re.fullmatch(r"\[kv-cache\] 2 tokens in \d+ ms \((\d+\.\d|inf) tok/s\)", out[3])
    monkeypatch.setenv("NUTHATCH_NO_KV_CACHE", "1")
    monkeypatch.delenv("NUTHATCH_NORM_TOPK")
    assert olmoe_generate.main(["olmoe_generate", model_file, "3x", "hello"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert calls[-1] == ("full", [11], 3, False)
    assert out[3].startswith("[no-cache] 3 tokens in ")


def test_tools_refuse_short_arguments_and_failed_loads(model_file, tmp_path, monkeypatch, capsys):
    assert olmoe_generate.main(["g", model_file, "2"]) == 1
    assert olmoe_stream.main(["s", model_file, "2", "4"]) == 1
    assert olmoe_trace.main(["t", model_file, "2", "4"]) == 1
    assert "usage:" in capsys.readouterr().err
    monkeypatch.setattr(olmoe_generate.OlmoeModel, "Load", staticmethod(lambda p: None))
    assert olmoe_generate.main(["g", model_file, "2", "hi"]) == 1
    monkeypatch.setattr(olmoe_generate.OlmoeModel, "Load", staticmethod(lambda p: _Model()))
    assert olmoe_generate.main(["g", str(tmp_path / "none.gguf"), "2", "hi"]) == 1  # no vocabulary
    assert "load failed:" in capsys.readouterr().err


def test_stream_reads_experts_from_disk_and_reports_rss(model_file, monkeypatch, capsys):
    seen = {}

    def load(path, pinned_store=True):
        seen["pinned_store"] = pinned_store
        return _Model()

    def gen(model, ids, n, norm_topk, capacity):
        seen.update(ids=ids, n=n, capacity=capacity)
        return [16]

    monkeypatch.setattr(olmoe_stream.StreamingModel, "Load", staticmethod(load))
    monkeypatch.setattr(olmoe_stream, "StreamingGenerate", gen)
    assert olmoe_stream.main(["olmoe_stream", model_file, "1", "8", "hello"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert seen == {"pinned_store": False, "ids": [11], "n": 1, "capacity": 8}
    assert out[0] == "text: hello!"
    assert re.fullmatch(r"peak RSS: \d+ MB \(capacity=8 experts/layer, non-expert weights resident\)", out[1])


def test_trace_replays_three_policies(model_file, tmp_path, monkeypatch, capsys):
    rng = np.random.default_rng(5)
    L, E, K = 4, 16, 4

    def gen(model, ids, n, norm_topk, trace):
        trace.n_layers, trace.n_expert = L, E
        trace.records = [nh.RoutingRecord(t, l, rng.choice(E, K, replace=False).tolist())
                         for t in range(len(ids) + n - 1) for l in range(L)]
        return [16] * n

    monkeypatch.setattr(olmoe_trace.OlmoeModel, "Load", staticmethod(lambda p: _Model()))
    monkeypatch.setattr(olmoe_trace, "GreedyGenerateCachedTrace", gen)
    out_path = tmp_path / "trace.bin"
    monkeypatch.setenv("NUTHATCH_TRACE_OUT", str(out_path))
    assert olmoe_trace.main(["olmoe_trace", model_file, "12", "6", "hello", "world"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert out[0] == "text: hello world" + "!" * 12
    assert out[1] == f"trace: {13 * L} records over {L} layers, {E} experts/layer, budget=6/layer"
    assert out[2] == f"trace written: {out_path} (ok)"
    back = nh.RoutingTrace()
    assert nh.ReadRoutingTrace(str(out_path), back) and len(back.records) == 13 * L
    usage = nh.BuildUsage(back, E)
    want = [("learned", nh.Replay(back, nh.LearnedPinPolicy(L, 5, 1, usage))),
            ("lru", nh.Replay(back, nh.LruPolicy(L, 6))), ("os-page", nh.Replay(back, nh.OsPageCachePolicy(6 * L)))]
    rows = out[5:8]
    assert rows == [f"{n:<10s}  {100 * s.hit_rate():6.1f}%   {s.hits}/{s.accesses}" for n, s in want]
    h = [s.hit_rate() for _, s in want]
    assert out[9] == f"learned vs lru:  {100 * (h[0] - h[1]):+.1f} pp   vs os: {100 * (h[0] - h[2]):+.1f} pp"
