"""GPU parity: the sm_100a path through the C ABI against the CPU oracle.

The kernels and the oracle share one arithmetic contract (the order in which
super-block values and f32 products are summed, and the exp used by softmax
and SiLU; see the oracle's header), so the whole-token path is expected to be
bit-identical:
  * integer/byte work is bit-exact: Q8_K activation quantisation, K-quant
    dequantisation, routing ids, greedy ids, slot-cache hit/miss counts;
  * per-layer hidden states and logits are compared for exact equality
    (EXACT); the hot path's stated bound, max |gpu - oracle| / max |oracle|
    <= 2e-2 (REL_TOL), is checked as well and is what a divergence would be
    judged against;
  * a greedy id or routing record may differ only where the oracle shows a
    near-tie below NEAR_TIE (1e-4) at that point;
  * standalone GEMV rows on random activations: <= GEMV_TOL relative.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import nuthatch_b200 as nh
import oracle
from nuthatch_b200 import synth
from nuthatch_b200._lib import lib
from tests.ref_fixtures import write_slot_fixture, write_tiny_olmoe

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2
GEMV_TOL = 2e-5
NEAR_TIE = 1e-4


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


EXACT = True


def assert_matches(got, want, what=""):
    err = rel_err(got, want)
    assert err <= REL_TOL, f"{what} relative error {err:.3g} above the stated bound"
    if EXACT:
        assert np.array_equal(np.asarray(got), np.asarray(want)), f"{what} not bit-identical (rel err {err:.3g})"


def torch_dev():
    import torch

    assert torch.cuda.is_available()
    return torch


def to_dev(a: np.ndarray):
    torch = torch_dev()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream_ptr():
    torch = torch_dev()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def assert_token_parity(gpu_tokens, ora: dict, n_prompt: int):
    """Identical greedy ids; a divergence is accepted only where the oracle
    shows a near-tie (< NEAR_TIE) at or before the diverging step."""
    g, o = list(gpu_tokens), list(ora["tokens"])
    if g == o:
        return
    s = next(i for i in range(len(o)) if g[i] != o[i])
    gaps = []
    if "logit_gap" in ora:
        gaps.append(float(ora["logit_gap"][s]))
    if "gap" in ora:
        upto = n_prompt + s  # tokens processed before the id of step s was chosen
        gaps.append(float(ora["gap"][:upto].min()))
    assert gaps and min(gaps) < NEAR_TIE, f"greedy ids diverge at step {s} without a near-tie: {g} vs {o} {gaps}"


def agreeing_steps(gpu_tokens, ora_tokens) -> int:
    """Generated steps whose inputs agree: every step up to and including the
    first one whose chosen id differs (its hidden states and logits were
    formed from the same ids), or all of them."""
    for i, (a, b) in enumerate(zip(gpu_tokens, ora_tokens)):
        if a != b:
            return i + 1
    return len(ora_tokens)


def assert_prefix_parity(g: dict, ora: dict, n_prompt: int, per_layer: bool = False):
    """Hidden states, logits and routing records over the agreeing steps
    (all of them unless the ids diverge at a near-tie)."""
    s = agreeing_steps(g["tokens"], ora["tokens"])
    if per_layer:
        for l in range(g["hidden"].shape[1]):
            assert_matches(g["hidden"][:s, l], ora["hidden"][:s, l], f"layer {l}")
    else:
        assert_matches(g["hidden"][:s], ora["hidden"][:s])
    if "logits" in g and "logits" in ora:
        assert_matches(g["logits"][:s], ora["logits"][:s])
    if "sel" in g and "sel" in ora:
        n_tok = n_prompt + s - 1  # processed tokens whose inputs agree
        assert_trace_parity(g["sel"][:n_tok], ora["sel"][:n_tok], ora["gap"][:n_tok])


def assert_trace_parity(g_sel, o_sel, o_gap):
    """Routing records (ids in descending probability) are bit-exact wherever the
    oracle's top-(k+1) has no adjacent gap below NEAR_TIE."""
    ok = o_gap >= NEAR_TIE
    bad = np.any(g_sel != o_sel, axis=-1) & ok
    assert not bad.any(), (f"{int(bad.sum())} routing records differ away from near-ties; "
                           f"smallest oracle gap among them {float(o_gap[bad].min()):.3g}")


# ------------------------------------------------------------------ primitives
def test_quantize_q8k_bit_exact(gpu):
    rng = np.random.default_rng(11)
    x = rng.standard_normal(256 * 12).astype(np.float32)
    x[256:512] = 0.0  # an all-zero block
    x[512 + 17] = -7.5  # the largest magnitude is negative
    x[768:1024] = np.float32(0.5)  # every element ties for the largest magnitude
    x[1024 + 3], x[1024 + 200] = 4.0, -4.0  # tie between +max and -max: the first wins
    xd = to_dev(x)
    out = torch_dev().zeros(12 * 292, dtype=torch_dev().uint8, device="cuda")
    assert lib().nh_quantize_q8k(C.c_void_p(xd.data_ptr()), x.size, C.c_void_p(out.data_ptr()), stream_ptr()) == 0
    torch_dev().cuda.synchronize()
    assert out.cpu().numpy().tobytes() == oracle.quantize_q8k(x)


def test_exp_bit_exact(gpu):
    from tests.test_formats_oracle import exp_inputs

    x = exp_inputs()
    xd = to_dev(x)
    y = torch_dev().zeros(x.size, dtype=torch_dev().float32, device="cuda")
    assert lib().nh_exp_cw(C.c_void_p(xd.data_ptr()), x.size, C.c_void_p(y.data_ptr()), stream_ptr()) == 0
    torch_dev().cuda.synchronize()
    ref = np.array([oracle.olib().oracle_exp(float(v)) for v in x], dtype=np.float32)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.fixture(scope="module")
def mini_path(synth_dir):
    return synth.cached(synth.MINI, synth_dir)


def test_dequantize_bit_exact(gpu, mini_path):
    from gguf import GGUFReader

    r = GGUFReader(str(mini_path))
    for t in r.tensors:
        raw = np.asarray(t.data).view(np.uint8).reshape(-1)
        n0 = int(t.shape[0])
        rows = int(np.prod(t.shape)) // n0
        ref = oracle.dequant(int(t.tensor_type), raw.tobytes(), n0 * rows)
        wd = to_dev(np.concatenate([raw, np.zeros(256, np.uint8)]))
        y = torch_dev().zeros(n0 * rows, dtype=torch_dev().float32, device="cuda")
        assert lib().nh_dequantize(C.c_void_p(wd.data_ptr()), int(t.tensor_type), n0, rows,
                                   C.c_void_p(y.data_ptr()), stream_ptr()) == 0
        torch_dev().cuda.synchronize()
        assert np.array_equal(y.cpu().numpy(), ref), t.name


@pytest.mark.parametrize("K", [256, 512, 1024, 2048, 4096])
@pytest.mark.parametrize("qtype", [12, 14, 0])
def test_gemv_matches_oracle(gpu, K, qtype, tmp_path):
    # Weights from the synthetic writer's quantisers (a one-layer model of the shape).
    rows = 77
    spec = synth.SynthSpec(n_layers=1, n_embd=K, n_head=2, n_head_kv=2, n_ff=256, n_expert=2, n_expert_used=1,
                           n_vocab=rows, seed=K + qtype, quant=0 if qtype == 0 else 1)
    p = synth.write(spec, tmp_path / "w.gguf")
    from gguf import GGUFReader

    t = next(t for t in GGUFReader(str(p)).tensors if t.name == ("output.weight" if qtype != 12 else "token_embd.weight"))
    assert int(t.tensor_type) == qtype
    raw = np.asarray(t.data).view(np.uint8).reshape(-1)
    rng = np.random.default_rng(K)
    x = rng.standard_normal(K).astype(np.float32)
    ref = oracle.matvec(qtype, raw.tobytes(), K, rows, x)
    wd = to_dev(np.concatenate([raw, np.zeros(256, np.uint8)]))
    xd = to_dev(x)
    y = torch_dev().zeros(rows, dtype=torch_dev().float32, device="cuda")
    assert lib().nh_gemv(None, C.c_void_p(wd.data_ptr()), qtype, K, rows, C.c_void_p(xd.data_ptr()), None, 0.0,
                         C.c_void_p(y.data_ptr()), stream_ptr()) == 0
    torch_dev().cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) <= GEMV_TOL


# ------------------------------------------------------------------ whole-token path
@pytest.fixture(scope="module")
def mini_models(mini_path):
    m = nh.OlmoeModel.Load(str(mini_path))
    assert m is not None
    return m, oracle.OracleModel(str(mini_path))


@pytest.mark.parametrize("norm_topk", [False, True])
def test_mini_generate_matches_oracle(gpu, mini_models, norm_topk):
    m, om = mini_models
    oracle.set_threads(8)
    prompt = np.random.default_rng(5).integers(0, 1000, 12).tolist()
    n = 10
    ora = om.generate(prompt, n, norm_topk=norm_topk, mode=0, trace=True, hidden=True, logits=True)
    g = nh.generate_ex(m, prompt, n, norm_topk, trace=True, hidden=True, logits=True)
    assert_token_parity(g["tokens"], ora, len(prompt))
    assert_prefix_parity(g, ora, len(prompt))
    # Graph replay and eager launches run the same kernels: identical bits.
    e = nh.generate_ex(m, prompt, n, norm_topk, use_graph=False, hidden=True)
    assert e["tokens"] == g["tokens"]
    assert np.array_equal(e["hidden"], g["hidden"])


def test_mini_gqa_and_all_experts(gpu, synth_dir):
    p = synth.cached(synth.MINI_GQA, synth_dir)
    m = nh.OlmoeModel.Load(str(p))
    om = oracle.OracleModel(str(p))
    prompt = [5, 9, 100, 700, 3]
    ora = om.generate(prompt, 8, mode=0, trace=True, hidden=True)
    g = nh.generate_ex(m, prompt, 8, False, hidden=True)
    assert_token_parity(g["tokens"], ora, len(prompt))
    assert_matches(g["hidden"], ora["hidden"])


def test_top5_tool_matches_oracle_full_forward(gpu, mini_models, mini_path, capsys):
    """olmoe_forward (olmoe_forward_main.cc:17-65): the last position's logits
    equal the oracle's full-sequence forward bit for bit, and the printed top 5
    are its five largest."""
    from nuthatch_b200 import olmoe_forward

    m, om = mini_models
    toks = np.random.default_rng(21).integers(0, 1000, 9).tolist()
    full = om.forward(toks)[-1]
    assert np.array_equal(olmoe_forward.last_logits(m, toks), full)
    best = olmoe_forward.top_k(full)
    assert olmoe_forward.main(["olmoe_forward", str(mini_path)] + [str(t) for t in toks]) == 0
    out = capsys.readouterr().out.splitlines()
    assert out[0].startswith("loaded: layers=2 ") and out[1] == "top-5 next-token logits (after pos 8):"
    assert out[2:] == [f"  tok {i:<6d} logit {v:.4f}" for i, v in best]


def test_long_context_split_attention(gpu, mini_models):
    # A prompt longer than one attention split (256 positions) exercises the
    # multi-CTA softmax combine.
    m, om = mini_models
    prompt = np.random.default_rng(9).integers(0, 1000, 600).tolist()
    ora = om.generate(prompt, 6, mode=0, trace=True, hidden=True, logits=True)
    g = nh.generate_ex(m, prompt, 6, False, hidden=True, logits=True)
    assert_token_parity(g["tokens"], ora, len(prompt))
    assert_matches(g["hidden"], ora["hidden"])
    assert_matches(g["logits"], ora["logits"])


# ------------------------------------------------------------------ the reference's own anchors
@pytest.fixture(scope="module")
def tiny_path(tmp_path_factory):
    return write_tiny_olmoe(tmp_path_factory.mktemp("tiny") / "gen_olmoe.gguf")


def test_reference_anchors_on_tiny_fixture(gpu, tiny_path):
    m = nh.OlmoeModel.Load(tiny_path)
    assert m is not None and m.config().n_vocab == 16
    om = oracle.OracleModel(tiny_path)
    # GreedyDeterministicInVocab
    a = nh.GreedyGenerate(m, [3, 7], 4, True)
    assert len(a) == 4 and all(0 <= t < 16 for t in a)
    assert a == nh.GreedyGenerate(m, [3, 7], 4, True)
    # CachedMatchesUncached (both norm_topk settings), and both equal the oracle.
    for nt in (False, True):
        ref = nh.GreedyGenerate(m, [3, 7, 2, 5], 6, nt)
        assert ref == nh.GreedyGenerateCached(m, [3, 7, 2, 5], 6, nt)
        assert ref == om.generate([3, 7, 2, 5], 6, norm_topk=nt, mode=1)["tokens"]
    # CachedTraceWellFormedAndReplayable
    tr = nh.RoutingTrace()
    gen = nh.GreedyGenerateCachedTrace(m, [3, 7, 2], 5, False, tr)
    assert gen == nh.GreedyGenerateCached(m, [3, 7, 2], 5, False)
    assert tr.n_layers == 2 and tr.n_expert == 4 and tr.records
    assert len(tr.records) % 2 == 0
    for r in tr.records:
        assert len(r.experts) == 2 and r.layer < 2 and all(e < 4 for e in r.experts)
    st = nh.Replay(tr, nh.LruPolicy(tr.n_layers, 2))
    assert st.accesses == sum(len(r.experts) for r in tr.records) and st.hits + st.misses == st.accesses


def test_reference_streaming_matches_resident(gpu, tiny_path):
    sm = nh.StreamingModel.Load(tiny_path)
    full = nh.OlmoeModel.Load(tiny_path)
    assert sm is not None and full is not None
    for nt in (False, True):
        streamed = nh.StreamingGenerate(sm, [3, 7, 2], 6, nt, 3)
        assert streamed == nh.GreedyGenerateCached(full, [3, 7, 2], 6, nt)
    assert nh.StreamingGenerate(sm, [], 4, False, 3) == []
    assert nh.StreamingGenerate(sm, [1], 0, False, 3) == []


def test_reference_slot_cache_kat(gpu, tmp_path):
    path = write_slot_fixture(tmp_path / "slots.gguf")
    rd = nh.ExpertReader.Open(path)
    cfg = nh.OlmoeConfig(1, 8, 1, 1, 4, 5, 2, 0, 0, 10000.0, 1e-5)
    c = nh.ExpertSlotCache.Create(cfg, 0, 2, rd)
    assert c is not None
    name = "blk.0.ffn_gate_exps.weight"
    eb = rd.ExpertBytes(name)

    def slot_matches(expert, slot):
        assert c.slot_bytes(0, slot, eb) == rd.ReadExpert(name, expert)

    m = c.Ensure([0, 1])
    assert (c.misses(), c.hits()) == (2, 0)
    slot_matches(0, m[0])
    slot_matches(1, m[1])
    assert m[0] != m[1]
    c.Ensure([0, 1])
    assert (c.hits(), c.misses()) == (2, 2)
    c.Ensure([0])
    assert c.hits() == 3
    m2 = c.Ensure([2])
    assert c.misses() == 3
    slot_matches(2, m2[2])
    c.Ensure([0])
    assert c.hits() == 4
    c.Ensure([1])
    assert c.misses() == 4
    # DedupWithinBatchAndBadInputs
    c3 = nh.ExpertSlotCache.Create(cfg, 0, 3, rd)
    assert len(c3.Ensure([3, 3, 3])) == 1 and c3.misses() == 1
    assert nh.ExpertSlotCache.Create(cfg, 0, 0, rd) is None
    assert nh.ExpertSlotCache.Create(cfg, 9, 3, rd) is None


# ------------------------------------------------------------------ streaming
@pytest.mark.parametrize("capacity", [4, 8, 16])
def test_mini_streaming_lru_matches_oracle(gpu, mini_path, mini_models, capacity):
    m, om = mini_models
    sm = nh.StreamingModel.Load(str(mini_path))
    prompt = np.random.default_rng(21).integers(0, 1000, 10).tolist()
    s = nh.streaming_generate_ex(sm, prompt, 12, False, capacity, trace=True)
    ora = om.stream_generate(prompt, 12, False, capacity)
    resident = nh.GreedyGenerateCached(m, prompt, 12, False)
    assert s["tokens"] == resident
    assert s["tokens"] == ora["tokens"]
    assert np.array_equal(s["hits"], ora["hits"]) and np.array_equal(s["misses"], ora["misses"])
    # The counts are those of LruPolicy replaying the same routing (capacity >= k).
    tr = nh.RoutingTrace(m.config().n_layers, m.config().n_expert,
                         [nh.RoutingRecord(t, l, s["sel"][t, l].tolist()) for t in range(s["sel"].shape[0])
                          for l in range(s["sel"].shape[1])])
    st = nh.Replay(tr, nh.LruPolicy(tr.n_layers, capacity))
    assert st.hits == int(s["hits"].sum()) and st.misses == int(s["misses"].sum())


@pytest.mark.parametrize("capacity", [2, 4, 8])
def test_mini_streaming_learned_pin_matches_oracle(gpu, mini_path, mini_models, capacity):
    m, om = mini_models
    cfg = m.config()
    sm = nh.StreamingModel.Load(str(mini_path))
    # Calibration: usage histogram from a resident run on a different prompt.
    cal = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(m, np.random.default_rng(77).integers(0, 1000, 16).tolist(), 16, False, cal)
    usage = nh.BuildUsage(cal, cfg.n_expert).counts
    prompt = np.random.default_rng(21).integers(0, 1000, 10).tolist()
    pin = (capacity * 3 + 3) // 4 if capacity > 1 else 1
    s = nh.streaming_generate_ex(sm, prompt, 12, False, capacity, policy="learned_pin", usage=usage, trace=True)
    ora = om.stream_generate(prompt, 12, False, capacity, policy=1, pin_slots=pin, usage=usage)
    assert s["tokens"] == nh.GreedyGenerateCached(m, prompt, 12, False)
    assert s["tokens"] == ora["tokens"]
    assert np.array_equal(s["hits"], ora["hits"]) and np.array_equal(s["misses"], ora["misses"])
    tr = nh.RoutingTrace(cfg.n_layers, cfg.n_expert,
                         [nh.RoutingRecord(t, l, s["sel"][t, l].tolist()) for t in range(s["sel"].shape[0])
                          for l in range(cfg.n_layers)])
    st = nh.Replay(tr, nh.LearnedPinPolicy(cfg.n_layers, pin, capacity - pin, nh.UsageHistogram(usage)))
    assert st.hits == int(s["hits"].sum())


# ------------------------------------------------------------------ full OLMoE-1B-7B shape
@pytest.fixture(scope="module")
def olmoe_path(synth_dir):
    return synth.cached(synth.OLMOE_1B7B, synth_dir)


def test_olmoe_1b7b_resident_decode_matches_oracle(gpu, olmoe_path):
    """Resident bs1 decode: 16-token seeded prompt, 24 greedy ids."""
    m = nh.OlmoeModel.Load(str(olmoe_path))
    assert m is not None
    cfg = m.config()
    assert (cfg.n_layers, cfg.n_embd, cfg.n_expert, cfg.n_vocab) == (16, 2048, 64, 50304)
    om = oracle.OracleModel(str(olmoe_path))
    import os

    oracle.set_threads(min(32, os.cpu_count() or 8))
    prompt = np.random.default_rng(1).integers(0, cfg.n_vocab, 16).tolist()
    ora = om.generate(prompt, 24, mode=0, trace=True, hidden=True, logits=True)
    g = nh.generate_ex(m, prompt, 24, False, trace=True, hidden=True, logits=True)
    assert_token_parity(g["tokens"], ora, len(prompt))
    assert_prefix_parity(g, ora, len(prompt), per_layer=True)


def test_olmoe_streaming_fresh_learned_pin_pools_match_resident(gpu, synth_dir):
    """Full-width streaming with freshly created learned-pin slot pools (pinned
    experts preloaded at creation) and with reused pools: tokens equal the
    resident decode and hit counts are identical across repeats.  Guards the
    ordering of the pool zeroing before the preload copies."""
    path = synth.cached(synth.OLMOE_1B7B_SKEW, synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    cfg = m.config()
    cal = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(m, np.random.default_rng(7).integers(0, cfg.n_vocab, 16).tolist(), 16, False, cal)
    usage = nh.BuildUsage(cal, cfg.n_expert).counts
    prompt = np.random.default_rng(8).integers(0, cfg.n_vocab, 16).tolist()
    ref = nh.GreedyGenerateCached(m, prompt, 16, False)
    del m
    for cap in (4, 8):
        pin = (cap * 3 + 3) // 4
        hits = set()
        for trial in range(2):  # two freshly loaded models
            sm = nh.StreamingModel.Load(str(path))
            for call in range(2):  # the first call creates the pools, the second reuses them
                r = nh.streaming_generate_ex(sm, prompt, 16, False, cap, policy="learned_pin", pin_slots=pin,
                                             usage=usage)
                assert r["tokens"] == ref, (cap, trial, call)
                hits.add(int(r["hits"].sum()))
            sm.close()
        assert len(hits) == 1, (cap, hits)
