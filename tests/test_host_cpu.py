"""CPU: the C-ABI library's exports, and the host-side logic behind it
(cache policies and sweeps, routing-trace formats, GGUF probing, the expert
reader) against the reference's own compiled code (oracle/_ref) and the
golden fixture it produced (tests/golden/policy_replay.json)."""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import re
from pathlib import Path

import numpy as np
import pytest
from gguf import GGUFReader

import nuthatch_b200 as nh
import oracle
from nuthatch_b200 import synth
from nuthatch_b200._lib import LIB_PATH, NhConfig, lib
from tests.golden.make_policy_golden import LRU_BUDGETS, OS_CAPACITIES, pin_has_tie, traces

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = json.loads((ROOT / "tests" / "golden" / "policy_replay.json").read_text())


def _declared(header: Path) -> list[str]:
    """Function names declared in a C header (prototypes ending in ');')."""
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    names = []
    for m in re.finditer(r"\b(nh_\w+)\s*\(([^;{}]*)\)\s*;", text):
        names.append(m.group(1))
    return sorted(set(names))


@pytest.mark.parametrize("header", ["nh_kernels.h", "nh_api.h"])
def test_library_exports_every_declared_symbol(header):
    names = _declared(ROOT / "include" / header)
    assert len(names) > 10
    so = C.CDLL(str(LIB_PATH))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def test_product_library_has_no_phase_trace_hooks():
    """The per-CTA phase timestamps exist only in the diagnostic build
    (python -m nuthatch_b200.build --phase-trace); the product library's
    kernels record nothing and export no ring setters."""
    so = C.CDLL(str(LIB_PATH))
    units = ("gemv", "attention", "moe", "misc", "grouped_tc", "batch")
    assert not any(hasattr(so, f"nh_phase_trace_set_{u}") for u in units)


def _trace(name):
    L, E, recs = traces()[name]
    return nh.RoutingTrace(L, E, [nh.RoutingRecord(t, l, ex) for t, l, ex in recs])


@pytest.mark.parametrize("name", sorted(GOLDEN["traces"]))
def test_policy_replay_matches_reference_golden(name):
    g = GOLDEN["traces"][name]
    tr = _trace(name)
    assert len(tr.records) == g["n_records"]
    flat = [(r.layer, r.experts) for r in tr.records]
    for b, hits in g["lru"].items():
        st = nh.Replay(tr, nh.LruPolicy(tr.n_layers, int(b)))
        assert (st.hits, st.accesses) == (hits, g["accesses"]), ("lru", b)
        assert oracle.replay(0, flat, tr.n_layers, tr.n_expert, int(b))[0] == hits
    for c, hits in g["os"].items():
        assert nh.Replay(tr, nh.OsPageCachePolicy(int(c))).hits == hits, ("os", c)
        assert oracle.replay(1, flat, tr.n_layers, tr.n_expert, int(c))[0] == hits
    usage = nh.BuildUsage(tr, tr.n_expert)
    for key, hits in g["learned_pin"].items():
        pin, lru = (int(x) for x in key.split(","))
        st = nh.Replay(tr, nh.LearnedPinPolicy(tr.n_layers, pin, lru, usage))
        assert st.hits == hits, ("learned_pin", key)
        assert oracle.replay(2, flat, tr.n_layers, tr.n_expert, pin, lru)[0] == hits


def _random_trace(seed, L=3, E=24, k=6, n_tok=120):
    rng = np.random.default_rng(seed)
    p = rng.dirichlet(np.full(E, 0.4))
    recs = [(t, l, rng.choice(E, k, replace=False, p=p).tolist()) for t in range(n_tok) for l in range(L)]
    return L, E, recs


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref (reference policy code) not built")
@pytest.mark.parametrize("seed", range(6))
def test_policy_replay_matches_reference_live(seed):
    L, E, recs = _random_trace(seed)
    tr = nh.RoutingTrace(L, E, [nh.RoutingRecord(t, l, ex) for t, l, ex in recs])
    flat = [(l, ex) for _, l, ex in recs]
    for b in (1, 3, 6, 12, 24):
        assert nh.Replay(tr, nh.LruPolicy(L, b)).hits == oracle.replay(0, flat, L, E, b, use_ref=True)[0]
    for c in (6, 20, 72):
        assert nh.Replay(tr, nh.OsPageCachePolicy(c)).hits == oracle.replay(1, flat, L, E, c, use_ref=True)[0]
    usage = nh.BuildUsage(tr, E)
    for b in (4, 8, 12):
        pin = int(math.ceil(0.75 * b))
        if pin_has_tie(recs, L, pin):
            continue  # the reference breaks count ties by hash-map order
        ours = nh.Replay(tr, nh.LearnedPinPolicy(L, pin, b - pin, usage)).hits
        assert ours == oracle.replay(2, flat, L, E, pin, b - pin, use_ref=True)[0]


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref (reference policy code) not built")
def test_sweep_budgets_matches_reference():
    L, E, recs = traces()["zipf_l4_e64_k8"]
    tr = nh.RoutingTrace(L, E, [nh.RoutingRecord(t, l, ex) for t, l, ex in recs])
    budgets = [4, 8, 16]
    ours = nh.SweepBudgets(tr, budgets)
    ref = oracle.ref_sweep_budgets([(l, ex) for _, l, ex in recs], L, E, budgets)
    assert len(ours) == len(ref) == 3
    for (b, learned, lru, osp), (rl, rr, ro) in zip(ours, ref):
        assert lru == pytest.approx(rr, abs=0) and osp == pytest.approx(ro, abs=0)
        if not pin_has_tie(recs, L, int(math.ceil(0.75 * b))):
            assert learned == pytest.approx(rl, abs=0)


def test_routing_trace_binary_round_trip_and_reference_reader(tmp_path):
    tr = _trace("phased_l3_e32_k8")
    path = tmp_path / "t.bin"
    assert nh.WriteRoutingTrace(tr, str(path))
    back = nh.RoutingTrace()
    assert nh.ReadRoutingTrace(str(path), back)
    assert (back.n_layers, back.n_expert) == (tr.n_layers, tr.n_expert)
    assert [(r.token, r.layer, r.experts) for r in back.records] == [(r.token, r.layer, r.experts) for r in tr.records]
    if oracle.ref_available():
        nl, ne, recs = oracle.ref_read_trace(str(path), False)
        assert (nl, ne) == (tr.n_layers, tr.n_expert)
        assert recs == [(r.token, r.layer, r.experts) for r in tr.records]


def test_routing_trace_rejects_truncated_and_garbage(tmp_path):
    tr = _trace("uniform_l2_e16_k4")
    good = tmp_path / "good.bin"
    assert nh.WriteRoutingTrace(tr, str(good))
    raw = good.read_bytes()
    for i, cut in enumerate((8, len(raw) // 2, len(raw) - 3)):
        bad = tmp_path / f"cut{i}.bin"
        bad.write_bytes(raw[:cut])
        assert not nh.ReadRoutingTrace(str(bad), nh.RoutingTrace()), cut
        if oracle.ref_available():
            assert oracle.ref_read_trace(str(bad), False) is None
    junk = tmp_path / "junk.bin"
    junk.write_bytes(b"not a trace at all")
    assert not nh.ReadRoutingTrace(str(junk), nh.RoutingTrace())


def test_routing_trace_text_format(tmp_path):
    # One record per line: layer, then the selected experts.  Lines without a
    # layer number are skipped; a line with a layer but no experts consumes a
    # token number and is dropped (routing_trace.cc:83-104).
    path = tmp_path / "t.txt"
    path.write_text("0 3 7 1\n1 2 2 9\n\n# comment\n0 5 4\n1\n2 8 0\n")
    ours = nh.RoutingTrace()
    assert nh.ReadRoutingTraceText(str(path), ours)
    recs = [(r.token, r.layer, r.experts) for r in ours.records]
    assert recs == [(0, 0, [3, 7, 1]), (1, 1, [2, 2, 9]), (2, 0, [5, 4]), (4, 2, [8, 0])]
    assert (ours.n_layers, ours.n_expert) == (3, 10)
    if oracle.ref_available():
        assert oracle.ref_read_trace(str(path), True) == (3, 10, recs)


@pytest.fixture(scope="module")
def mini(synth_dir):
    return synth.cached(synth.MINI, synth_dir)


def test_gguf_probe_reads_the_config_without_a_gpu(mini, tmp_path):
    c = NhConfig()
    n = lib().nh_gguf_probe(str(mini).encode(), C.byref(c))
    s = synth.MINI
    assert n > 0
    assert (c.n_layers, c.n_embd, c.n_head, c.n_head_kv, c.n_ff, c.n_expert, c.n_expert_used, c.n_vocab) == (
        s.n_layers, s.n_embd, s.n_head, s.n_head_kv, s.n_ff, s.n_expert, s.n_expert_used, s.n_vocab)
    assert c.rms_eps == pytest.approx(s.rms_eps) and c.rope_freq_base == pytest.approx(s.rope_freq_base)
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"GGUF" + b"\x00" * 4)
    assert lib().nh_gguf_probe(str(junk).encode(), C.byref(c)) < 0
    assert lib().nh_gguf_probe(str(tmp_path / "missing.gguf").encode(), C.byref(c)) < 0


def test_expert_reader_slices_match_gguf_py(mini):
    r = nh.ExpertReader.Open(str(mini))
    assert r is not None
    g = GGUFReader(str(mini))
    for name in ("blk.0.ffn_gate_exps.weight", "blk.1.ffn_down_exps.weight"):
        t = next(t for t in g.tensors if t.name == name)
        raw = np.asarray(t.data).view(np.uint8).reshape(-1)
        per = raw.size // int(t.shape[-1])
        assert r.ExpertBytes(name) == per
        for e in (0, 5, int(t.shape[-1]) - 1):
            assert r.ReadExpert(name, e) == raw[e * per:(e + 1) * per].tobytes()
    assert r.ExpertBytes("no.such.tensor") == 0


# The reference's recorded granite-3-MoE routing trace, found through the
# reference checkout named by NUTHATCH_REFERENCE (the test skips without it).
GRANITE = (Path(os.environ["NUTHATCH_REFERENCE"]) / "data" / "granite3moe.trace.txt"
           if os.environ.get("NUTHATCH_REFERENCE") else None)


@pytest.mark.skipif(GRANITE is None or not GRANITE.exists() or not oracle.ref_available(),
                    reason="the reference's granite routing trace is not available")
def test_granite_trace_sweep_matches_reference_and_published_rates():
    """The reference's recorded granite-3-MoE routing trace: LRU and OS page
    cache hit rates equal the reference's compiled sweep exactly; learned pin
    (whose count ties the reference breaks by hash-map order) within 0.2 pp;
    all three within 0.15 pp of the published table (bench-log.md:230-233)."""
    tr = nh.RoutingTrace()
    assert nh.ReadRoutingTraceText(str(GRANITE), tr)
    budgets = [4, 8, 12, 16]
    ours = nh.SweepBudgets(tr, budgets)
    ref = oracle.ref_sweep_budgets([(r.layer, r.experts) for r in tr.records], tr.n_layers, tr.n_expert, budgets)
    published = {4: (22.4, 4.7, 0.0), 8: (40.1, 30.4, 30.2), 12: (56.7, 47.7, 45.2), 16: (71.6, 62.7, 61.5)}
    for (b, learned, lru, osp), (rl, rr, ro) in zip(ours, ref):
        assert lru == rr and osp == ro, b
        assert abs(learned - rl) <= 0.002, b
        for got, want in zip((learned, lru, osp), published[b]):
            assert abs(100 * got - want) <= 0.15, (b, 100 * got, want)


def test_moe_layer_declines_uncovered_shapes_before_any_launch():
    """nh_moe_layer validates on the host and returns NH_E_ARG / NH_E_TYPE,
    launching nothing, where the fused kernel does not cover the layer (the
    engine then runs the router, gate/up and down kernels); the fake device
    pointers below are never dereferenced."""
    from nuthatch_b200._lib import NhMoeLayer

    fake = 1 << 20  # 16-byte aligned, never touched
    base = dict(state=fake, h=fake, ffn_norm=fake, eps=1e-5, router=fake, n_embd=2048, n_ff=1024, n_expert=64, k=8,
                n_layers=16, gate=fake, tg=12, gate_nb2=1024 * 8 * 144, up=fake, tu=12, up_nb2=1024 * 8 * 144,
                down=fake, td=14, down_nb2=2048 * 4 * 210, sel=fake, wts=fake, ff=fake, scratch=fake)

    def rc(**kw):
        a = NhMoeLayer(**{**base, **kw})
        return lib().nh_moe_layer(C.byref(a), None)

    assert lib().nh_moe_layer(None, None) == -1
    assert rc(scratch=None) == -1
    assert rc(tg=0) == -3 and rc(td=0) == -3               # F32 experts: the separate kernels
    assert rc(n_embd=2304) == -1                           # n_embd/256 = 9
    assert rc(n_ff=768) == -1                              # n_ff/256 = 3
    assert rc(n_ff=2048, k=8) == -1                        # 32/(n_ff/256) = 4 row groups for 8 experts
    assert rc(k=65) == -1 and rc(n_expert=300) == -1
    assert rc(router=fake + 4) == -1                       # router rows are bulk-copied
    assert rc(gate=fake + 8) == -1                         # Q4_K rows are read 16 bytes at a time
    assert lib().nh_moe_layer_scratch_bytes(64) >= 64 + 4 * 64


def test_calibrated_sweep_persists_through_trace_files(tmp_path):
    """The learned-pin calibration lifecycle: a calibration trace written with
    WriteRoutingTrace and read back gives the same usage histogram; the
    out-of-sample sweep with calibration == evaluation equals SweepBudgets,
    and learned pin calibrated on another trace is scored on the evaluation
    trace (LRU and OS columns do not depend on the calibration)."""
    cal = _trace("zipf_l4_e64_k8")
    L, E, recs = _random_trace(3, L=cal.n_layers, E=cal.n_expert, k=8, n_tok=150)
    ev = nh.RoutingTrace(L, E, [nh.RoutingRecord(t, l, ex) for t, l, ex in recs])
    path = tmp_path / "cal.bin"
    assert nh.WriteRoutingTrace(cal, str(path))
    back = nh.RoutingTrace()
    assert nh.ReadRoutingTrace(str(path), back)
    assert np.array_equal(nh.BuildUsage(back, E).counts, nh.BuildUsage(cal, E).counts)
    budgets = [4, 8, 16]
    assert nh.SweepBudgetsCalibrated(cal, cal, budgets) == nh.SweepBudgets(cal, budgets)
    out = nh.SweepBudgetsCalibrated(back, ev, budgets)
    ins = nh.SweepBudgets(ev, budgets)
    assert [r[2:] for r in out] == [r[2:] for r in ins]
    for (b, learned, _, _) in out:
        pin = int(math.ceil(0.75 * b))
        want = nh.Replay(ev, nh.LearnedPinPolicy(L, pin, b - pin, nh.BuildUsage(back, E))).hit_rate()
        assert learned == pytest.approx(want, abs=0)


def test_top5_tool_usage_and_tie_order(capsys):
    """olmoe_forward (olmoe_forward_main.cc:17-65): usage on too few
    arguments; the top 5 ordered by logit, ties to the lower id."""
    from nuthatch_b200 import olmoe_forward

    assert olmoe_forward.main(["olmoe_forward", "model.gguf"]) == 1
    assert "usage:" in capsys.readouterr().err
    lg = np.array([0.5, 2.0, 2.0, -1.0, 3.0, 0.5, 2.0], dtype=np.float32)
    assert olmoe_forward.top_k(lg) == [(4, 3.0), (1, 2.0), (2, 2.0), (6, 2.0), (0, 0.5)]


def _plan_waves_restated(sel, n_expert, per, pinned, first, count):
    """The wave rules written out plainly: served unpinned experts in order of
    first selection, `per` to a wave; selected pinned experts join wave 0
    after its unpinned ones."""
    waves, wave_of, pins = [], [-1] * n_expert, []
    for e in sel:
        if not first <= e < first + count or wave_of[e] >= 0:
            continue
        if e in pinned:
            wave_of[e] = 0
            pins.append(e)
            continue
        if not waves or len(waves[-1]) == per:
            waves.append([])
        waves[-1].append(e)
        wave_of[e] = len(waves) - 1
    if not waves:
        waves.append([])
    waves[0] += pins
    return waves, wave_of


def test_wave_plan_matches_restated_rules():
    """Batched streaming waves (nh_plan_waves, nh_group_wave_pairs) on seeded
    selections: mini, OLMoE and Granite expert counts, with pinned experts and
    expert-parallel shards; every pick of a served expert lands in exactly one
    wave's pairs, in slot order and (token, pick) order within a slot."""
    rng = np.random.default_rng(17)
    for n_expert, k, n_tok in ((16, 4, 6), (64, 8, 64), (32, 8, 32), (8, 8, 3)):
        for world in (1, 2, 4):
            for rank in range(world):
                count = n_expert // world
                first = rank * count
                for per in (1, 2, 5, 8):
                    sel = np.stack([rng.choice(n_expert, k, replace=False) for _ in range(n_tok)]).ravel()
                    pinned = set(rng.choice(np.arange(first, first + count), min(2, count), replace=False).tolist())
                    waves, wave_of = nh.plan_waves(sel, n_expert, per, pinned=sorted(pinned), shard=(first, count))
                    assert (waves, wave_of) == _plan_waves_restated(sel.tolist(), n_expert, per, pinned, first,
                                                                    count)
                    assert all(len([e for e in w if e not in pinned]) <= per for w in waves)
                    # Slots as an Ensure would give them: one per expert of the wave.
                    covered = []
                    for w, ids in enumerate(waves):
                        slot_of = [-1] * n_expert
                        for s, e in enumerate(ids):
                            slot_of[e] = s
                        off, cnt, act, out = nh.group_wave_pairs(sel, k, wave_of, w, slot_of, max(len(ids), 1))
                        want = [j for s in range(len(ids)) for j in range(sel.size) if sel[j] == ids[s]]
                        assert out == want and act == [j // k for j in want]
                        assert off == [sum(cnt[:s]) for s in range(len(cnt))]
                        covered += out
                    served = [j for j in range(sel.size) if first <= sel[j] < first + count]
                    assert sorted(covered) == served


def test_wave_plan_rejections():
    with pytest.raises(nh.NhError):
        nh.plan_waves([0, 16], 16, 2)                 # a selection outside [0, n_expert)
    with pytest.raises(nh.NhError):
        nh.plan_waves([0, 1], 16, 0)                  # unpinned experts and no LRU slot
    waves, _ = nh.plan_waves([3, 3], 16, 0, pinned=[3])  # pinned only: no LRU slot needed
    assert waves == [[3]]
    assert nh.plan_waves([5, 6], 16, 4, shard=(8, 8))[0] == [[]]  # nothing served here: one empty wave
    with pytest.raises(nh.NhError):
        nh.group_wave_pairs([1, 2], 2, [0] * 16, 0, [-1] * 16, 2)  # an expert of the wave without a slot


REF_TRACE_REPLAY = ROOT / "oracle" / "_ref" / "trace_replay"


def _tool_rows(argv, capsys):
    from nuthatch_b200 import trace_replay

    assert trace_replay.main(argv) == 0
    return capsys.readouterr().out.splitlines()


def _rows_with(lines, suffix):
    return [ln for ln in lines if ln.rstrip().endswith(suffix)]


def test_trace_replay_tool_budget_and_pin_curves(tmp_path, capsys):
    """trace_replay (trace_replay_main.cc): binary and text traces, default
    and given budgets, and the pin/LRU split; the rows carry SweepBudgets /
    SweepPinRatio's numbers in the reference tool's row formats."""
    tr = _trace("zipf_l4_e64_k8")
    path = tmp_path / "t.bin"
    assert nh.WriteRoutingTrace(tr, str(path))
    text = tmp_path / "t.txt"
    text.write_text("".join(f"{r.layer} {' '.join(map(str, r.experts))}\n" for r in tr.records))
    head = f"trace: {len(tr.records)} records, 4 layers, 64 experts/layer"
    for argv, want in ((["trace_replay", str(path)], [4, 8, 12, 16, 24, 32]),
                       (["trace_replay", "--text", str(text), "6", "20"], [6, 20])):
        out = _tool_rows(argv, capsys)
        assert out[0] == head
        rows = _rows_with(out, " pp")
        assert len(rows) == len(want)
        for ln, (b, learned, lru, osp) in zip(rows, nh.SweepBudgets(tr, want)):
            assert ln == (f"{b:6d}    {100 * learned:6.1f}%   {100 * lru:6.1f}%   {100 * osp:6.1f}%    "
                          f"{100 * (learned - lru):+.1f} pp")
    out = _tool_rows(["trace_replay", str(path), "pin", "8"], capsys)
    rows = _rows_with(out, "%")
    assert rows == [f"{p:5d} {lru:4d}   {100 * h:6.1f}%" for p, lru, h in nh.SweepPinRatio(tr, 8)]


def test_trace_replay_tool_rejections(tmp_path, capsys):
    from nuthatch_b200 import trace_replay

    assert trace_replay.main(["trace_replay"]) == 1
    assert trace_replay.main(["trace_replay", str(tmp_path / "missing.bin")]) == 1
    assert "read trace failed" in capsys.readouterr().err
    tr = _trace("uniform_l2_e16_k4")
    path = tmp_path / "t.bin"
    assert nh.WriteRoutingTrace(tr, str(path))
    assert trace_replay.main(["trace_replay", str(path), "eight"]) == 1
    assert trace_replay.main(["trace_replay", str(path), "pin", "-2"]) == 1


@pytest.mark.skipif(not REF_TRACE_REPLAY.exists(), reason="oracle/_ref/trace_replay (the reference tool) not built")
@pytest.mark.parametrize("name", ["zipf_l4_e64_k8", "phased_l3_e32_k8"])
def test_trace_replay_tool_rows_equal_reference_tool(tmp_path, capsys, name):
    """The numeric rows equal the reference's own trace_replay compiled from
    its sources, except the learned column where the pin cut falls on a count
    tie (the reference breaks it by hash-map order, this build by expert id)."""
    import subprocess

    L, E, recs = traces()[name]
    tr = _trace(name)
    path = tmp_path / "t.bin"
    assert nh.WriteRoutingTrace(tr, str(path))
    exact = 0
    for args in (["4", "8", "16", "24"], ["pin", "12"]):
        ref = subprocess.run([str(REF_TRACE_REPLAY), str(path), *args], capture_output=True, text=True, timeout=60)
        assert ref.returncode == 0, ref.stderr
        theirs = _rows_with(ref.stdout.splitlines(), " pp" if args[0] != "pin" else "%")
        ours = _rows_with(_tool_rows(["trace_replay", str(path), *args], capsys), " pp" if args[0] != "pin" else "%")
        assert len(ours) == len(theirs) > 0
        assert ref.stdout.splitlines()[0] == f"trace: {len(recs)} records, {L} layers, {E} experts/layer"
        for a, b in zip(ours, theirs):
            pin = int(b.split()[0]) if args[0] == "pin" else int(math.ceil(0.75 * int(b.split()[0])))
            if pin_has_tie(recs, L, pin):
                # Pin rows: the split only; budget rows: the lru and os columns.
                cols = slice(0, 2) if args[0] == "pin" else slice(2, 4)
                assert a.split()[cols] == b.split()[cols]
                continue
            assert a == b
            exact += 1
    assert exact >= 4
