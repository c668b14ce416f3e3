"""Phase timelines of the decode kernels from the diagnostic library build.

    python -m nuthatch_b200.build --phase-trace
    python -m nuthatch_b200.phase_trace decode      # batch-1 resident decode (configuration 1)
    python -m nuthatch_b200.phase_trace prefill     # tcgen05 products of a 1024-token prefill
    python -m nuthatch_b200.phase_trace streaming   # two-phase streaming decode, budget 32
    python -m nuthatch_b200.phase_trace batched     # mma.sync grouped products of a bs64 decode step
    python -m nuthatch_b200.phase_trace battention  # batched decode attention at 2048-token contexts

The diagnostic library records, per CTA of the stamped kernels, %globaltimer
stamps at fixed points (kernel entry, after griddepcontrol.wait, after the
activation preparation, after the router selection, ...; see
csrc/kernels/phase_trace.cuh) into a device ring.  The product library has
no stamps; run times under this build are a few percent longer.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import sys
import time

import numpy as np

UNITS = ("gemv", "attention", "moe", "misc", "grouped_tc", "batch")
KERNELS = {1: "gemv3", 2: "attention", 3: "moe_fused", 4: "embed", 5: "lm_head", 6: "grouped_tc", 7: "router",
           8: "gate_up", 9: "down", 10: "batch_mma"}
RING = 1 << 20  # records (kPhaseTraceCap); 128 bytes each


class Ring:
    """The device ring and its counter, registered with every stamped unit."""

    def __init__(self, units=UNITS):
        import torch

        from ._lib import lib

        self.torch = torch
        self.buf = torch.zeros(RING * 16, dtype=torch.int64, device="cuda")
        self.count = torch.zeros(1, dtype=torch.int32, device="cuda")
        L = lib()
        for unit in units:
            fn = getattr(L, f"nh_phase_trace_set_{unit}")
            fn.argtypes = [C.c_void_p, C.c_void_p]
            fn.restype = None
            fn(C.c_void_p(self.buf.data_ptr()), C.c_void_p(self.count.data_ptr()))

    def reset(self):
        self.torch.cuda.synchronize()
        self.buf.zero_()
        self.count.zero_()
        self.torch.cuda.synchronize()

    def records(self):
        """(kernel ids, stamps [n][12]) in entry order."""
        self.torch.cuda.synchronize()
        n = int(self.count.item())
        if n >= RING:
            raise SystemExit(f"{n} records overflow the ring of {RING}: trace a shorter run")
        raw = self.buf[: n * 16].cpu().numpy().view(np.uint64).reshape(n, 16).astype(np.int64)
        raw = raw[raw[:, 0] != 0]
        kid, t = raw[:, 0] >> 32, raw[:, 2:14]
        order = np.argsort(t[:, 0], kind="stable")
        return kid[order], t[order]


def launches(kid, t):
    """Consecutive records of one kernel id form one launch (a PDL successor's
    CTAs start only after every CTA of its predecessor passed its wait)."""
    cut = [0] + [i for i in range(1, len(kid)) if kid[i] != kid[i - 1]] + [len(kid)]
    return [(int(kid[a]), t[a:b]) for a, b in zip(cut[:-1], cut[1:])]


def decode(args):
    """Configuration 1: prompt 16, 24 greedy ids; one replayed step after warm-up.
    Per kernel role, each stamp's min / median / max over CTAs relative to the
    end of the previous launch's last CTA, medians over the step's launches."""
    import torch

    from . import OlmoeModel, synth
    from ._lib import lib

    torch.cuda.set_device(0)
    ring = Ring()
    L = lib()
    m = OlmoeModel.Load(str(synth.cached(synth.OLMOE_1B7B)))
    prompt = np.ascontiguousarray(np.random.default_rng(1).integers(0, m.config().n_vocab, 16).astype(np.int32))
    assert L.nh_decode_prepare(m._h, prompt.ctypes.data_as(C.POINTER(C.c_int32)), 16, 24) == 0
    for _ in range(4):
        assert L.nh_decode_run(m._h, 24) == 0
    ring.reset()
    stream = torch.cuda.ExternalStream(L.nh_model_stream(m._h))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    assert L.nh_decode_run(m._h, 24) == 0
    e1.record(stream)
    kid, t = ring.records()
    roles, prev_end, pos = {}, None, 0
    for k, tt in launches(kid, t):
        if k == 4:
            role, pos = "embed", 0
        elif k == 5:
            role = "lm_head"
        else:
            role = ["qkv", "attention", "out_proj", "moe_fused"][pos % 4]
            pos += 1
        if prev_end is not None:
            r = roles.setdefault(role, {"n": 0, "ctas": [], "ph": {}})
            r["n"] += 1
            r["ctas"].append(len(tt))
            for ph in range(12):
                col = tt[:, ph]
                col = col[col > 0]
                if col.size:
                    r["ph"].setdefault(ph, []).append(((col.min() - prev_end) / 1e3, (np.median(col) - prev_end) / 1e3,
                                                       (col.max() - prev_end) / 1e3))
        prev_end = int(tt[:, 9].max())
    print(json.dumps({"workload": "olmoe-1b7b bs1 decode, 24 positions", "step_ms": e0.elapsed_time(e1),
                      "us_per_token": e0.elapsed_time(e1) * 1e3 / 24}))
    print("stamp: min/median/max over CTAs, us after the previous launch's last CTA ended")
    for role in ("embed", "qkv", "attention", "out_proj", "moe_fused", "lm_head"):
        r = roles.get(role)
        if not r:
            continue
        cells = []
        for ph, v in sorted(r["ph"].items()):
            a = np.array(v)
            cells.append(f"{ph}:{np.median(a[:, 0]):.2f}/{np.median(a[:, 1]):.2f}/{np.median(a[:, 2]):.2f}")
        print(f"{role:10s} launches={r['n']:4d} ctas={int(np.median(r['ctas'])):4d}  " + "  ".join(cells))


def prefill(args):
    """One 1024-token prompt through the batched decode's chunked prefill: per
    tcgen05 launch form, the mean time per (tile, super-block) iteration in its
    four loop phases (thread 0 of every CTA)."""
    import torch

    from . import OlmoeModel, generate_batch_ex, synth

    torch.cuda.set_device(0)
    ring = Ring()
    m = OlmoeModel.Load(str(synth.cached(synth.OLMOE_1B7B)))
    prompt = np.random.default_rng(4).integers(0, m.config().n_vocab, 1024).tolist()
    generate_batch_ex(m, [prompt[:600]], 2, False)
    ring.reset()
    r = generate_batch_ex(m, [prompt], 2, False)
    kid, t = ring.records()
    s = kid == 6
    t = t[s]
    life = t[:, 9] - t[:, 0]
    print(json.dumps({"workload": "olmoe-1b7b prefill, 1 x 1024 tokens", "prefill_ms": r["prefill_ms"],
                      "grouped_tc_ctas": int(s.sum())}))
    for nmat in (1, 2):
        sel = t[:, 7] == nmat
        if not sel.any():
            continue
        it = t[sel, 6].sum()
        ph = [t[sel, 2 + k].sum() / it for k in range(4)]
        print(f"grouped_tc_kernel<{nmat}>: CTAs {int(sel.sum())}, iterations {int(it)}, "
              f"CTA time {life[sel].sum() / 1e6:.1f} ms; per iteration (ns): stage wait {ph[0]:.0f}, "
              f"widen + copies issued {ph[1]:.0f}, MMA {ph[2]:.0f}, epilogue {ph[3]:.0f}")


def streaming(args):
    """Two-phase streaming decode of the skewed OLMoE GGUF, slot budget 32 of
    64, LRU, prompt 64, 16 ids: per kernel its median duration and the median
    gap after the previous launch (the gap before gate/up is the host's slot
    decision round trip)."""
    import torch

    from . import StreamingModel, streaming_generate_ex, synth

    torch.cuda.set_device(0)
    ring = Ring()
    sm = StreamingModel.Load(str(synth.cached(synth.OLMOE_1B7B_SKEW)))
    prompt = np.random.default_rng(2).integers(0, sm.config().n_vocab, 64).tolist()
    streaming_generate_ex(sm, prompt, 8, False, 32)
    ring.reset()
    t0 = time.perf_counter()
    r = streaming_generate_ex(sm, prompt, 16, False, 32)
    wall = time.perf_counter() - t0
    kid, t = ring.records()
    stats, prev_end = {}, None
    lv = launches(kid, t)
    for i, (k, tt) in enumerate(lv):
        name = KERNELS.get(k, str(k))
        if name == "gemv3":
            name = "qkv" if i + 1 < len(lv) and lv[i + 1][0] == 2 else "out_proj"
        first, end = int(tt[:, 0].min()), int(tt[:, 9].max())
        d = stats.setdefault(name, {"dur": [], "gap": []})
        d["dur"].append((end - first) / 1e3)
        if prev_end is not None:
            d["gap"].append((first - prev_end) / 1e3)
        prev_end = end
    print(json.dumps({"workload": "olmoe-1b7b-skew streaming bs1, budget 32 LRU, prompt 64 + 16 ids",
                      "wall_ms": wall * 1e3, "hits": int(r["hits"].sum()), "misses": int(r["misses"].sum())}))
    for name in ("embed", "qkv", "attention", "out_proj", "router", "gate_up", "down", "lm_head"):
        d = stats.get(name)
        if d:
            print(f"{name:10s} launches={len(d['dur']):5d} duration median {np.median(d['dur']):6.2f} us, "
                  f"gap after previous launch median {np.median(d['gap']) if d['gap'] else 0:6.2f} us "
                  f"(mean {np.mean(d['gap']) if d['gap'] else 0:6.2f})")


def batched(args):
    """64 sequences, context 64, 4 decode steps after warm-up: per product of
    the mma.sync grouped kernel (by weight shape), the median launch span,
    the CTA lifetimes (median / max), warp 0's first token tile, and how the
    lifetimes follow the number of token tiles a CTA walks."""
    import torch

    from . import OlmoeModel, generate_batch_ex, synth

    torch.cuda.set_device(0)
    ring = Ring()
    m = OlmoeModel.Load(str(synth.cached(synth.OLMOE_1B7B)))
    prompts = np.random.default_rng(3).integers(0, m.config().n_vocab, (64, 64)).tolist()
    generate_batch_ex(m, prompts, 4, False)
    ring.reset()
    r = generate_batch_ex(m, prompts, 4, False)
    kid, t = ring.records()
    names = {(1024, 2048): "gate/up (grouped, SwiGLU)", (2048, 1024): "down (grouped)",
             (2048, 2048): "q / out_proj", (50304, 2048): "lm_head"}
    per = {}
    staged = bool((kid == 11).any())
    s = kid == (11 if staged else 10)
    t = t[s]
    # One launch = consecutive records with the same weight pointer (stamp 10);
    # the decode steps' launches come last: 16 layers x 6 products + lm_head per step.
    cut = [0] + [i for i in range(1, len(t)) if t[i, 10] != t[i - 1, 10]] + [len(t)]
    mma = [t[a:b] for a, b in zip(cut[:-1], cut[1:])]
    for tt in mma[-4 * 97:]:
        rows, K = int(tt[0, 8]) >> 32, int(tt[0, 8]) & 0xFFFFFFFF
        per.setdefault(names.get((rows, K), f"rows {rows} K {K}"), []).append(tt)
    print(json.dumps({"workload": "olmoe-1b7b bs64, context 64, 4 decode steps (+ chunked prefill)",
                      "decode_ms": r["decode_ms"], "prefill_ms": r["prefill_ms"],
                      "kernel": "batch_mma_staged_kernel" if staged else "batch_mma_kernel"}))
    for name, ls in per.items():
        span = [(x[:, 9].max() - x[:, 0].min()) / 1e3 for x in ls]
        life = np.concatenate([(x[:, 9] - x[:, 1]) / 1e3 for x in ls])
        first = np.concatenate([(x[:, 2] - x[:, 1]) / 1e3 for x in ls if (x[:, 2] > 0).all()] or [np.zeros(1)])
        ntt = np.concatenate([x[:, 6] for x in ls])
        line = (f"{name:26s} launches {len(ls):4d}  span median {np.median(span):7.1f} us  CTA life median "
                f"{np.median(life):6.1f} max {life.max():6.1f} us")
        if staged:
            cat = np.concatenate(ls)
            tot = cat[:, 2:5].sum(axis=0) / max(1, len(cat)) / 1e3
            line += f"  per CTA: rows wait {tot[0]:.1f} us, stage waits {tot[1]:.1f} us, multiply {tot[2]:.1f} us"
        else:
            line += f"  first tile {np.median(first):5.1f} us"
        for n in sorted(set(ntt.tolist()))[:4]:
            line += f"  [{int(n)} tiles: {np.median(life[ntt == n]):.1f} us x{int((ntt == n).sum())}]"
        print(line)


def battention(args):
    """4 sequences with 2048-token contexts, 2 decode steps: per launch of the
    batched attention kernel (one (head, 64-position split, sequence) per CTA)
    the span, and per CTA the time from its wait to the staged K/V rows, the
    scores and softmax, the V sums and partials, the ticket, and (for the last
    CTA of a (head, sequence)) the split combination."""
    import torch

    from . import OlmoeModel, generate_batch_ex, synth

    torch.cuda.set_device(0)
    ring = Ring(units=("batch",))  # the batched kernels only
    m = OlmoeModel.Load(str(synth.cached(synth.OLMOE_1B7B)))
    prompts = np.random.default_rng(3).integers(0, m.config().n_vocab, (4, 2048)).tolist()
    generate_batch_ex(m, [p[:64] for p in prompts], 2, False)
    ring.reset()
    r = generate_batch_ex(m, prompts, 2, False)
    kid, t = ring.records()
    s = kid == 12
    t = t[s]
    # Decode steps only: the last two steps x 16 layers of launches.
    gaps = np.where(np.diff(t[:, 0]) > 20_000)[0]
    starts = [0] + (gaps + 1).tolist()
    ls = [t[a:b] for a, b in zip(starts, starts[1:] + [len(t)])][-32:]
    span = [(x[:, 9].max() - x[:, 0].min()) / 1e3 for x in ls]
    cat = np.concatenate(ls)
    ph = lambda a, b: np.median((cat[:, b] - cat[:, a])[(cat[:, a] > 0) & (cat[:, b] > 0)]) / 1e3
    last = cat[cat[:, 7] == 1]
    print(json.dumps({"workload": "olmoe-1b7b batched decode, 4 x 2048 contexts, 2 steps",
                      "decode_ms": r["decode_ms"], "launches": len(ls), "ctas_per_launch": int(np.median([len(x) for x in ls]))}))
    print(f"launch span median {np.median(span):.1f} us; per CTA (median): entry->wait {ph(0, 1):.2f}, "
          f"wait->K/V staged {ph(1, 2):.2f}, scores+softmax {ph(2, 3):.2f}, V sums+partials {ph(3, 4):.2f}, "
          f"ticket {ph(4, 5):.2f}, non-last end {ph(5, 9):.2f} us; combine (last CTAs) "
          f"{np.median((last[:, 9] - last[:, 5]) / 1e3) if len(last) else 0:.2f} us; CTA life {ph(0, 9):.2f} us")


def main() -> None:
    modes = {"decode": decode, "prefill": prefill, "streaming": streaming, "batched": batched,
             "battention": battention}
    mode = sys.argv[1] if len(sys.argv) > 1 else "decode"
    if mode not in modes:
        raise SystemExit(f"usage: python -m nuthatch_b200.phase_trace [{'|'.join(modes)}]")
    os.environ["NH_PHASE_TRACE_LIB"] = "1"
    from ._lib import PHASE_TRACE_LIB_PATH

    if not PHASE_TRACE_LIB_PATH.exists():
        raise SystemExit(f"{PHASE_TRACE_LIB_PATH} is missing: python -m nuthatch_b200.build --phase-trace")
    modes[mode](sys.argv[2:])


if __name__ == "__main__":
    main()
