#!/usr/bin/env python3
"""Benchmark: OLMoE-1B-7B-shaped Q4_K_M resident greedy decode, batch 1.

Workload (the headline configuration): a seeded random-init GGUF of the
OLMoE-1B-7B shape (16 layers, n_embd 2048, 16x128 MHA heads, 64 experts
top-8, expert FFN 1024, vocab 50304; Q4_K with attn_v/ffn_down on odd layers
and output in Q6_K), a 16-token seeded prompt, 24 greedy ids.

One timed step = the 24 decode positions of that request (the last prompt
position first, as its logits choose the first id), replayed from the saved
KV-cache cursor with every input already in HBM.  value = decode tokens/s
over all ranks (replicas: each GPU decodes its own sequence).  e2e = the
same metric through the public API call GreedyGenerateCached (host prompt in,
host ids out, prompt prefill included as in the reference's own timing).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_PROMPT = 16
N_PREDICT = 24
METRIC = "OLMoE Q4_K_M decode tok/s (bs1, bs64) at 1/2/4/8 B200; % HBM roofline"
WORKLOAD = "olmoe-1b7b-q4km-resident-decode-bs1 (prompt 16, 24 greedy tokens)"

# Algorithmic bytes (weights read once per token; KV averaged over positions
# 16..39; norms; embedding row).  Per layer: attention 9,437,184 B (10,518,528
# on Q6_K attn_v layers), router 524,288 B, 8 experts x 3,538,944 B (4,079,616
# on Q6_K ffn_down layers); lm_head 84,510,720 B.
GATE_UP_BYTES = 8 * 2 * 1024 * 1152  # one nh_moe_gate_up launch: 8 experts x (gate + up) rows of 1152 B
# One nh_moe_layer launch (router + gate/up + down), averaged over the 16
# layers: router 524,288 B + gate/up 18,874,368 B + down 8 x 2048 rows of 576 B
# (Q4_K layers) or 840 B (Q6_K layers), 8 of each.
MOE_LAYER_BYTES = 524288 + GATE_UP_BYTES + (8 * 2048 * 576 + 8 * 2048 * 840) // 2


def step_bytes_per_token(cfg_layers=16) -> float:
    attn = 8 * 9437184 + 8 * 10518528
    experts = 8 * (8 * 3538944) + 8 * (8 * 4079616)
    router = 16 * 524288
    norms = 16 * 4 * 2048 * 4 + 2048 * 4
    lm_head = 84510720
    emb = 1152
    kv = 262144 * np.mean(np.arange(16, 40) + 1)
    return float(attn + experts + router + norms + lm_head + emb + kv)


def prompt_ids(n_vocab: int) -> list[int]:
    return np.random.default_rng(1).integers(0, n_vocab, N_PROMPT).tolist()


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def traffic_summary(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[f"{kernel}_dram_bytes_per_launch"])
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except Exception:
                continue
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_oracle_run(path: str, n_predict: int, threads: int) -> tuple[float, list[int]]:
    """One GreedyGenerateCached-equivalent oracle call (one-shot prompt prefill + decode); seconds."""
    import oracle

    oracle.set_threads(threads)
    om = oracle.OracleModel(path)
    p = prompt_ids(om.cfg["n_vocab"])
    t0 = time.perf_counter()
    out = om.generate(p, n_predict, mode=0)
    dt = time.perf_counter() - t0
    om.close()
    return dt, out["tokens"]


def max_over_ranks(value: float, dist, device: str = "cuda") -> float:
    """The largest of every rank's value (timings: the job is as slow as its
    slowest rank); the value itself without a process group."""
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from nuthatch_b200 import synth

    path = str(synth.cached(synth.OLMOE_1B7B))
    threads = os.cpu_count() or 1
    # Size the per-step sample so that the whole run stays within a few minutes.
    dt, _ = cpu_oracle_run(path, 4, threads)
    per_token = dt / (N_PROMPT + 3)
    budget_s = 150.0
    n_pred = N_PREDICT
    while n_pred > 4 and (args.steps + args.warmup) * per_token * (N_PROMPT + n_pred - 1) > budget_s:
        n_pred //= 2
    for _ in range(args.warmup):
        cpu_oracle_run(path, n_pred, threads)
    times = [cpu_oracle_run(path, n_pred, threads)[0] for _ in range(args.steps)]
    value = n_pred * len(times) / sum(times)
    sample = f"GreedyGenerateCached restatement: prompt {N_PROMPT} + {n_pred} greedy ids per step, one-shot prefill"
    # The reference runs its graphs on 4 threads (generate.cc:38,90): the same
    # sample at that count, when it fits in about a minute.
    ref_threads = min(4, threads)
    est = dt * threads / ref_threads * (N_PROMPT + n_pred - 1) / (N_PROMPT + 3)
    at_ref = {"threads": ref_threads, "value": None, "unit": "tok/s"}
    if est <= 60.0:
        t4 = cpu_oracle_run(path, n_pred, ref_threads)[0]
        at_ref["value"] = n_pred / t4
    else:
        at_ref["skipped"] = f"estimated {est:.0f} s"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4k/q6k x q8k int dot, f32",
            "data": "synthetic (seeded random-init GGUF)",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": N_PROMPT + N_PREDICT,
                       "parallelism": "host CPU", "l2": "n/a"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                             "host_nproc": os.cpu_count(), "at_reference_threads": at_ref},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's own ggml build is unavailable here (ggml absent); timed: the C++ restatement "
                    "of its CPU path (oracle/) on all host threads"}
    print(json.dumps(line), flush=True)


def run_streaming(args) -> None:
    """Streaming decode (two-phase, HBM expert slot pool) on the skewed
    OLMoE-1B-7B-shaped GGUF: prompt 64, 256 greedy ids, budget B experts per
    layer, learned-pin (pin = ceil(0.75 B)) calibrated on a resident routing
    trace of a different seeded prompt, and LRU at the same budget.  Timed end
    to end through StreamingGenerate (host ids in and out, token-by-token
    prefill included); one JSON line per (policy, budget)."""
    import math

    import torch

    import nuthatch_b200 as nh
    from nuthatch_b200 import build, synth

    build.build_product()
    torch.cuda.set_device(0)
    path = str(synth.cached(synth.OLMOE_1B7B_SKEW))
    n_prompt, n_pred = 64, args.stream_tokens
    rng = np.random.default_rng(7)
    resident = nh.OlmoeModel.Load(path)
    cfg = resident.config()
    calib_prompt = rng.integers(0, cfg.n_vocab, n_prompt).tolist()
    prompt = np.random.default_rng(8).integers(0, cfg.n_vocab, n_prompt).tolist()
    trace = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(resident, calib_prompt, n_pred, False, trace)
    usage = nh.BuildUsage(trace, cfg.n_expert).counts
    ref = nh.GreedyGenerateCached(resident, prompt, n_pred, False)
    # Realised expert-frequency skew of the calibration trace (share of the top quarter of experts).
    per = np.sort(usage.astype(np.float64), axis=1)[:, ::-1]
    skew = float(np.mean(per[:, : cfg.n_expert // 4].sum(1) / per.sum(1)))
    del resident
    torch.cuda.empty_cache()
    sm = nh.StreamingModel.Load(path)
    for budget in args.budgets:
        for policy in ("learned_pin", "lru"):
            pin = int(math.ceil(0.75 * budget)) if policy == "learned_pin" else 0
            kw = dict(policy=policy, pin_slots=pin, usage=usage if policy == "learned_pin" else None)
            for _ in range(args.warmup):
                nh.streaming_generate_ex(sm, prompt, 8, False, budget, **kw)
            times, out = [], None
            for _ in range(args.steps):
                t0 = time.perf_counter()
                out = nh.streaming_generate_ex(sm, prompt, n_pred, False, budget, **kw)
                times.append(time.perf_counter() - t0)
            hits, misses = int(out["hits"].sum()), int(out["misses"].sum())
            dt = float(np.median(times))
            line = {"metric": f"OLMoE streaming decode tok/s (bs1, budget {budget}, {policy})",
                    "value": n_pred / dt, "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": 1000 * dt, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "q4k/q6k x q8k int dot, f32 accumulate",
                    "data": "synthetic (seeded random-init GGUF of the OLMoE-1B-7B shape, log-Zipf router skew)",
                    "config": {"workload": f"olmoe-1b7b-q4km-skew-streaming-bs1 (prompt {n_prompt}, {n_pred} greedy "
                                           f"tokens, budget {budget} of {cfg.n_expert} per layer)",
                               "policy": policy, "pin_slots": pin, "calibration": "resident trace, different prompt",
                               "top_quarter_expert_share": skew},
                    "hits": hits, "misses": misses, "hit_rate": hits / max(1, hits + misses),
                    "h2d_bytes_per_token": out["h2d_bytes"] / (n_prompt + n_pred - 1),
                    "tokens_match_resident": out["tokens"] == ref,
                    "step": "one StreamingGenerate call (prefill token by token + decode), host ids in/out"}
            print(json.dumps(line), flush=True)
    sm.close()


def run_batched(args) -> None:
    """Batched resident decode: n_seq independent sequences, each with a
    seeded random-id context of `context` tokens processed into its KV cache
    (one position per step, as the decode steps do), then `steps` greedy
    decode steps.  Timed on the device from the last context position to the
    end (decode_ms); value = sequences x decoded ids / time."""
    import torch

    import nuthatch_b200 as nh
    from nuthatch_b200 import build, synth

    build.build_product()
    torch.cuda.set_device(0)
    path = str(synth.cached(synth.OLMOE_1B7B))
    m = nh.OlmoeModel.Load(path)
    cfg = m.config()
    B, ctx, n_pred = args.batch_seqs, args.batch_context, args.batch_steps
    prompts = np.random.default_rng(3).integers(0, cfg.n_vocab, (B, ctx)).tolist()
    nh.generate_batch_ex(m, [p[:8] for p in prompts[:2]], 2, False)  # loads and configures the kernels
    clocks = ClockSampler(0)
    r = nh.generate_batch_ex(m, prompts, n_pred, False)
    clk = clocks.stop()
    ms = r["decode_ms"]
    value = B * n_pred / (ms / 1000.0)
    # Parity on a seeded subset: two sequences decoded alone give the same ids.
    subset_ok = all(r["tokens"][b] == nh.GreedyGenerateCached(m, prompts[b], n_pred, False) for b in (0, B - 1))
    # Algorithmic bytes per decode step at the mean decode position: weights
    # (attention, router, every expert a step touches, lm_head) and the KV rows read.
    pos_mean = ctx - 1 + (n_pred - 1) / 2.0
    kv = B * cfg.n_layers * (pos_mean + 1) * 2 * cfg.n_head_kv * (cfg.n_embd // cfg.n_head) * 4
    weights = 8 * 9437184 + 8 * 10518528 + 16 * 524288 + 8 * 64 * 3538944 + 8 * 64 * 4079616 + 84510720
    step_bytes = kv + weights
    peaks = measured_peaks()
    achieved = step_bytes / (ms / 1000.0 / n_pred) / 1e9
    line = {"metric": f"OLMoE Q4_K_M batched decode tok/s (bs{B}, {ctx}-token contexts)", "value": value,
            "unit": "tok/s", "n_gpus": 1, "steps": n_pred, "warmup": 1, "ms_per_step": ms / n_pred,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4k/q6k x q8k int dot, f32 accumulate, f32 KV",
            "data": "synthetic (seeded random-init GGUF of the OLMoE-1B-7B shape, seeded random-id contexts)",
            "config": {"workload": f"olmoe-1b7b-q4km-batched-decode (bs{B}, context {ctx}, {n_pred} greedy steps)",
                       "global_batch": B, "seq_len": ctx + n_pred, "parallelism": "single GPU",
                       "step": "one decode position of every sequence (CUDA graph replay)",
                       "l2": "inputs larger than L2 (KV cache and weights)"},
            "clocks": clk,
            "step_roofline": {"bytes_per_step": step_bytes, "kv_bytes_per_step": kv, "achieved": achieved,
                              "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"]},
            "subset_matches_single_sequence": subset_ok}
    print(json.dumps(line), flush=True)


def run_prefill(args) -> None:
    """Configuration 4: 8 sequences of 4096 seeded random ids, prompt prefill
    then 64 greedy ids each, through GreedyGenerateCachedBatch: the prompt
    positions of all sequences run as 512-row chunks of the batched kernels
    (tcgen05 grouped expert products, causal prefill attention), then the
    batched decode steps.  Under torchrun (N ranks, one GPU each) the
    sequences are split over the ranks (attention data-parallel) and the
    experts sharded E/N per GPU with NCCL all-gather / all-to-all per MoE
    layer: the total work is fixed, so scaling is strong.  Device-timed
    parts (CUDA events on the decode stream), max over ranks; value = prefill
    tokens of all sequences / prefill time.  At N=1 the same prompts are
    also run one sequence at a time (GreedyGenerateCached), for comparison."""
    import datetime

    import torch

    import nuthatch_b200 as nh
    from nuthatch_b200 import build, synth
    from nuthatch_b200._lib import lib

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    build.build_product()
    L = lib()
    assert L.nh_set_device(local_rank) == 0
    if rank == 0:
        synth.cached(synth.OLMOE_1B7B)
    if dist is not None:
        dist.barrier()
    path = str(synth.cached(synth.OLMOE_1B7B))
    cfg_model = nh.OlmoeModel.Load(path) if world == 1 else None
    n_seq, n_prompt, n_pred = args.prefill_seqs, args.prefill_tokens, args.prefill_decode
    from nuthatch_b200._lib import NhConfig

    cfg = NhConfig()
    assert L.nh_gguf_probe(path.encode(), C.byref(cfg)) > 0
    if n_seq % world != 0 or cfg.n_expert % world != 0:
        if rank == 0:
            print(json.dumps({"workload": "prefill", "unavailable": f"{n_seq} sequences / {cfg.n_expert} experts "
                                                                    f"do not split over {world} GPUs"}))
        return
    prompts = np.random.default_rng(4).integers(0, cfg.n_vocab, (n_seq, n_prompt), dtype=np.int32)
    per = n_seq // world
    mine = prompts[rank * per:(rank + 1) * per].tolist()
    ep = None
    if world > 1:
        box = [nh.ExpertGroup.new_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ep = nh.ExpertGroup(box[0], world, rank)
        first, count = nh.ExpertGroup.shard(cfg.n_expert, world, rank)
        model = nh.OlmoeModel.LoadExpertShard(path, first, count)
    else:
        model = cfg_model
    if model is None:
        raise SystemExit("model load failed")
    # Warm-up: buffers, kernel attributes, NCCL connections, graphs.
    nh.generate_batch_ex(model, [p[:600] for p in mine], 2, False, ep=ep)
    clocks = ClockSampler(local_rank)
    r = nh.generate_batch_ex(model, mine, n_pred, False, ep=ep)
    clk = clocks.stop()
    pre_ms = max_over_ranks(r["prefill_ms"], dist)
    dec_ms = max_over_ranks(r["decode_ms"], dist)
    single = None
    if world == 1:
        out = np.zeros(n_pred, dtype=np.int32)
        pf, dc = C.c_double(0), C.c_double(0)
        s_pre = s_dec = 0.0
        same = True
        for b in range(n_seq):
            pc = np.ascontiguousarray(prompts[b])
            assert L.nh_generate_timed(model._h, pc.ctypes.data_as(C.POINTER(C.c_int32)), pc.size, n_pred, 0,
                                       out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(pf), C.byref(dc)) == 0
            s_pre += pf.value
            s_dec += dc.value
            same = same and out.tolist() == r["tokens"][b]
        single = {"api": "GreedyGenerateCached per sequence (nh_generate_timed)",
                  "prefill_tok_s": n_seq * (n_prompt - 1) / (s_pre / 1000.0),
                  "decode_tok_s": n_seq * n_pred / (s_dec / 1000.0), "ids_equal_batched": same}
    if ep is not None:
        model.close()
        ep.close()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    n_pre = n_seq * (n_prompt - 1)
    # Per prefill token: 2 x active parameters (attention 4 d^2, router d E,
    # 8 experts x 3 d F, per layer) + causal attention 4 x (p+1) x d per layer.
    active = cfg.n_layers * (4 * cfg.n_embd ** 2 + cfg.n_embd * cfg.n_expert +
                             cfg.n_expert_used * 3 * cfg.n_embd * cfg.n_ff)
    attn = cfg.n_layers * 4 * cfg.n_embd * (n_prompt / 2.0)
    flops = n_pre * (2 * active + attn)
    peaks = measured_peaks()
    tflops = flops / (pre_ms / 1000.0) / 1e12
    line = {"metric": f"OLMoE Q4_K_M prompt prefill tok/s ({n_seq} x {n_prompt} tokens) + decode",
            "value": n_pre / (pre_ms / 1000.0), "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": pre_ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4k/q6k x q8k int dot, f32 accumulate, f32 KV",
            "data": "synthetic (seeded random-init GGUF of the OLMoE-1B-7B shape, seeded random-id prompts)",
            "config": {"workload": f"olmoe-1b7b-q4km-prefill ({n_seq} x {n_prompt} prompt, {n_pred} greedy ids)",
                       "parallelism": f"ep{world} (experts {cfg.n_expert // world} per GPU, "
                                      f"{per} sequences per GPU)" if world > 1 else "single GPU",
                       "step": "the prompt prefill of all sequences (512-row chunks)"},
            "clocks": clk, "decode_tok_s": n_seq * n_pred / (dec_ms / 1000.0), "decode_ms": dec_ms,
            "prefill_roofline": {"bound": "tensor", "flops": flops, "achieved": tflops,
                                 "peak": peaks.get("bf16_tflops"), "unit": "TFLOP/s",
                                 "note": "int8 tensor-core products against the measured bf16 dense peak"},
            "one_sequence_at_a_time": single}
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_granite(args) -> None:
    """Configuration 5: a Granite-3-MoE-shaped seeded GGUF (24 layers, n_embd
    1024, GQA 16/8 x 64, 32 experts top-8, FFN 512), batched streaming decode
    of 32 sequences with 1024-token seeded contexts and 256 greedy steps,
    every layer's experts streamed through a slot budget of 8 per layer for
    the whole job (LRU, and learned pin calibrated on a resident trace of
    another prompt).  A step's batch selects more distinct experts than the
    pool holds, so each layer runs in waves.  Under torchrun (N ranks, one GPU
    each) the budget is split 8/N slots per GPU, each GPU streaming only its
    32/N experts (expert parallelism: NCCL all-gather of the tokens' rows and
    selections, all-to-all of the pick rows) and decoding 32/N sequences: the
    total work and budget are fixed, so scaling is strong.  Device-timed
    decode part, max over ranks; value = sequences x ids / time.  Parity:
    each rank's first two sequences against the resident batched decode of a
    shorter run of the same prompts (through the same expert group)."""
    import datetime

    import torch

    import nuthatch_b200 as nh
    from nuthatch_b200 import build, synth
    from nuthatch_b200._lib import lib

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    build.build_product()
    assert lib().nh_set_device(local_rank) == 0
    if rank == 0:
        synth.cached(synth.GRANITE_MOE)
    if dist is not None:
        dist.barrier()
    path = str(synth.cached(synth.GRANITE_MOE))
    B, ctx, n_pred, budget = args.granite_seqs, args.granite_context, args.granite_steps, args.granite_budget
    m = nh.OlmoeModel.Load(path)
    cfg = m.config()
    if B % world != 0 or cfg.n_expert % world != 0 or budget % world != 0:
        if rank == 0:
            print(json.dumps({"workload": "granite", "unavailable": f"{B} sequences / {cfg.n_expert} experts / "
                                                                    f"budget {budget} do not split over {world} GPUs"}))
        if dist is not None:
            dist.destroy_process_group()
        return
    cap = budget // world
    per = B // world
    prompts = np.random.default_rng(5).integers(0, cfg.n_vocab, (B, ctx)).tolist()
    mine = prompts[rank * per:(rank + 1) * per]
    cal = nh.RoutingTrace()
    nh.GreedyGenerateCachedTrace(m, np.random.default_rng(6).integers(0, cfg.n_vocab, 64).tolist(), 64, False, cal)
    usage = nh.BuildUsage(cal, cfg.n_expert).counts
    check = nh.generate_batch_ex(m, mine[:2], 8, False)["tokens"]
    m.close()
    ep = None
    if world > 1:
        box = [nh.ExpertGroup.new_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ep = nh.ExpertGroup(box[0], world, rank)

    def job_sum(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        return float(t.item())

    sm = nh.StreamingModel.Load(path)
    rows = {}
    for policy in ("lru", "learned_pin"):
        # Learned pin keeps at least one LRU slot per GPU for the waves.
        pin = min((cap * 3 + 3) // 4, cap - 1)
        if policy == "learned_pin" and pin < 1:
            rows[policy] = {"unavailable": f"{cap} slot per GPU leaves no LRU slot beside a pinned one"}
            continue
        kw = dict(policy="learned_pin", pin_slots=pin, usage=usage) if policy == "learned_pin" else {}
        ok = nh.streaming_generate_batch_ex(sm, mine[:2], 8, False, cap, ep=ep, **kw)["tokens"] == check
        clocks = ClockSampler(local_rank)
        r = nh.streaming_generate_batch_ex(sm, mine, n_pred, False, cap, ep=ep, **kw)
        clk = clocks.stop()
        ms = max_over_ranks(r["decode_ms"], dist)
        hits, acc = job_sum(int(r["hits"].sum())), job_sum(int((r["hits"] + r["misses"]).sum()))
        rows[policy] = {"tok_s": B * n_pred / (ms / 1000.0), "decode_ms": ms, "hit_rate": hits / max(acc, 1),
                        "waves_per_gpu": job_sum(r["waves"]) / world, "h2d_gb": job_sum(r["h2d_bytes"]) / 1e9,
                        "slots_per_gpu": cap, "pinned_per_gpu": pin if policy == "learned_pin" else 0,
                        "subset_matches_resident": job_sum(0.0 if ok else 1.0) == 0.0, "clocks": clk}
    sm.close()
    if ep is not None:
        ep.close()
    if rank == 0:
        line = {"metric": f"Granite-shaped Q4_K_M batched streaming decode tok/s (bs{B}, {ctx}-token contexts, "
                          f"budget {budget} of {cfg.n_expert})",
                "value": rows["lru"]["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": n_pred, "warmup": 1,
                "ms_per_step": rows["lru"]["decode_ms"] / n_pred, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "q4k/q6k x q8k int dot, f32 accumulate, f32 KV",
                "data": "synthetic (seeded random-init Granite-3-MoE-shaped GGUF, seeded random-id contexts)",
                "config": {"workload": f"granite-shape-batched-streaming (bs{B}, context {ctx}, {n_pred} greedy "
                                       f"steps, slot budget {budget} per layer for the job)",
                           "parallelism": f"ep{world} ({cfg.n_expert // world} experts and {cap} slots per layer "
                                          f"per GPU, {per} sequences per GPU)" if world > 1 else "single GPU",
                           "experts": "pinned host store -> HBM slot pool per layer, waves when the batch's "
                                      "distinct experts exceed the pool"},
                "policies": rows}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_tokenizer(args) -> None:
    """The tokenizer (host only, no GPU): Encode throughput over seeded
    multi-script text of about 8 MB (words of Latin, Cyrillic, Greek, Arabic,
    Devanagari and CJK scripts, digits, punctuation, emoji, mixed whitespace)
    with a 16,000-entry byte-level BPE vocabulary trained on the same kind of
    text by the HF `tokenizers` trainer (the real OLMoE vocabulary is not
    available offline).  value = input MB/s on one host thread; the oracle's
    restatement (Python, rescanning merges) is timed on a 200 KB sample."""
    import json as _json

    from tokenizers import Tokenizer as HfTokenizer, models, pre_tokenizers, trainers

    import nuthatch_b200 as nh
    from nuthatch_b200 import build
    from oracle.tokenizer import OracleTokenizer

    build.build_product()
    words = ["the", "quick", "brown", "fox", "jumps", "over", "lazy", "dog", "Paris", "naïve", "café", "Straße",
             "東京", "数据", "Москва", "λόγος", "مرحبا", "हिन्दी", "2024", "3.14", "don't", "it's", "we're", "!!", "?",
             "...", "(x)", "#1", "😀", "€5"]
    spaces = [" "] * 12 + ["\n", "\n\n", "  ", "\t"]
    rng = np.random.default_rng(7)

    def text(n_words: int) -> str:
        w = rng.integers(len(words), size=n_words)
        sp = rng.integers(len(spaces), size=n_words)
        return "".join(words[a] + spaces[b] for a, b in zip(w, sp))

    hf = HfTokenizer(models.BPE())
    hf.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    hf.train_from_iterator([text(200) for _ in range(2000)],
                           trainers.BpeTrainer(vocab_size=16000, show_progress=False,
                                               initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    model = _json.loads(hf.to_str())["model"]
    vocab = [t for t, _ in sorted(model["vocab"].items(), key=lambda kv: kv[1])]
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    tok = nh.Tokenizer.FromLists(vocab, merges)
    body = text(1_200_000)
    raw = body.encode()
    tok.Encode(body[:10000])
    times = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        ids = tok.Encode(raw)
        times.append(time.perf_counter() - t0)
    best = min(times)
    t0 = time.perf_counter()
    hf.encode(body)
    hf_s = time.perf_counter() - t0
    sample = body[:200_000]
    ora = OracleTokenizer(vocab, merges)
    t0 = time.perf_counter()
    ora_ids = ora.encode(sample)
    ora_s = time.perf_counter() - t0
    same = tok.Encode(sample) == ora_ids
    line = {"metric": "tokenizer Encode MB/s (GPT-2 byte-level BPE, 16k vocabulary)", "value": len(raw) / best / 1e6,
            "unit": "MB/s", "n_gpus": 0, "steps": len(times), "warmup": 1, "ms_per_step": best * 1000.0,
            "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bytes",
            "data": "synthetic (seeded multi-script text; vocabulary trained on the same kind of text)",
            "config": {"workload": f"tokenizer-encode ({len(raw) / 1e6:.1f} MB, {len(ids)} ids)",
                       "parallelism": "one host thread"},
            "tokens_per_s": len(ids) / best,
            "hf_tokenizers_mb_s": {"value": len(raw) / hf_s / 1e6,
                                   "note": "HF tokenizers' encode of the same text (GPT-2 pre-split, one call), "
                                           "for context"},
            "cpu_baseline": {"value": len(sample.encode()) / ora_s / 1e6, "unit": "MB/s", "cores": 1, "kind": "port",
                             "sample": "200 KB of the same text through oracle/tokenizer.py",
                             "ids_equal": same}}
    print(json.dumps(line), flush=True)


def run_ep_batched(args, dist, rank: int, world: int, local_rank: int, path: str, full_model) -> dict | None:
    """Expert-parallel batched decode (the configuration-3 workload: bs64,
    2048-token seeded contexts, 128 greedy steps) over the `world` GPUs of
    this job: experts sharded n_expert/world per GPU (each rank loads only its
    shard), sequences split evenly (data-parallel attention), NCCL all-gather
    of the tokens' Q8_K rows and selections and an all-to-all of the pick rows
    per MoE layer.  Device-timed decode part, max over ranks; value = global
    sequences x decoded ids / time.  Rank 0 checks its first sequence against
    the single-GPU GreedyGenerateCached of it."""
    import torch

    import nuthatch_b200 as nh

    cfg = full_model.config()
    B, ctx, n_pred = args.batch_seqs, args.batch_context, args.batch_steps
    if B % world != 0 or cfg.n_expert % world != 0:
        return None
    box = [nh.ExpertGroup.new_id() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(box, src=0)
    ep = nh.ExpertGroup(box[0], world, rank)
    first, count = nh.ExpertGroup.shard(cfg.n_expert, world, rank)
    shard = nh.OlmoeModel.LoadExpertShard(path, first, count)
    if shard is None:
        raise SystemExit("expert shard load failed")
    prompts = np.random.default_rng(3).integers(0, cfg.n_vocab, (B, ctx)).tolist()
    per = B // world
    mine = prompts[rank * per:(rank + 1) * per]
    # Warm-up call (kernel configuration, NCCL connections), then the run.
    nh.generate_batch_ex(shard, [p[:8] for p in mine], 2, False, ep=ep)
    clocks = ClockSampler(local_rank)
    r = nh.generate_batch_ex(shard, mine, n_pred, False, ep=ep)
    clk = clocks.stop()
    ms = max_over_ranks(r["decode_ms"], dist)
    subset_ok = None
    if rank == 0:
        subset_ok = r["tokens"][0] == nh.GreedyGenerateCached(full_model, mine[0], n_pred, False)
    shard.close()
    ep.close()
    value = B * n_pred / (ms / 1000.0)
    pos_mean = ctx - 1 + (n_pred - 1) / 2.0
    kv = per * cfg.n_layers * (pos_mean + 1) * 2 * cfg.n_head_kv * (cfg.n_embd // cfg.n_head) * 4
    # Per rank and step: replicated attention weights, router and lm_head, its
    # own experts (every expert a step touches, all of them at bs64), its KV.
    weights = (8 * 9437184 + 8 * 10518528 + 16 * 524288 + 84510720 +
               (8 * 64 * 3538944 + 8 * 64 * 4079616) // world)
    peaks = measured_peaks()
    achieved = (kv + weights) / (ms / 1000.0 / n_pred) / 1e9
    coll = ep_collective_times(dist, world, per, cfg) if dist is not None else None
    if coll is not None:
        coll["share_of_step"] = coll["per_step_ms"] / (ms / n_pred)
    return {"metric": f"OLMoE Q4_K_M expert-parallel batched decode tok/s (bs{B}, {ctx}-token contexts)",
            "value": value, "unit": "tok/s", "n_gpus": world, "ms_per_step": ms / n_pred,
            "experts_per_gpu": count, "sequences_per_gpu": per, "steps": n_pred,
            "collectives": "per MoE layer: NCCL all-gather of Q8_K rows + top-k ids, all-to-all of pick rows",
            "timing": "device time of the decode part (CUDA events on the decode stream), max over ranks",
            "clocks": clk,
            "step_roofline_per_gpu": {"bytes_per_step": kv + weights, "achieved": achieved, "peak": peaks["hbm_gbs"],
                                      "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"]},
            "subset_matches_single_gpu": subset_ok, "collective_times": coll}


def ep_collective_times(dist, world: int, per: int, cfg) -> dict:
    """The two exchanges of one expert-parallel MoE layer at the decode's
    sizes, timed alone with torch's NCCL process group (CUDA events, 20
    repetitions after 3, max over ranks): the all-gather of every rank's
    Q8_K rows (2432 bytes per token at n_embd 2048) and the all-to-all of
    pick rows ([per][k][n_embd] f32 per rank pair).  The library issues the
    same two collectives from its own NCCL communicator inside the step."""
    import torch

    q8_row = (cfg.n_embd // 256) * 304
    ag_src = torch.zeros(per * q8_row, dtype=torch.uint8, device="cuda")
    ag_dst = torch.zeros(world * per * q8_row, dtype=torch.uint8, device="cuda")
    blk = per * cfg.n_expert_used * cfg.n_embd
    a2a_src = torch.zeros(world * blk, dtype=torch.float32, device="cuda")
    a2a_dst = torch.zeros(world * blk, dtype=torch.float32, device="cuda")

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(20):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) * 1000.0 / 20, dist)

    ag = timed(lambda: dist.all_gather_into_tensor(ag_dst, ag_src))
    a2a = timed(lambda: dist.all_to_all_single(a2a_dst, a2a_src))
    per_layer = ag + a2a
    return {"all_gather_us": ag, "all_to_all_us": a2a, "per_layer_us": per_layer,
            "per_step_ms": per_layer * cfg.n_layers / 1000.0,
            "limiting": "all_to_all of pick rows" if a2a >= ag else "all_gather of Q8_K rows",
            "bytes": {"all_gather_per_rank": per * q8_row, "all_to_all_per_rank_pair": blk * 4}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="prefill, warm-up, then exactly one timed-step's decode and exit (for ncu launch lists)")
    ap.add_argument("--profile-layers", type=int, default=0,
                    help="with --profile: the same OLMoE-1B-7B width cut to this many layers (small ncu captures)")
    ap.add_argument("--workload", default="resident", choices=["resident", "streaming", "batched", "prefill", "granite",
                                                                     "tokenizer"])
    ap.add_argument("--batch-seqs", type=int, default=64)
    ap.add_argument("--batch-context", type=int, default=2048)
    ap.add_argument("--batch-steps", type=int, default=128)
    ap.add_argument("--budgets", type=int, nargs="*", default=[4, 8, 16, 32])
    ap.add_argument("--stream-tokens", type=int, default=256)
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel batched section")
    ap.add_argument("--granite-seqs", type=int, default=32)
    ap.add_argument("--granite-context", type=int, default=1024)
    ap.add_argument("--granite-steps", type=int, default=256)
    ap.add_argument("--granite-budget", type=int, default=8)
    ap.add_argument("--prefill-seqs", type=int, default=8)
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--prefill-decode", type=int, default=64)
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.workload == "batched":
        run_batched(args)
        return
    if args.workload == "prefill":
        run_prefill(args)
        return
    if args.workload == "granite":
        run_granite(args)
        return
    if args.workload == "tokenizer":
        run_tokenizer(args)
        return
    if args.workload == "streaming":
        args.steps = min(args.steps, 3)
        run_streaming(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    import torch

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))

    def barrier():
        if dist is not None:
            dist.barrier()

    from nuthatch_b200 import build, synth

    build.build_product()
    import nuthatch_b200 as nh
    from nuthatch_b200._lib import lib

    L = lib()
    assert L.nh_set_device(local_rank) == 0
    spec = synth.OLMOE_1B7B
    if args.profile and args.profile_layers > 0:
        spec = synth.replace(spec, n_layers=args.profile_layers)
    if rank == 0:
        path = str(synth.cached(spec))
    barrier()
    path = str(synth.cached(spec))
    m = nh.OlmoeModel.Load(path)
    if m is None:
        raise SystemExit("model load failed")
    cfg = m.config()
    prompt = np.ascontiguousarray(np.asarray(prompt_ids(cfg.n_vocab), dtype=np.int32))
    pp = prompt.ctypes.data_as(C.POINTER(C.c_int32))
    assert L.nh_decode_prepare(m._h, pp, N_PROMPT, N_PREDICT) == 0
    stream = torch.cuda.ExternalStream(L.nh_model_stream(m._h))
    out = np.zeros(N_PREDICT, dtype=np.int32)
    op = out.ctypes.data_as(C.POINTER(C.c_int32))

    for _ in range(args.warmup):
        assert L.nh_decode_run(m._h, N_PREDICT) == 0
    assert L.nh_decode_result(m._h, N_PREDICT, op) == 0
    ref_tokens = out.tolist()
    if args.profile:
        # Launches after the warm-up: exactly one step = N_PREDICT x launches_per_token kernels.
        assert L.nh_decode_run(m._h, N_PREDICT) == 0
        assert L.nh_decode_result(m._h, N_PREDICT, op) == 0
        print(json.dumps({"profile_step_launches": N_PREDICT * L.nh_generate_launches(m._h),
                          "launches_before": (N_PROMPT - 1 + args.warmup * N_PREDICT) * L.nh_generate_launches(m._h)}))
        return

    # ---- timed region: K decode steps, inputs resident in HBM (weights 4.2 GB > L2)
    clocks = ClockSampler(local_rank)
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        L.nh_decode_run(m._h, N_PREDICT)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    assert L.nh_decode_result(m._h, N_PREDICT, op) == 0
    assert out.tolist() == ref_tokens, "replayed decode diverged"
    ms = max_over_ranks(ms, dist)
    ms_per_step = ms / args.steps
    value = world * N_PREDICT * args.steps / (ms / 1000.0)
    launches_per_token = L.nh_generate_launches(m._h)
    gpu_launches = args.steps * N_PREDICT * launches_per_token

    # ---- dominant kernel timed alone on the same stream, cycling through all
    # 16 layers so every launch streams its weights from HBM: the fused MoE
    # block (router + gate/up + down) when the step uses it, else gate/up.
    fused = launches_per_token == 2 + 4 * 16
    which, kbytes = (3, MOE_LAYER_BYTES) if fused else (0, GATE_UP_BYTES)
    reps = 20
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    L.nh_decode_kernel_loop(m._h, which, 2)
    k0.record(stream)
    n_k = L.nh_decode_kernel_loop(m._h, which, reps)
    k1.record(stream)
    torch.cuda.synchronize()
    assert n_k > 0, f"kernel loop failed ({n_k})"
    k_ms = k0.elapsed_time(k1) / n_k
    peaks = measured_peaks()
    achieved = kbytes / (k_ms / 1000.0) / 1e9
    traffic = traffic_summary("moe_layer" if fused else "moe_gate_up")
    kname = ("nh_moe_layer (router + 8 experts gate/up + down, Q4_K/Q6_K)" if fused
             else "nh_moe_gate_up (8 experts x gate+up, Q4_K)")
    roofline = {"kernel": kname, "bound": "hbm", "achieved": achieved,
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "algorithmic_bytes_per_launch": kbytes, "avg_launch_us": k_ms * 1000.0,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)"}
    tok_s_1 = N_PREDICT * args.steps / (ms / 1000.0)
    step_bytes = step_bytes_per_token()
    step_gbs = step_bytes * tok_s_1 / 1e9
    step_roofline = {"bytes_per_token": step_bytes, "achieved": step_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": step_gbs / peaks["hbm_gbs"]}

    # ---- e2e: the public API call with host buffers (prompt H2D, ids D2H inside)
    for _ in range(2):
        nh.GreedyGenerateCached(m, prompt.tolist(), N_PREDICT, False)
    barrier()
    e2e_steps = max(3, min(args.steps, 50))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        got = nh.GreedyGenerateCached(m, prompt.tolist(), N_PREDICT, False)
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, dist)
    assert got == ref_tokens
    e2e = {"value": world * N_PREDICT * e2e_steps / e2e_s, "unit": "tok/s",
           "h2d_bytes_per_step": N_PROMPT * 4 + 32, "d2h_bytes_per_step": N_PREDICT * 4 + 32,
           "api": "GreedyGenerateCached (nh_generate, mode 0)"}

    ep_line = None if args.no_ep else run_ep_batched(args, dist, rank, world, local_rank, path, m)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        dt, cpu_tokens = cpu_oracle_run(path, 8, threads)
        cpu = {"value": 8 / dt, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"oracle GreedyGenerateCached: prompt {N_PROMPT} (one-shot prefill) + 8 greedy ids, "
                         f"{dt:.1f} s", "ids_match_gpu": cpu_tokens == ref_tokens[:8]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "q4k/q6k x q8k int dot, f32 accumulate",
                "data": "synthetic (seeded random-init GGUF of the OLMoE-1B-7B shape)",
                "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": N_PROMPT + N_PREDICT,
                           "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                           "step": f"{N_PREDICT} decode positions", "l2": "inputs larger than L2 (4.2 GB weights)"},
                "clocks": clk, "roofline": roofline, "step_roofline": step_roofline, "e2e": e2e,
                "gpu_launches": gpu_launches, "cpu_baseline": cpu, "ep_batched": ep_line}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
