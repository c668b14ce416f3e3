"""Expert-parallel batched decode (experts sharded E/N per GPU, tokens
all-gathered, pick rows returned by an all-to-all, combine in top-k order on
the token's GPU, moe.cc:51-60): every sequence's ids equal the single-GPU
batched decode, which equals decoding it alone.

* One rank (world size 1) on one GPU: the EP code path with its own NCCL
  communicator, against nh_generate_batch, with the full model and with a
  shard model that holds every expert.
* Two ranks (two GPUs; skipped on a one-GPU box): each process loads only
  its expert shard and decodes its half of the sequences; ids equal the
  single-GPU batch, with CUDA graphs and eagerly.
* Batched streaming with expert parallelism (configuration 5 across GPUs):
  each rank streams only its E/N experts through its own slots per layer
  (LRU and learned pin), in waves; ids equal the single-GPU resident batch.
  The one-rank form equals the single-GPU streaming batch.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import nuthatch_b200 as nh
from nuthatch_b200 import synth
from nuthatch_b200._lib import lib

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict", [
    ("MINI", 6, 5, 8),
    ("OLMOE_1B7B", 4, 6, 6),
])
def test_ep_one_rank_matches_single_gpu_batch(gpu, synth_dir, spec_name, n_seq, n_prompt, n_predict):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    cfg = m.config()
    prompts = np.random.default_rng(5).integers(0, cfg.n_vocab, (n_seq, n_prompt)).tolist()
    ref = nh.generate_batch_ex(m, prompts, n_predict, False)["tokens"]
    ep = nh.ExpertGroup(nh.ExpertGroup.new_id(), 1, 0)
    try:
        assert nh.generate_batch_ex(m, prompts, n_predict, False, ep=ep)["tokens"] == ref
        shard = nh.OlmoeModel.LoadExpertShard(str(path), 0, cfg.n_expert)
        assert shard is not None
        assert nh.generate_batch_ex(shard, prompts, n_predict, False, ep=ep)["tokens"] == ref
        shard.close()
    finally:
        ep.close()
    # A partial shard serves only the expert-parallel call.
    part = nh.OlmoeModel.LoadExpertShard(str(path), 0, cfg.n_expert // 2)
    assert part is not None
    with pytest.raises(nh.NhError):
        nh.generate_ex(part, prompts[0], 2, False)
    with pytest.raises(nh.NhError):
        nh.generate_batch_ex(part, prompts, 2, False)
    part.close()


def _gpu_count() -> int:
    import torch

    return torch.cuda.device_count()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict,use_graph", [
    ("MINI", 3, 5, 8, True),
    ("OLMOE_1B7B", 4, 6, 6, True),
    ("OLMOE_1B7B", 2, 4, 4, False),
])
def test_ep_two_ranks_match_single_gpu_batch(gpu, synth_dir, tmp_path, spec_name, n_seq, n_prompt, n_predict,
                                             use_graph):
    world = 2
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    out = tmp_path / "ep.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "ep_worker.py"), str(path), str(out), str(n_seq), str(n_prompt), str(n_predict),
           "1", "1" if use_graph else "0"]
    subprocess.run(cmd, env=env, cwd=ROOT, check=True)
    res = json.loads(out.read_text())
    m = nh.OlmoeModel.Load(str(path))
    ref = nh.generate_batch_ex(m, res["prompts"], n_predict, False)["tokens"]
    assert res["tokens"] == ref
    assert all(ms > 0 for ms in res["decode_ms"])


@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict,capacity,policy", [
    ("MINI", 5, 5, 6, 4, "lru"),
    ("GRANITE_MOE", 4, 6, 4, 8, "learned_pin"),
])
def test_ep_one_rank_streaming_batch_matches_single_gpu(gpu, synth_dir, spec_name, n_seq, n_prompt, n_predict,
                                                        capacity, policy):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    m = nh.OlmoeModel.Load(str(path))
    cfg = m.config()
    prompts = np.random.default_rng(7).integers(0, cfg.n_vocab, (n_seq, n_prompt)).tolist()
    ref = nh.generate_batch_ex(m, prompts, n_predict, False)["tokens"]
    kw = {}
    if policy == "learned_pin":
        cal = nh.RoutingTrace()
        nh.GreedyGenerateCachedTrace(m, prompts[0], 8, False, cal)
        kw = dict(policy="learned_pin", pin_slots=(capacity * 3 + 3) // 4, usage=nh.BuildUsage(cal, cfg.n_expert).counts)
    m.close()
    sm = nh.StreamingModel.Load(str(path))
    single = nh.streaming_generate_batch_ex(sm, prompts, n_predict, False, capacity, **kw)
    ep = nh.ExpertGroup(nh.ExpertGroup.new_id(), 1, 0)
    try:
        grouped = nh.streaming_generate_batch_ex(sm, prompts, n_predict, False, capacity, ep=ep, **kw)
    finally:
        ep.close()
    sm.close()
    assert single["tokens"] == ref and grouped["tokens"] == ref
    assert grouped["waves"] == single["waves"]
    assert np.array_equal(grouped["hits"], single["hits"]) and np.array_equal(grouped["misses"], single["misses"])


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("spec_name,n_seq,n_prompt,n_predict,capacity,policy", [
    ("MINI", 3, 5, 6, 2, "lru"),                 # 8 of 16 experts per GPU, 2 slots: several waves
    ("GRANITE_MOE", 4, 6, 4, 4, "lru"),          # configuration 5's budget 8 across two GPUs: 4 each
    ("GRANITE_MOE", 4, 6, 4, 4, "learned_pin"),
])
def test_ep_two_ranks_streaming_batch_match_single_gpu_batch(gpu, synth_dir, tmp_path, spec_name, n_seq, n_prompt,
                                                             n_predict, capacity, policy):
    world = 2
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    out = tmp_path / "ep_stream.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "ep_worker.py"), str(path), str(out), str(n_seq), str(n_prompt), str(n_predict),
           "0", "0", f"stream:{capacity}:{policy}"]
    subprocess.run(cmd, env=env, cwd=ROOT, check=True)
    res = json.loads(out.read_text())
    m = nh.OlmoeModel.Load(str(path))
    ref = nh.generate_batch_ex(m, res["prompts"], n_predict, False)["tokens"]
    assert res["tokens"] == ref
    assert all(w > 0 for w in res["waves"]) and all(b > 0 for b in res["h2d_bytes"])
