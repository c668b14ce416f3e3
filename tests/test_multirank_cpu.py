"""CPU, world size 2 over gloo: the multi-rank pieces of bench.py and the
host side of expert parallelism.  Batch-1 decode does not shard, so N GPUs
run N replicas with no data-path collective; the only cross-rank step is
taking the slowest rank's time, and the reference arm runs on rank 0 alone.
Expert-parallel batched streaming plans each rank's slot-pool waves over the
all-gathered selections; the plans of both ranks must cover every pick once,
on the rank that owns its expert."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = r"""
import datetime, json, os, sys
sys.path.insert(0, sys.argv[1])
import torch.distributed as dist
import bench
dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
rank = dist.get_rank()
got = bench.max_over_ranks(10.0 + 5.0 * rank, dist, device="cpu")
dist.barrier()
dist.destroy_process_group()
print(json.dumps({"rank": rank, "max": got}))
"""


def test_max_over_ranks_gloo_world_size_2(tmp_path):
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER, str(ROOT)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        out, err = p.communicate(timeout=120)
        assert p.returncode == 0, err[-2000:]
        outs.append(json.loads(out.strip().splitlines()[-1]))
    assert sorted(o["rank"] for o in outs) == [0, 1]
    assert all(o["max"] == 15.0 for o in outs)


def test_max_over_ranks_without_a_group_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(3.25, None) == 3.25


def test_reference_arm_on_nonzero_rank_exits_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


EP_WAVES_WORKER = r"""
import datetime, json, os, sys
sys.path.insert(0, sys.argv[1])
import numpy as np
import torch
import torch.distributed as dist
import nuthatch_b200 as nh
dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
rank, world = dist.get_rank(), dist.get_world_size()
n_expert, k, n_tok, per = 32, 8, 16, 4
rng = np.random.default_rng(100 + rank)
mine = np.stack([rng.choice(n_expert, k, replace=False) for _ in range(n_tok)]).astype(np.int32)
# The selections of every rank's tokens, rank-major, as after the all-gather.
parts = [torch.zeros_like(torch.from_numpy(mine)) for _ in range(world)]
dist.all_gather(parts, torch.from_numpy(mine))
sel = torch.cat(parts).numpy().ravel()
first, count = rank * (n_expert // world), n_expert // world
waves, wave_of = nh.plan_waves(sel, n_expert, per, shard=(first, count))
picks = []
for w, ids in enumerate(waves):
    slot_of = [-1] * n_expert
    for s, e in enumerate(ids):
        slot_of[e] = s
    picks += nh.group_wave_pairs(sel, k, wave_of, w, slot_of, per)[3]
got = [None] * world
dist.all_gather_object(got, {"rank": rank, "picks": sorted(picks), "waves": len(waves),
                             "sel": sel.tolist()})
dist.barrier()
dist.destroy_process_group()
if rank == 0:
    print(json.dumps(got))
"""


def test_expert_parallel_wave_plans_gloo_world_size_2():
    """The host side of expert-parallel batched streaming on two gloo ranks:
    every rank plans its own expert shard over the all-gathered selections,
    and the ranks' wave pairs together cover every pick exactly once, each on
    the rank that owns its expert (the rank the combine reads it from)."""
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, "-c", EP_WAVES_WORKER, str(ROOT)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        out, err = p.communicate(timeout=120)
        assert p.returncode == 0, err[-2000:]
        outs.append(out)
    got = json.loads(outs[0].strip().splitlines()[-1])
    sel = got[0]["sel"]
    assert got[1]["sel"] == sel and len(sel) == 2 * 16 * 8
    owner = {j: sel[j] // 16 for j in range(len(sel))}
    for g in got:
        assert all(owner[j] == g["rank"] for j in g["picks"])
        assert 1 <= g["waves"] <= 4  # 16 served experts through 4 LRU slots
    assert sorted(got[0]["picks"] + got[1]["picks"]) == list(range(len(sel)))
