"""CPU, world size 2 over gloo: the multi-rank pieces of bench.py.  Batch-1
decode does not shard, so N GPUs run N replicas with no data-path
collective; the only cross-rank step is taking the slowest rank's time, and
the reference arm runs on rank 0 alone."""
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
