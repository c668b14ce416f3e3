"""One rank of the expert-parallel GPU test (launched by tests/test_gpu_ep.py
under torch.distributed.run, one process per GPU).

Rank 0 makes the group id; it travels to the other ranks over a gloo process
group.  Every rank loads its expert shard, decodes its share of the seeded
prompts with nh_generate_batch_timed, and rank 0 writes every rank's ids (in
sequence order) and decode times to the output file.

An optional eighth argument `stream:<capacity>:<policy>` runs the batched
streaming form instead (nh_stream_generate_batch_ep): every rank loads the
streaming model and streams its expert shard through `capacity` slots per
layer; learned pin takes its usage from a resident trace of the first prompt.
The per-rank wave and H2D counts are written too."""
from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import nuthatch_b200 as nh  # noqa: E402
from nuthatch_b200._lib import NhConfig, lib  # noqa: E402


def prompts_for(n_total: int, n_prompt: int, n_vocab: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, n_vocab, (n_total, n_prompt), dtype=np.int32)


def main() -> None:
    path, out, n_seq, n_prompt, n_predict, shard_load, use_graph = (
        sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5]), sys.argv[6] == "1",
        sys.argv[7] == "1")
    mode = sys.argv[8] if len(sys.argv) > 8 else "resident"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    assert lib().nh_set_device(local) == 0
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    box = [nh.ExpertGroup.new_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    ep = nh.ExpertGroup(box[0], world, rank)
    c = NhConfig()
    assert lib().nh_gguf_probe(path.encode(), c) > 0
    prompts = prompts_for(n_seq * world, n_prompt, c.n_vocab, 11)
    mine = prompts[rank * n_seq:(rank + 1) * n_seq]
    extra = {}
    if mode.startswith("stream:"):
        _, capacity, policy = mode.split(":")
        kw = {}
        if policy == "learned_pin":
            full = nh.OlmoeModel.Load(path)
            cal = nh.RoutingTrace()
            nh.GreedyGenerateCachedTrace(full, prompts[0].tolist(), 8, False, cal)
            kw = dict(policy="learned_pin", pin_slots=(int(capacity) * 3 + 3) // 4,
                      usage=nh.BuildUsage(cal, c.n_expert).counts)
            full.close()
        m = nh.StreamingModel.Load(path)
        assert m is not None
        r = nh.streaming_generate_batch_ex(m, mine.tolist(), n_predict, False, int(capacity), ep=ep, **kw)
        extra = {"waves": r["waves"], "h2d_bytes": r["h2d_bytes"]}
    else:
        first, count = nh.ExpertGroup.shard(c.n_expert, world, rank)
        m = nh.OlmoeModel.LoadExpertShard(path, first, count) if shard_load else nh.OlmoeModel.Load(path)
        assert m is not None
        r = nh.generate_batch_ex(m, mine.tolist(), n_predict, False, use_graph=use_graph, ep=ep)
    gathered = [None] * world
    dist.all_gather_object(gathered, dict(extra, tokens=r["tokens"], decode_ms=r["decode_ms"]))
    if rank == 0:
        res = {"tokens": [t for g in gathered for t in g["tokens"]], "decode_ms": [g["decode_ms"] for g in gathered],
               "prompts": prompts.tolist()}
        for k in extra:
            res[k] = [g[k] for g in gathered]
        Path(out).write_text(json.dumps(res))
    m.close()
    ep.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
