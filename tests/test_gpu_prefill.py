"""One-shot prompt prefill (the reference's first GreedyGenerateCached step,
generate.cc:63-91): the prompt positions before the last run as rows of the
batched kernels instead of one position per step.

* nh_prefill_qk + nh_prefill_attention against nh_attention_step run position
  by position over the same inputs: identical K/V rows and attention outputs
  (both follow the 64-position split arithmetic).
* Whole generation with the batched prefill against the position-by-position
  prompt (NH_PREFILL=0, a separate process since it is read once): identical
  ids, routing trace, per-layer hidden states and logits, including prompts
  longer than one prefill chunk; and against the oracle's GreedyGenerateCached.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from nuthatch_b200 import synth
from nuthatch_b200._lib import lib

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REL_TOL = 2e-2


@pytest.mark.parametrize("n_head,n_head_kv,head_dim,pos0,n_tok", [
    (16, 16, 128, 0, 150),    # OLMoE heads: one to three splits, queries of every regime
    (16, 16, 128, 70, 45),    # rows that start after cached positions
    (16, 8, 64, 0, 33),       # Granite-shaped GQA, a partial query block
    (4, 4, 128, 100, 200),    # more queries than one block, four splits
])
def test_prefill_attention_matches_position_by_position(gpu, n_head, n_head_kv, head_dim, pos0, n_tok):
    import torch

    L = lib()
    dev = torch.device("cuda")
    rng = np.random.default_rng(1000 * n_head + n_tok)
    dq, dkv = n_head * head_dim, n_head_kv * head_dim
    max_seq = pos0 + n_tok + 8
    eps, scale = 1e-5, 1.0 / float(np.sqrt(head_dim))
    cs = np.zeros(max_seq * head_dim, dtype=np.float32)
    L.nh_rope_table(10000.0, head_dim, max_seq, cs.ctypes.data_as(C.POINTER(C.c_float)))
    rope = torch.from_numpy(cs).to(dev)
    qn = torch.from_numpy(rng.uniform(0.5, 1.5, dq).astype(np.float32)).to(dev)
    kn = torch.from_numpy(rng.uniform(0.5, 1.5, dkv).astype(np.float32)).to(dev)
    q = torch.from_numpy(rng.standard_normal((n_tok, dq)).astype(np.float32)).to(dev)
    k = torch.from_numpy(rng.standard_normal((n_tok, dkv)).astype(np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((n_tok, dkv)).astype(np.float32)).to(dev)
    cache0 = rng.standard_normal((2, max_seq, dkv)).astype(np.float32)
    kc = {n: torch.from_numpy(cache0[0].copy()).to(dev) for n in ("pf", "step")}
    vc = {n: torch.from_numpy(cache0[1].copy()).to(dev) for n in ("pf", "step")}
    P = lambda t: C.c_void_p(t.data_ptr())
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    qr = torch.empty(n_tok, dq, device=dev)
    out_pf = torch.empty(n_tok, dq, device=dev)
    assert L.nh_prefill_qk(P(q), P(k), P(v), P(qn), P(kn), eps, n_tok, pos0, n_head, n_head_kv, head_dim, P(rope),
                           P(kc["pf"]), P(vc["pf"]), max_seq, P(qr), s) == 0
    assert L.nh_prefill_attention(P(qr), n_tok, pos0, n_head, n_head_kv, head_dim, scale, P(kc["pf"]), P(vc["pf"]),
                                  max_seq, P(out_pf), s) == 0

    scratch = torch.zeros(int(L.nh_attention_scratch_bytes(n_head, head_dim, max_seq)), dtype=torch.uint8,
                          device=dev)
    out_step = torch.empty(n_tok, dq, device=dev)
    state = torch.zeros(8, dtype=torch.int32, device=dev)
    for t in range(n_tok):
        state[0] = pos0 + t
        assert L.nh_attention_step(P(state), P(q[t]), P(k[t]), P(v[t]), P(qn), P(kn), eps, n_head, n_head_kv,
                                   head_dim, P(rope), scale, P(kc["step"]), P(vc["step"]), max_seq, P(scratch),
                                   P(out_step[t]), s) == 0
    torch.cuda.synchronize()
    a, b = out_pf.cpu().numpy(), out_step.cpu().numpy()
    assert np.all(np.isfinite(a))
    assert np.max(np.abs(a - b)) <= REL_TOL * np.max(np.abs(b))
    assert np.array_equal(a, b)
    assert np.array_equal(kc["pf"].cpu().numpy(), kc["step"].cpu().numpy())
    assert np.array_equal(vc["pf"].cpu().numpy(), vc["step"].cpu().numpy())


@pytest.mark.parametrize("n_seq,n_tok,pos0", [(3, 40, 0), (5, 17, 90), (2, 70, 33)])
def test_prefill_seqs_match_one_sequence_at_a_time(gpu, n_seq, n_tok, pos0):
    """The one-launch forms over n_seq sequences (embed with strided ids,
    QK/append into per-sequence caches, causal attention) equal the
    single-sequence forms called once per sequence."""
    import torch

    L = lib()
    dev = torch.device("cuda")
    rng = np.random.default_rng(7 * n_seq + n_tok)
    n_head, n_head_kv, head_dim = 16, 8, 64
    dq, dkv = n_head * head_dim, n_head_kv * head_dim
    max_seq = pos0 + n_tok + 5
    n_vocab, P_ids = 300, pos0 + n_tok + 3
    eps, scale = 1e-5, 1.0 / float(np.sqrt(head_dim))
    cs = np.zeros(max_seq * head_dim, dtype=np.float32)
    L.nh_rope_table(10000.0, head_dim, max_seq, cs.ctypes.data_as(C.POINTER(C.c_float)))
    rope = torch.from_numpy(cs).to(dev)
    qn = torch.from_numpy(rng.uniform(0.5, 1.5, dq).astype(np.float32)).to(dev)
    kn = torch.from_numpy(rng.uniform(0.5, 1.5, dkv).astype(np.float32)).to(dev)
    R = n_seq * n_tok
    q = torch.from_numpy(rng.standard_normal((R, dq)).astype(np.float32)).to(dev)
    k = torch.from_numpy(rng.standard_normal((R, dkv)).astype(np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((R, dkv)).astype(np.float32)).to(dev)
    cache0 = rng.standard_normal((2, n_seq, max_seq, dkv)).astype(np.float32)
    kc = {n: torch.from_numpy(cache0[0].copy()).to(dev) for n in ("all", "one")}
    vc = {n: torch.from_numpy(cache0[1].copy()).to(dev) for n in ("all", "one")}
    table = torch.from_numpy(rng.standard_normal((n_vocab, dq)).astype(np.float32)).to(dev)
    ids = torch.from_numpy(rng.integers(0, n_vocab, (n_seq, P_ids)).astype(np.int32)).to(dev)
    P = lambda t: C.c_void_p(t.data_ptr())
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    h_all, qr_all, out_all = (torch.empty(R, dq, device=dev) for _ in range(3))
    assert L.nh_prefill_embed_seqs(C.c_void_p(ids.data_ptr() + 4 * pos0), P_ids, n_seq, n_tok, P(table), 0, dq,
                                   n_vocab, P(h_all), P(err), s) == 0
    assert L.nh_prefill_qk_seqs(P(q), P(k), P(v), P(qn), P(kn), eps, n_seq, n_tok, pos0, n_head, n_head_kv, head_dim,
                                P(rope), P(kc["all"]), P(vc["all"]), max_seq, P(qr_all), s) == 0
    assert L.nh_prefill_attention_seqs(P(qr_all), n_seq, n_tok, pos0, n_head, n_head_kv, head_dim, scale,
                                       P(kc["all"]), P(vc["all"]), max_seq, P(out_all), s) == 0

    h_one, qr_one, out_one = (torch.empty(R, dq, device=dev) for _ in range(3))
    for b in range(n_seq):
        rows = slice(b * n_tok, (b + 1) * n_tok)
        assert L.nh_prefill_embed(C.c_void_p(ids[b].data_ptr() + 4 * pos0), n_tok, P(table), 0, dq, n_vocab,
                                  P(h_one[rows]), P(err), s) == 0
        assert L.nh_prefill_qk(P(q[rows]), P(k[rows]), P(v[rows]), P(qn), P(kn), eps, n_tok, pos0, n_head,
                               n_head_kv, head_dim, P(rope), P(kc["one"][b]), P(vc["one"][b]), max_seq,
                               P(qr_one[rows]), s) == 0
        assert L.nh_prefill_attention(P(qr_one[rows]), n_tok, pos0, n_head, n_head_kv, head_dim, scale,
                                      P(kc["one"][b]), P(vc["one"][b]), max_seq, P(out_one[rows]), s) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want_h = table.cpu().numpy()[ids.cpu().numpy()[:, pos0:pos0 + n_tok].reshape(-1)]
    assert np.array_equal(h_all.cpu().numpy(), want_h)
    assert np.array_equal(h_all.cpu().numpy(), h_one.cpu().numpy())
    assert np.array_equal(qr_all.cpu().numpy(), qr_one.cpu().numpy())
    assert np.all(np.isfinite(out_all.cpu().numpy()))
    assert np.array_equal(out_all.cpu().numpy(), out_one.cpu().numpy())
    assert np.array_equal(kc["all"].cpu().numpy(), kc["one"].cpu().numpy())
    assert np.array_equal(vc["all"].cpu().numpy(), vc["one"].cpu().numpy())


def test_prefill_rejects_shapes_it_does_not_cover(gpu):
    L = lib()
    null = None
    # head_dim not a multiple of 32, and rows beyond the cache: refused before any launch.
    assert L.nh_prefill_attention(null, 4, 0, 4, 4, 48, 0.1, null, null, 16, null, null) == -1
    assert L.nh_prefill_qk(null, null, null, null, null, 1e-5, 8, 10, 4, 4, 128, null, null, null, 16, null,
                           null) == -1


SCRIPT = r"""
import sys
import numpy as np
import nuthatch_b200 as nh
path, out, n_prompt, n_predict, norm_topk = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5] == "1"
m = nh.OlmoeModel.Load(path)
prompt = np.random.default_rng(n_prompt + 7).integers(0, m.config().n_vocab, n_prompt).tolist()
g = nh.generate_ex(m, prompt, n_predict, norm_topk, trace=True, hidden=True, logits=True)
np.savez(out, tokens=np.array(g["tokens"]), hidden=g["hidden"], logits=g["logits"], sel=g["sel"], gap=g["gap"],
         prompt=np.array(prompt))
"""


def _run(path, out, prefill, n_prompt, n_predict, norm_topk):
    env = dict(os.environ, NH_PREFILL="1" if prefill else "0")
    subprocess.run([sys.executable, "-c", SCRIPT, str(path), str(out), str(n_prompt), str(n_predict),
                    "1" if norm_topk else "0"], env=env, cwd=ROOT, check=True, timeout=600)
    return np.load(out)


@pytest.mark.parametrize("spec_name,n_prompt,n_predict,norm_topk,with_oracle", [
    ("MINI", 12, 10, False, True),
    ("MINI", 12, 10, True, True),
    ("MINI_GQA", 40, 6, False, True),
    ("MINI", 700, 4, False, False),        # two prefill chunks (512 + 187 rows), eleven splits
    ("OLMOE_1B7B", 16, 24, False, True),   # the benchmark workload
    ("OLMOE_1B7B", 300, 4, False, False),  # >= 128 rows: Q4_K products on tcgen05, Q6_K on mma.sync
])
def test_generation_with_prefill_matches_position_by_position(gpu, synth_dir, tmp_path, spec_name, n_prompt,
                                                              n_predict, norm_topk, with_oracle):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    pf = _run(path, tmp_path / "pf.npz", True, n_prompt, n_predict, norm_topk)
    st = _run(path, tmp_path / "st.npz", False, n_prompt, n_predict, norm_topk)
    for key in ("tokens", "hidden", "logits", "sel", "gap"):
        assert np.array_equal(pf[key], st[key]), key
    if with_oracle:
        ora = oracle.OracleModel(str(path)).generate(pf["prompt"].tolist(), n_predict, mode=0, norm_topk=norm_topk,
                                                      hidden=True)
        assert pf["tokens"].tolist() == ora["tokens"]
        err = np.max(np.abs(pf["hidden"] - ora["hidden"])) / np.max(np.abs(ora["hidden"]))
        assert err <= REL_TOL, err
