"""The per-layer cooperative MoE kernel (nh_moe_layer: router, gate/up and
down in one grid) against the three separate kernels it replaces in resident
decode: greedy ids, per-layer hidden states, logits and routing records are
identical bit for bit, with CUDA graphs and eagerly.  Each form runs in its
own process (NH_FUSED_MOE is read once per process)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from nuthatch_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys
import numpy as np
import nuthatch_b200 as nh
path, out, n_prompt, n_predict, norm_topk = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5] == "1"
m = nh.OlmoeModel.Load(path)
prompt = np.random.default_rng(n_prompt).integers(0, m.config().n_vocab, n_prompt).tolist()
g = nh.generate_ex(m, prompt, n_predict, norm_topk, trace=True, hidden=True, logits=True)
e = nh.generate_ex(m, prompt, n_predict, norm_topk, use_graph=False, trace=True, hidden=True, logits=True)
np.savez(out, tokens=np.array(g["tokens"]), hidden=g["hidden"], logits=g["logits"], sel=g["sel"],
         e_tokens=np.array(e["tokens"]), e_hidden=e["hidden"], e_sel=e["sel"])
"""


def _run(path, out, fused, n_prompt, n_predict, norm_topk):
    env = dict(os.environ, NH_FUSED_MOE="1" if fused else "0")
    subprocess.run([sys.executable, "-c", SCRIPT, str(path), str(out), str(n_prompt), str(n_predict),
                    "1" if norm_topk else "0"], env=env, cwd=ROOT, check=True, timeout=900)
    return np.load(out)


@pytest.mark.parametrize("spec_name,n_prompt,n_predict,norm_topk", [
    ("MINI", 12, 10, False),       # n_embd 512, n_ff 256, 16 experts top-4
    ("MINI", 12, 10, True),        # renormalised top-k weights
    ("MINI_GQA", 5, 8, False),     # every expert selected (top-8 of 8)
    ("OLMOE_1B7B", 16, 12, False),  # the full-size layer: 64 experts top-8, Q4_K/Q6_K mix
])
def test_fused_moe_layer_matches_separate_kernels(gpu, synth_dir, tmp_path, spec_name, n_prompt, n_predict,
                                                  norm_topk):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    fused = _run(path, tmp_path / "fused.npz", True, n_prompt, n_predict, norm_topk)
    split = _run(path, tmp_path / "split.npz", False, n_prompt, n_predict, norm_topk)
    for key in ("tokens", "hidden", "logits", "sel", "e_tokens", "e_hidden", "e_sel"):
        assert np.array_equal(fused[key], split[key]), key
    assert np.array_equal(fused["tokens"], fused["e_tokens"])
    assert np.array_equal(fused["hidden"], fused["e_hidden"])
