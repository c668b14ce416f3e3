"""The fused form of resident decode against the separate kernels it
replaces: the MoE-block kernel (nh_moe_layer: router, gate/up and down in one
grid) and the six separate kernels per layer.  Greedy ids, per-layer hidden
states, logits and routing records are identical bit for bit across the two,
with CUDA graphs and eagerly.  Each form runs in its own process
(NH_FUSED_MOE is read once per process)."""
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
from nuthatch_b200._lib import lib
path, out, n_prompt, n_predict, norm_topk = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5] == "1"
m = nh.OlmoeModel.Load(path)
prompt = np.random.default_rng(n_prompt).integers(0, m.config().n_vocab, n_prompt).tolist()
g = nh.generate_ex(m, prompt, n_predict, norm_topk, trace=True, hidden=True, logits=True)
e = nh.generate_ex(m, prompt, n_predict, norm_topk, use_graph=False, trace=True, hidden=True, logits=True)
np.savez(out, tokens=np.array(g["tokens"]), hidden=g["hidden"], logits=g["logits"], sel=g["sel"],
         e_tokens=np.array(e["tokens"]), e_hidden=e["hidden"], e_sel=e["sel"],
         launches=np.array(lib().nh_generate_launches(m._h)))
"""

FORMS = {"moe": {}, "split": {"NH_FUSED_MOE": "0"}}


def _run(path, out, env_over, n_prompt, n_predict, norm_topk):
    env = dict(os.environ, **env_over)
    subprocess.run([sys.executable, "-c", SCRIPT, str(path), str(out), str(n_prompt), str(n_predict),
                    "1" if norm_topk else "0"], env=env, cwd=ROOT, check=True, timeout=300)
    return np.load(out)


@pytest.mark.parametrize("spec_name,n_prompt,n_predict,norm_topk", [
    ("MINI", 12, 10, False),       # n_embd 512, n_ff 256, 16 experts top-4
    ("MINI", 12, 10, True),        # renormalised top-k weights
    ("MINI_GQA", 5, 8, False),     # GQA, every expert selected (top-8 of 8)
    ("MINI", 200, 4, False),       # four 64-position attention splits per head
    ("OLMOE_1B7B", 420, 3, False),  # 7 splits x 16 heads: more attention items than attention CTAs
    ("OLMOE_1B7B", 16, 12, False),  # the full-size layer: 64 experts top-8, Q4_K/Q6_K mix
])
def test_fused_forms_match_separate_kernels(gpu, synth_dir, tmp_path, spec_name, n_prompt, n_predict, norm_topk):
    path = synth.cached(getattr(synth, spec_name), synth_dir)
    res = {k: _run(path, tmp_path / f"{k}.npz", env, n_prompt, n_predict, norm_topk) for k, env in FORMS.items()}
    n_layers = getattr(synth, spec_name).n_layers
    # The forms really differ: 4 and 6 kernels per layer (plus embed and lm_head).
    assert [int(res[k]["launches"]) for k in FORMS] == [2 + 4 * n_layers, 2 + 6 * n_layers]
    for key in ("tokens", "hidden", "logits", "sel", "e_tokens", "e_hidden", "e_sel"):
        assert np.array_equal(res["moe"][key], res["split"][key]), key
    assert np.array_equal(res["moe"]["tokens"], res["moe"]["e_tokens"])
    assert np.array_equal(res["moe"]["hidden"], res["moe"]["e_hidden"])
