"""CPU: GGUF/K-quant formats, the oracle's arithmetic, and the reference
tests' structural anchors on the oracle itself."""
from __future__ import annotations

import numpy as np
import pytest
from gguf import GGUFReader
from gguf.quants import dequantize

import oracle
from nuthatch_b200 import synth
from tests.ref_fixtures import write_tiny_olmoe


@pytest.fixture(scope="module")
def mini(synth_dir):
    return synth.cached(synth.MINI, synth_dir)


def test_synth_gguf_readable_by_gguf_py(mini):
    r = GGUFReader(str(mini))
    names = {t.name for t in r.tensors}
    assert "token_embd.weight" in names and "output.weight" in names
    assert "blk.1.ffn_down_exps.weight" in names
    kinds = {t.name: int(t.tensor_type) for t in r.tensors}
    assert kinds["blk.1.attn_v.weight"] == 14 and kinds["blk.0.attn_v.weight"] == 12
    assert kinds["output.weight"] == 14 and kinds["blk.0.ffn_gate_inp.weight"] == 0
    assert r.fields["general.architecture"].contents() == "olmoe"


def test_synth_is_seeded_and_thread_independent(tmp_path):
    a = synth.write(synth.MINI, tmp_path / "a.gguf", threads=1).read_bytes()
    b = synth.write(synth.MINI, tmp_path / "b.gguf", threads=7).read_bytes()
    assert a == b
    c = synth.write(synth.replace(synth.MINI, seed=99), tmp_path / "c.gguf").read_bytes()
    assert a != c


def test_oracle_dequant_matches_gguf_py(mini):
    """Pins the Q4_K/Q6_K/F32 bit layouts against gguf-py's dequantisers."""
    r = GGUFReader(str(mini))
    for t in r.tensors:
        ref = dequantize(t.data, t.tensor_type).reshape(-1).astype(np.float32)
        mine = oracle.dequant(int(t.tensor_type), np.asarray(t.data).tobytes(), ref.size)
        assert np.array_equal(ref, mine), t.name


def _q8k_blocks(raw: bytes):
    n = len(raw) // 292
    out = []
    for b in range(n):
        blk = raw[292 * b:292 * (b + 1)]
        d = np.frombuffer(blk[:4], np.float32)[0]
        qs = np.frombuffer(blk[4:260], np.int8)
        bs = np.frombuffer(blk[260:292], np.int16)
        out.append((d, qs, bs))
    return out


def test_q8k_quantisation_semantics():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(256 * 4).astype(np.float32)
    x[256:512] = 0
    x[600] = -9.0
    blocks = _q8k_blocks(oracle.quantize_q8k(x))
    for b, (d, qs, bs) in enumerate(blocks):
        xb = x[256 * b:256 * (b + 1)]
        assert np.array_equal(bs, qs.reshape(16, 16).astype(np.int32).sum(1))
        if not np.any(xb):
            assert d == 0 and not np.any(qs)
            continue
        i = int(np.argmax(np.abs(xb)))
        assert qs[i] == -127  # the largest magnitude maps to -127
        assert np.max(np.abs(qs.astype(np.float32) * d - xb)) <= abs(d) * 0.5 + 1e-6


@pytest.mark.parametrize("name", ["blk.0.attn_q.weight", "blk.1.attn_v.weight", "output.weight",
                                  "blk.0.ffn_gate_inp.weight"])
def test_oracle_integer_dot_equals_dequantised_dot(mini, name):
    """Two independent oracle paths agree: integer super-block dots versus
    f32 dots of the dequantised weights with the dequantised Q8_K activation."""
    r = GGUFReader(str(mini))
    t = next(t for t in r.tensors if t.name == name)
    n0 = int(t.shape[0])
    rows = int(np.prod(t.shape)) // n0
    raw = np.asarray(t.data).tobytes()
    x = np.random.default_rng(1).standard_normal(n0).astype(np.float32)
    y = oracle.matvec(int(t.tensor_type), raw, n0, rows, x)
    w = dequantize(t.data, t.tensor_type).reshape(rows, n0).astype(np.float64)
    if int(t.tensor_type) == 0:
        xq = x.astype(np.float64)
    else:
        xq = np.concatenate([q.astype(np.float64) * float(d) for d, q, _ in _q8k_blocks(oracle.quantize_q8k(x))])
    ref = w @ xq
    assert np.max(np.abs(y - ref)) <= 1e-4 * np.max(np.abs(ref))


def exp_inputs():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-104, 89, 20000), rng.uniform(-1, 1, 20000), rng.uniform(-20, 0, 20000),
                        [0.0, -0.0, 1.0, -1.0, 88.7, -87.3, -103.9, 88.72283935546875, -104.0, 89.0]])
    return x.astype(np.float32)


def test_exp_cw_accuracy():
    """The shared exp (Cody-Waite + degree-7 Taylor) is within 2 ulp of exp
    over the range the softmax and SiLU use; it saturates like expf."""
    x = exp_inputs()
    got = np.array([oracle.olib().oracle_exp(float(v)) for v in x], dtype=np.float32)
    ref = np.exp(x.astype(np.float64))
    finite = (ref < np.finfo(np.float32).max) & (ref > np.finfo(np.float32).tiny)
    ulp = np.spacing(ref[finite].astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got[finite] - ref[finite]) / ulp) <= 2.0
    assert got[x > 88.8].tolist() == [np.inf] * int((x > 88.8).sum())
    assert np.all(got[x < -104] == 0)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    return write_tiny_olmoe(tmp_path_factory.mktemp("tiny") / "gen_olmoe.gguf")


def test_oracle_reference_anchors(tiny):
    om = oracle.OracleModel(tiny)
    assert om.cfg["n_vocab"] == 16 and om.cfg["n_layers"] == 2
    for nt in (False, True):
        a = om.generate([3, 7, 2, 5], 6, norm_topk=nt, mode=1)["tokens"]  # GreedyGenerate
        b = om.generate([3, 7, 2, 5], 6, norm_topk=nt, mode=0)["tokens"]  # GreedyGenerateCached
        c = om.generate([3, 7, 2, 5], 6, norm_topk=nt, mode=2)["tokens"]  # token-by-token (streaming order)
        assert a == b == c
        assert all(0 <= t < 16 for t in a)


def test_oracle_causality(tiny):
    """ForwardTest.ShapeFiniteCausal: changing the last id leaves position-0 logits unchanged."""
    om = oracle.OracleModel(tiny)
    l0 = om.forward([3, 7, 1, 4], norm_topk=True)
    l1 = om.forward([3, 7, 1, 9], norm_topk=True)
    assert l0.shape == (4, 16) and np.all(np.isfinite(l0))
    assert np.array_equal(l0[0], l1[0])
    assert not np.array_equal(l0[3], l1[3])


def test_oracle_full_forward_last_row_equals_cached_step(tiny, mini):
    """The top-5 tool's logits (one cached step after a one-pass prompt) are
    the last row of the full-sequence forward (olmoe_forward_main.cc:39-52),
    bit for bit, with and without norm_topk."""
    for path in (tiny, str(mini)):
        om = oracle.OracleModel(path)
        for toks in ([3, 7, 1, 4], [5], [1, 2, 3, 4, 5, 6, 7, 8, 9]):
            for nt in (False, True):
                full = om.forward(toks, norm_topk=nt)[-1]
                step = om.generate(toks, 1, norm_topk=nt, mode=0, logits=True)["logits"][0]
                assert np.array_equal(full, step)


def test_oracle_thread_count_does_not_change_results(mini):
    om = oracle.OracleModel(str(mini))
    outs = []
    for n in (1, 3, 8, 2):
        oracle.set_threads(n)
        outs.append(om.generate([1, 2, 3, 4, 5], 5, mode=0, hidden=True))
    for o in outs[1:]:
        assert o["tokens"] == outs[0]["tokens"]
        assert np.array_equal(o["hidden"], outs[0]["hidden"])
