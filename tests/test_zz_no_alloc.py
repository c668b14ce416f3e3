"""nh_attention_step_static: the attention step for callers that cannot
allocate device memory (allocator hooks and pool callbacks, where allocating
would re-enter the allocator; plugin hosts that own every device allocation;
processes already at their allocator's limit).  Its split-combine scratch is
the library's own static device array, so the caller passes no scratch.

Checked against nh_attention_step (caller-provided scratch) on the same
inputs, on two calls in a row, within the tolerance the other parity tests use
(2e-2 relative) and, since both run the same kernel, bit for bit.  This file
is collected last so a stop-at-first-failure run has already run every other
test; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from nuthatch_b200._lib import lib

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2
NH_E_CAPACITY = -7
NH_E_ARG = -1


def _rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.mark.parametrize("n_head,n_head_kv,head_dim,max_seq,positions", [
    (16, 16, 128, 256, (130, 131)),   # OLMoE heads, three 64-position splits
    (16, 8, 64, 1024, (63, 64)),      # Granite-shaped GQA, one split then two
])
def test_static_scratch_matches_caller_scratch(gpu, n_head, n_head_kv, head_dim, max_seq, positions):
    import torch

    L = lib()
    dev = torch.device("cuda")
    rng = np.random.default_rng(n_head * 1000 + max_seq)
    dq, dkv = n_head * head_dim, n_head_kv * head_dim
    eps, scale = 1e-5, 1.0 / float(np.sqrt(head_dim))
    cs = np.zeros(max_seq * head_dim, dtype=np.float32)
    L.nh_rope_table(10000.0, head_dim, max_seq, cs.ctypes.data_as(C.POINTER(C.c_float)))
    rope = torch.from_numpy(cs).to(dev)
    qn = torch.from_numpy(rng.uniform(0.5, 1.5, dq).astype(np.float32)).to(dev)
    kn = torch.from_numpy(rng.uniform(0.5, 1.5, dkv).astype(np.float32)).to(dev)
    cache0 = rng.standard_normal((2, max_seq, dkv)).astype(np.float32)
    caches = {name: (torch.from_numpy(cache0[0].copy()).to(dev), torch.from_numpy(cache0[1].copy()).to(dev))
              for name in ("caller", "static")}
    scratch = torch.zeros(int(L.nh_attention_scratch_bytes(n_head, head_dim, max_seq)), dtype=torch.uint8,
                          device=dev)
    state = torch.zeros(8, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    s = C.c_void_p(stream.cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())

    for pos in positions:  # two calls in a row; the second reuses what the first left in the array
        q = torch.from_numpy(rng.standard_normal(dq).astype(np.float32)).to(dev)
        k = torch.from_numpy(rng.standard_normal(dkv).astype(np.float32)).to(dev)
        v = torch.from_numpy(rng.standard_normal(dkv).astype(np.float32)).to(dev)
        state.zero_()
        state[0] = pos
        outs = {}
        for name in ("caller", "static"):
            kc, vc = caches[name]
            out = torch.full((dq,), float("nan"), dtype=torch.float32, device=dev)
            if name == "caller":
                rc = L.nh_attention_step(P(state), P(q), P(k), P(v), P(qn), P(kn), eps, n_head, n_head_kv, head_dim,
                                         P(rope), scale, P(kc), P(vc), max_seq, P(scratch), P(out), s)
            else:
                rc = L.nh_attention_step_static(P(state), P(q), P(k), P(v), P(qn), P(kn), eps, n_head, n_head_kv,
                                                head_dim, P(rope), scale, P(kc), P(vc), max_seq, P(out), s)
            assert rc == 0, (name, rc)
            outs[name] = out
        torch.cuda.synchronize()
        assert int(state[5].item()) == 0, "device-side error recorded"
        a, b = outs["static"].cpu().numpy(), outs["caller"].cpu().numpy()
        assert np.all(np.isfinite(a))
        assert _rel_err(a, b) <= REL_TOL, (pos, _rel_err(a, b))
        assert np.array_equal(a, b), pos
        for i in range(2):  # the appended K/V rows agree too
            assert np.array_equal(caches["static"][i].cpu().numpy(), caches["caller"][i].cpu().numpy()), (pos, i)


def test_static_scratch_rejects_sizes_beyond_its_capacity(gpu):
    L = lib()
    # 16 heads x 128 fit up to max_seq 7936 in the 1 MiB array; 8192 does not.
    assert L.nh_attention_scratch_bytes(16, 128, 7936) <= 1 << 20 < L.nh_attention_scratch_bytes(16, 128, 8192)
    null = None
    assert L.nh_attention_step_static(null, null, null, null, null, null, 1e-5, 16, 16, 128, null, 0.088, null,
                                      null, 8192, null, null) == NH_E_CAPACITY
    assert L.nh_attention_step_static(null, null, null, null, null, null, 1e-5, 65, 65, 64, null, 0.125, null,
                                      null, 64, null, null) == NH_E_CAPACITY
    # Within capacity, a call with missing buffers is refused by the argument
    # checks, which run before the counters are cleared on the stream.
    assert L.nh_attention_step_static(null, null, null, null, null, null, 1e-5, 16, 16, 128, null, 0.088, null,
                                      null, 64, null, null) == NH_E_ARG
