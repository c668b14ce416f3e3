"""The tcgen05 grouped Q4_K product (nh_batch_rowdot_tc: one kind::i8 MMA per
32-value sub-block, accumulators in tensor memory) against the mma.sync and
dp4a engines of nh_batch_rowdot on the same inputs: identical bits, for
ungrouped (dense projection) and grouped (per-expert token lists, SwiGLU)
products, every K the kernels take, partial row and token tiles, and empty
groups."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from nuthatch_b200._lib import lib

pytestmark = pytest.mark.gpu

ENGINE_DP4A, ENGINE_MMA, ENGINE_TC = 1, 2, 3
STORE, RESIDUAL, SWIGLU = 0, 1, 2
Q4K = 12


class NhGroupedRowDot(C.Structure):
    _fields_ = [("w", C.c_void_p), ("w2", C.c_void_p), ("mstride", C.c_uint64), ("mstride2", C.c_uint64),
                ("type", C.c_int32), ("type2", C.c_int32), ("n", C.c_int64), ("rows", C.c_int64),
                ("n_groups", C.c_int32), ("off", C.c_void_p), ("cnt", C.c_void_p), ("act_idx", C.c_void_p),
                ("out_idx", C.c_void_p), ("n_tok", C.c_int32), ("max_tokens", C.c_int32), ("q8", C.c_void_p),
                ("out", C.c_void_p), ("out_stride", C.c_int64), ("mode", C.c_int32), ("engine", C.c_int32),
                ("err", C.c_void_p)]


def q4k_blocks(rng, n_blocks: int) -> np.ndarray:
    """Random but well-formed Q4_K super-blocks: small positive d/dmin."""
    b = rng.integers(0, 256, (n_blocks, 144), dtype=np.uint8)
    d = rng.uniform(1e-3, 4e-3, n_blocks).astype(np.float16).view(np.uint16)
    dm = rng.uniform(1e-4, 2e-3, n_blocks).astype(np.float16).view(np.uint16)
    b[:, 0] = d & 0xFF
    b[:, 1] = d >> 8
    b[:, 2] = dm & 0xFF
    b[:, 3] = dm >> 8
    return b


def run(engine, *, w, w2, n, rows, n_groups, off, cnt, act_idx, out_idx, n_tok, max_tokens, q8, out0, mode,
        mstride):
    import torch

    L = lib()
    out = out0.clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    g = NhGroupedRowDot(P(w), P(w2), mstride, mstride, Q4K, Q4K, n, rows, n_groups, P(off), P(cnt), P(act_idx),
                        P(out_idx), n_tok, max_tokens, P(q8), P(out), out.shape[1], mode, engine, P(err))
    rc = L.nh_batch_rowdot_tc(C.byref(g), None) if engine == ENGINE_TC else L.nh_batch_rowdot(C.byref(g), None)
    assert rc == 0, (engine, rc)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


def prep_q8(x_np, n):
    import torch

    L = lib()
    rows = x_np.shape[0]
    x = torch.from_numpy(x_np).cuda()
    q8 = torch.zeros(int(L.nh_batch_q8_bytes(rows, n)), dtype=torch.uint8, device="cuda")
    L.nh_batch_prep.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_float, C.c_int, C.c_int64,
                                C.c_void_p, C.c_void_p, C.c_void_p]
    assert L.nh_batch_prep(C.c_void_p(x.data_ptr()), n, rows, None, 1e-5, 0, n, C.c_void_p(q8.data_ptr()), None,
                           None) == 0
    return q8


@pytest.mark.parametrize("n,rows,n_tok,mode", [
    (2048, 2048, 300, STORE),      # OLMoE Q/O projections of a prefill chunk: partial token tile
    (2048, 2048, 128, RESIDUAL),   # residual accumulate
    (1024, 2048, 200, STORE),      # K = 4 super-blocks (expert down shape)
    (512, 200, 160, STORE),        # partial row tile, K = 2
    (256, 384, 129, RESIDUAL),     # K = 1
])
def test_tc_dense_matches_other_engines(gpu, n, rows, n_tok, mode):
    import torch

    lib().nh_batch_rowdot_tc.argtypes = [C.c_void_p, C.c_void_p]
    lib().nh_batch_rowdot.argtypes = [C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(n + rows + n_tok)
    nb = n // 256
    w = torch.from_numpy(np.concatenate([q4k_blocks(rng, rows * nb).reshape(-1), np.zeros(256, np.uint8)])).cuda()
    q8 = prep_q8(rng.standard_normal((n_tok, n)).astype(np.float32), n)
    out0 = torch.from_numpy(rng.standard_normal((n_tok, rows)).astype(np.float32)).cuda()
    kw = dict(w=w, w2=None, n=n, rows=rows, n_groups=1, off=None, cnt=None, act_idx=None, out_idx=None, n_tok=n_tok,
              max_tokens=n_tok, q8=q8, out0=out0, mode=mode, mstride=0)
    tc = run(ENGINE_TC, **kw)
    mma = run(ENGINE_MMA, **kw)
    assert np.all(np.isfinite(tc))
    assert np.array_equal(tc, mma)
    assert np.array_equal(tc, run(ENGINE_DP4A, **kw))


@pytest.mark.parametrize("n,rows,n_groups,n_tok,k", [
    (2048, 1024, 64, 512, 8),   # OLMoE gate/up of a 512-row prefill chunk
    (1024, 512, 32, 300, 8),    # Granite-shaped experts
    (512, 256, 8, 200, 4),      # mini shapes, some large groups
])
def test_tc_grouped_swiglu_matches_other_engines(gpu, n, rows, n_groups, n_tok, k):
    import torch

    lib().nh_batch_rowdot_tc.argtypes = [C.c_void_p, C.c_void_p]
    lib().nh_batch_rowdot.argtypes = [C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(n_groups * 7 + n_tok)
    nb = n // 256
    mstride = rows * nb * 144
    w = torch.from_numpy(np.concatenate([q4k_blocks(rng, n_groups * rows * nb).reshape(-1),
                                         np.zeros(256, np.uint8)])).cuda()
    w2 = torch.from_numpy(np.concatenate([q4k_blocks(rng, n_groups * rows * nb).reshape(-1),
                                          np.zeros(256, np.uint8)])).cuda()
    # Per-token top-k selections -> per-group lists in (token, slot) order;
    # group 0 is left empty on purpose.
    sel = np.stack([rng.choice(np.arange(1, n_groups), k, replace=False) for _ in range(n_tok)])
    pairs = [(e, t * k + i) for t in range(n_tok) for i, e in enumerate(sel[t])]
    cnt = np.bincount(sel.reshape(-1), minlength=n_groups).astype(np.int32)
    off = np.concatenate([[0], np.cumsum(cnt)[:-1]]).astype(np.int32)
    order = sorted(range(len(pairs)), key=lambda j: (pairs[j][0], pairs[j][1]))
    out_idx = np.array([pairs[j][1] for j in order], dtype=np.int32)
    act_idx = (out_idx // k).astype(np.int32)
    q8 = prep_q8(rng.standard_normal((n_tok, n)).astype(np.float32), n)
    out0 = torch.zeros((n_tok * k, rows), dtype=torch.float32, device="cuda")
    T = lambda a: torch.from_numpy(a).cuda()
    kw = dict(w=w, w2=w2, n=n, rows=rows, n_groups=n_groups, off=T(off), cnt=T(cnt), act_idx=T(act_idx),
              out_idx=T(out_idx), n_tok=n_tok, max_tokens=n_tok, q8=q8, out0=out0, mode=SWIGLU, mstride=mstride)
    tc = run(ENGINE_TC, **kw)
    assert np.all(np.isfinite(tc))
    assert np.array_equal(tc, run(ENGINE_MMA, **kw))
    # Plain grouped store (the down projection's form) too.
    kw.update(w2=None, mode=STORE)
    assert np.array_equal(run(ENGINE_TC, **kw), run(ENGINE_MMA, **kw))


def test_tc_declines_what_it_does_not_cover(gpu):
    import torch

    lib().nh_batch_rowdot_tc.argtypes = [C.c_void_p, C.c_void_p]
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    # Q6_K weights: NH_E_TYPE; K = 768 (not a power-of-two block count): NH_E_ARG.
    g = NhGroupedRowDot(P(w), None, 0, 0, 14, 14, 512, 16, 1, None, None, None, None, 8, 8, P(w), P(w), 16, 0, 3,
                        None)
    assert lib().nh_batch_rowdot_tc(C.byref(g), None) == -3
    g = NhGroupedRowDot(P(w), None, 0, 0, Q4K, Q4K, 768, 16, 1, None, None, None, None, 8, 8, P(w), P(w), 16, 0, 3,
                        None)
    assert lib().nh_batch_rowdot_tc(C.byref(g), None) == -1
