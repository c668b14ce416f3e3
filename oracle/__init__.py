"""ORACLE — test infrastructure only.

The CPU restatement of nuthatch's forward (liboracle.so, built from
olmoe_oracle.cc) and the reference's own compiled cache/trace/io code
(_ref/libref.so).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use this package, as the checker; the product never imports it.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
P = C.POINTER


class OracleConfig(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_ff", C.c_uint32), ("n_expert", C.c_uint32),
                ("n_expert_used", C.c_uint32), ("n_vocab", C.c_uint32), ("n_ctx_train", C.c_uint32),
                ("rope_freq_base", C.c_float), ("rms_eps", C.c_float)]


def _ptr(a, t):
    return None if a is None else a.ctypes.data_as(P(t))


_olib = None
_rlib = None


def olib() -> C.CDLL:
    global _olib
    if _olib is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        L = C.CDLL(str(so))
        L.oracle_model_load.restype = C.c_void_p
        L.oracle_model_load.argtypes = [C.c_char_p]
        L.oracle_model_free.argtypes = [C.c_void_p]
        L.oracle_model_config.argtypes = [C.c_void_p, P(OracleConfig)]
        L.oracle_set_threads.argtypes = [C.c_int]
        L.oracle_threads.restype = C.c_int
        L.oracle_generate.restype = C.c_int
        L.oracle_generate.argtypes = [C.c_void_p, C.c_int, P(C.c_int32), C.c_int, C.c_int, C.c_int, P(C.c_int32),
                                      P(C.c_int32), P(C.c_float), P(C.c_float), P(C.c_float), P(C.c_float)]
        L.oracle_stream_generate.restype = C.c_int
        L.oracle_stream_generate.argtypes = [C.c_void_p, P(C.c_int32), C.c_int, C.c_int, C.c_int, C.c_int,
                                             C.c_int, C.c_int, P(C.c_uint64), P(C.c_int32), P(C.c_int64),
                                             P(C.c_int64)]
        L.oracle_forward.restype = C.c_int
        L.oracle_forward.argtypes = [C.c_void_p, P(C.c_int32), C.c_int, C.c_int, P(C.c_float)]
        L.oracle_dequant.argtypes = [C.c_int, C.c_void_p, C.c_int64, P(C.c_float)]
        L.oracle_quantize_q8k.argtypes = [P(C.c_float), C.c_int64, C.c_void_p]
        L.oracle_matvec.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, P(C.c_float), P(C.c_float)]
        L.oracle_rms_norm_mul.argtypes = [P(C.c_float), P(C.c_float), C.c_int64, C.c_float, P(C.c_float)]
        L.oracle_rope_neox.argtypes = [P(C.c_float), C.c_int, C.c_int, C.c_float]
        L.oracle_softmax.argtypes = [P(C.c_float), C.c_int64]
        L.oracle_exp.restype = C.c_float
        L.oracle_exp.argtypes = [C.c_float]
        L.oracle_replay.restype = C.c_int64
        L.oracle_replay.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32), P(C.c_int64),
                                    P(C.c_uint32), C.c_uint32, C.c_uint32, P(C.c_int64)]
        L.oracle_tensor_info.argtypes = [C.c_void_p, C.c_char_p, P(C.c_int64), P(C.c_int), P(C.c_uint64),
                                         P(C.c_uint64)]
        _olib = L
    return _olib


def ref_available() -> bool:
    return (HERE / "_ref" / "libref.so").exists()


def rlib() -> C.CDLL:
    """The reference's own src/cache + src/trace + src/io compiled into oracle/_ref."""
    global _rlib
    if _rlib is None:
        L = C.CDLL(str(HERE / "_ref" / "libref.so"))
        L.ref_replay.restype = C.c_int64
        L.ref_replay.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32), P(C.c_int64),
                                 P(C.c_uint32), C.c_uint32, C.c_uint32, P(C.c_int64)]
        L.ref_sweep_budgets.argtypes = [C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32), P(C.c_int64),
                                        P(C.c_uint32), P(C.c_uint32), C.c_int, P(C.c_double)]
        L.ref_sweep_pin_ratio.argtypes = [C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32), P(C.c_int64),
                                          P(C.c_uint32), C.c_uint32, P(C.c_double)]
        L.ref_write_trace.argtypes = [C.c_char_p, C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32),
                                      P(C.c_uint32), P(C.c_int64), P(C.c_uint32)]
        L.ref_read_trace.restype = C.c_int64
        L.ref_read_trace.argtypes = [C.c_char_p, C.c_int, P(C.c_uint32), P(C.c_uint32), P(C.c_int64), C.c_int64,
                                     C.c_int64, P(C.c_uint32), P(C.c_uint32), P(C.c_int64), P(C.c_uint32)]
        L.ref_read_at.argtypes = [C.c_char_p, C.c_uint64, C.c_uint64, C.c_void_p]
        _rlib = L
    return _rlib


def set_threads(n: int) -> None:
    olib().oracle_set_threads(int(n))


class OracleModel:
    def __init__(self, path: str):
        self._h = olib().oracle_model_load(str(path).encode())
        if not self._h:
            raise RuntimeError(f"oracle could not load {path}")
        c = OracleConfig()
        olib().oracle_model_config(self._h, C.byref(c))
        self.cfg = {f: getattr(c, f) for f, _ in OracleConfig._fields_}

    def generate(self, prompt, n_predict: int, norm_topk: bool = False, mode: int = 0, trace: bool = False,
                 hidden: bool = False, logits: bool = False) -> dict:
        """mode 0 cached (one-shot prefill), 1 uncached, 2 token-by-token prefill."""
        c = self.cfg
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        n_tok = p.size + n_predict - 1
        L, K = c["n_layers"], c["n_expert_used"]
        toks = np.zeros(n_predict, dtype=np.int32)
        sel = np.zeros((n_tok, L, K), dtype=np.int32) if trace else None
        gap = np.zeros((n_tok, L), dtype=np.float32) if trace else None
        hid = np.zeros((n_predict, L, c["n_embd"]), dtype=np.float32) if hidden else None
        lg = np.zeros((n_predict, c["n_vocab"]), dtype=np.float32) if logits else None
        lgap = np.zeros(n_predict, dtype=np.float32)
        olib().oracle_generate(self._h, mode, _ptr(p, C.c_int32), int(p.size), n_predict, int(norm_topk),
                               _ptr(toks, C.c_int32), _ptr(sel, C.c_int32), _ptr(gap, C.c_float),
                               _ptr(hid, C.c_float), _ptr(lg, C.c_float), _ptr(lgap, C.c_float))
        out = {"tokens": toks.tolist(), "logit_gap": lgap}
        if trace:
            out["sel"], out["gap"] = sel, gap
        if hidden:
            out["hidden"] = hid
        if logits:
            out["logits"] = lg
        return out

    def forward(self, tokens, norm_topk: bool = False) -> np.ndarray:
        """Logits of every position of a full-sequence forward, [T][V]."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.zeros((t.size, self.cfg["n_vocab"]), dtype=np.float32)
        if olib().oracle_forward(self._h, _ptr(t, C.c_int32), int(t.size), int(norm_topk), _ptr(out, C.c_float)):
            raise RuntimeError("oracle forward failed")
        return out

    def stream_generate(self, prompt, n_predict: int, norm_topk: bool, capacity: int, policy: int = 0,
                        pin_slots: int = 0, usage: np.ndarray | None = None) -> dict:
        c = self.cfg
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        toks = np.zeros(n_predict, dtype=np.int32)
        hits = np.zeros(c["n_layers"], dtype=np.int64)
        misses = np.zeros(c["n_layers"], dtype=np.int64)
        u = None if usage is None else np.ascontiguousarray(np.asarray(usage, dtype=np.uint64))
        rc = olib().oracle_stream_generate(self._h, _ptr(p, C.c_int32), int(p.size), n_predict, int(norm_topk),
                                           capacity, policy, pin_slots, _ptr(u, C.c_uint64), _ptr(toks, C.c_int32),
                                           _ptr(hits, C.c_int64), _ptr(misses, C.c_int64))
        if rc != 0:
            raise RuntimeError(f"oracle stream_generate failed ({rc})")
        return {"tokens": toks.tolist(), "hits": hits, "misses": misses}

    def tensor_info(self, name: str):
        ne = (C.c_int64 * 4)()
        t = C.c_int()
        off = C.c_uint64()
        nb = C.c_uint64()
        if olib().oracle_tensor_info(self._h, name.encode(), ne, C.byref(t), C.byref(off), C.byref(nb)) != 0:
            return None
        return {"ne": tuple(ne), "type": t.value, "offset": off.value, "nbytes": nb.value}

    def close(self):
        if self._h:
            olib().oracle_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequant(type_: int, raw: bytes, n: int) -> np.ndarray:
    y = np.zeros(n, dtype=np.float32)
    buf = C.create_string_buffer(raw, len(raw))
    olib().oracle_dequant(type_, buf, n, _ptr(y, C.c_float))
    return y


def quantize_q8k(x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = C.create_string_buffer(x.size // 256 * 292)
    olib().oracle_quantize_q8k(_ptr(x, C.c_float), x.size, out)
    return out.raw


def matvec(type_: int, raw: bytes, n: int, rows: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    buf = C.create_string_buffer(raw, len(raw))
    olib().oracle_matvec(type_, buf, n, rows, _ptr(x, C.c_float), _ptr(y, C.c_float))
    return y


def flat_trace(records, n_layers):
    """records: list of (layer, [experts]) -> arrays for the replay ABIs."""
    layer = np.array([l for l, _ in records] or [0], dtype=np.uint32)
    offsets = np.zeros(len(records) + 1, dtype=np.int64)
    if records:
        offsets[1:] = np.cumsum([len(e) for _, e in records])
    experts = np.array([x for _, e in records for x in e] or [0], dtype=np.uint32)
    return layer, offsets, experts


def replay(kind: int, records, n_layers: int, n_expert: int, a: int, b: int = 0, use_ref: bool = False):
    layer, offsets, experts = flat_trace(records, n_layers)
    acc = C.c_int64()
    L = rlib() if use_ref else olib()
    fn = L.ref_replay if use_ref else L.oracle_replay
    hits = fn(kind, n_layers, n_expert, len(records), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
              _ptr(experts, C.c_uint32), a, b, C.byref(acc))
    return int(hits), int(acc.value)


def ref_replay_pin_usage(records, n_layers: int, n_expert: int, pin: int, lru: int, usage) -> tuple[int, int]:
    """The reference's compiled LearnedPinPolicy(pin, lru) over the records with
    a given usage histogram (dense [n_layers][n_expert] counts): (hits, accesses)."""
    layer, offsets, experts = flat_trace(records, n_layers)
    u = np.ascontiguousarray(np.asarray(usage, dtype=np.uint64).reshape(n_layers, n_expert))
    acc = C.c_int64()
    fn = rlib().ref_replay_pin_usage
    fn.restype = C.c_int64
    fn.argtypes = [C.c_uint32, C.c_uint32, C.c_int64, P(C.c_uint32), P(C.c_int64), P(C.c_uint32), C.c_uint32,
                   C.c_uint32, P(C.c_uint64), P(C.c_int64)]
    hits = fn(n_layers, n_expert, len(records), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
              _ptr(experts, C.c_uint32), pin, lru, _ptr(u, C.c_uint64), C.byref(acc))
    return int(hits), int(acc.value)


def ref_sweep_budgets(records, n_layers, n_expert, budgets):
    layer, offsets, experts = flat_trace(records, n_layers)
    b = np.asarray(budgets, dtype=np.uint32)
    out = np.zeros(3 * len(b), dtype=np.float64)
    n = rlib().ref_sweep_budgets(n_layers, n_expert, len(records), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
                                 _ptr(experts, C.c_uint32), _ptr(b, C.c_uint32), len(b), _ptr(out, C.c_double))
    return out[:3 * n].reshape(n, 3)


def ref_read_trace(path: str, text: bool):
    L = rlib()
    nl, ne, tot = C.c_uint32(), C.c_uint32(), C.c_int64()
    n = L.ref_read_trace(str(path).encode(), int(text), C.byref(nl), C.byref(ne), C.byref(tot), 0, 0, None, None,
                         None, None)
    if n < 0:
        return None
    token = np.zeros(max(n, 1), dtype=np.uint32)
    layer = np.zeros(max(n, 1), dtype=np.uint32)
    offsets = np.zeros(n + 1, dtype=np.int64)
    experts = np.zeros(max(tot.value, 1), dtype=np.uint32)
    L.ref_read_trace(str(path).encode(), int(text), C.byref(nl), C.byref(ne), C.byref(tot), n, tot.value,
                     _ptr(token, C.c_uint32), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
                     _ptr(experts, C.c_uint32))
    recs = [(int(token[i]), int(layer[i]), experts[offsets[i]:offsets[i + 1]].tolist()) for i in range(n)]
    return nl.value, ne.value, recs
