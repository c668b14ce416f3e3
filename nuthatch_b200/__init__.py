"""nuthatch-b200: nuthatch's per-token OLMoE forward (resident and two-phase
streaming) on B200, as sm_100a CUDA kernels behind a C ABI.

This module mirrors the reference's C++ surface (namespace ``nuthatch``) with
the same names and argument meanings; every call goes through
libnuthatch_b200.so (``include/nh_api.h``).  Factories return ``None`` on
failure, as the reference's return nullptr.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import NhConfig, lib

__all__ = ["OlmoeConfig", "OlmoeModel", "StreamingModel", "GreedyGenerate", "GreedyGenerateCached",
           "GreedyGenerateCachedTrace", "StreamingGenerate", "generate_ex", "streaming_generate_ex",
           "RoutingRecord", "RoutingTrace", "WriteRoutingTrace", "ReadRoutingTrace", "ReadRoutingTraceText",
           "ReplayStats", "LruPolicy", "OsPageCachePolicy", "LearnedPinPolicy", "BuildUsage", "Replay",
           "SweepBudgets", "SweepBudgetsCalibrated", "SweepPinRatio", "ExpertReader", "ExpertSlotCache", "NhError", "ExpertGroup", "Tokenizer"]


class NhError(RuntimeError):
    pass


def _ptr(a: np.ndarray | None, ctype):
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(ctype))


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().nh_last_error().decode()
        raise NhError(f"{what} failed with code {rc}{': ' + msg if msg else ''}")


@dataclass
class OlmoeConfig:
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    n_vocab: int
    n_ctx_train: int
    rope_freq_base: float
    rms_eps: float

    def head_dim(self) -> int:
        return self.n_embd // self.n_head if self.n_head else 0

    @staticmethod
    def _from(c: NhConfig) -> "OlmoeConfig":
        return OlmoeConfig(c.n_layers, c.n_embd, c.n_head, c.n_head_kv, c.n_ff, c.n_expert, c.n_expert_used,
                           c.n_vocab, c.n_ctx_train, c.rope_freq_base, c.rms_eps)


@dataclass
class DTensorInfo:
    ne: tuple
    type: int
    data: int  # device pointer
    nbytes: int


class OlmoeModel:
    """The whole GGUF resident in HBM (olmoe_model.h:41-68)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def Load(path: str) -> Optional["OlmoeModel"]:
        h = lib().nh_model_load(str(path).encode())
        return OlmoeModel(h) if h else None

    @staticmethod
    def LoadExpertShard(path: str, first: int, count: int) -> Optional["OlmoeModel"]:
        """Non-expert tensors and experts [first, first+count) of each layer
        (expert parallelism); serves only generate_batch_ex with an ExpertGroup."""
        h = lib().nh_model_load_expert_shard(str(path).encode(), int(first), int(count))
        return OlmoeModel(h) if h else None

    def config(self) -> OlmoeConfig:
        c = NhConfig()
        _check(lib().nh_model_config(self._h, C.byref(c)), "nh_model_config")
        return OlmoeConfig._from(c)

    def tensor(self, name: str) -> Optional[DTensorInfo]:
        ne = (C.c_int64 * 4)()
        t = C.c_int32()
        d = C.c_void_p()
        nb = C.c_uint64()
        if lib().nh_model_tensor(self._h, name.encode(), ne, C.byref(t), C.byref(d), C.byref(nb)) != 0:
            return None
        return DTensorInfo(tuple(ne), t.value, d.value or 0, nb.value)

    def layer_tensor(self, layer: int, suffix: str) -> Optional[DTensorInfo]:
        return self.tensor(f"blk.{layer}.{suffix}")

    def launches_per_step(self) -> int:
        return lib().nh_generate_launches(self._h)

    def close(self) -> None:
        if self._h:
            lib().nh_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def generate_ex(model: OlmoeModel, ids: Sequence[int], n_predict: int, norm_topk: bool, *, mode: int = 0,
                use_graph: bool = True, trace: bool = False, hidden: bool = False, logits: bool = False) -> dict:
    """nh_generate with optional routing trace, per-layer hidden states and logits."""
    cfg = model.config()
    prompt = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    n_prompt = int(prompt.size)
    out = {"tokens": []}
    if n_prompt == 0 or n_predict <= 0:
        return out
    toks = np.zeros(n_predict, dtype=np.int32)
    n_tok = n_prompt + n_predict - 1
    L, K = cfg.n_layers, cfg.n_expert_used
    sel = np.zeros((n_tok, L, K), dtype=np.int32) if trace else None
    gap = np.zeros((n_tok, L), dtype=np.float32) if trace else None
    hid = np.zeros((n_predict, L, cfg.n_embd), dtype=np.float32) if hidden else None
    lg = np.zeros((n_predict, cfg.n_vocab), dtype=np.float32) if logits else None
    rc = lib().nh_generate(model._h, mode, _ptr(prompt, C.c_int32), n_prompt, n_predict, int(norm_topk),
                           int(use_graph), _ptr(toks, C.c_int32), _ptr(sel, C.c_int32), _ptr(gap, C.c_float),
                           _ptr(hid, C.c_float), _ptr(lg, C.c_float))
    _check(rc, "nh_generate")
    out["tokens"] = toks.tolist()
    if trace:
        out["sel"], out["gap"] = sel, gap
    if hidden:
        out["hidden"] = hid
    if logits:
        out["logits"] = lg
    return out


def GreedyGenerate(model: OlmoeModel, ids: Sequence[int], n_predict: int, norm_topk: bool) -> list[int]:
    """Full recompute per step (generate.cc:10-53)."""
    return generate_ex(model, ids, n_predict, norm_topk, mode=1)["tokens"]


def GreedyGenerateCached(model: OlmoeModel, ids: Sequence[int], n_predict: int, norm_topk: bool) -> list[int]:
    """KV-cached greedy decode (generate.cc:55-106)."""
    return generate_ex(model, ids, n_predict, norm_topk)["tokens"]


@dataclass
class RoutingRecord:
    token: int
    layer: int
    experts: list


@dataclass
class RoutingTrace:
    n_layers: int = 0
    n_expert: int = 0
    records: list = field(default_factory=list)

    def flat(self):
        layer = np.array([r.layer for r in self.records], dtype=np.uint32)
        token = np.array([r.token for r in self.records], dtype=np.uint32)
        offsets = np.zeros(len(self.records) + 1, dtype=np.int64)
        if self.records:
            offsets[1:] = np.cumsum([len(r.experts) for r in self.records])
        experts = np.array([e for r in self.records for e in r.experts], dtype=np.uint32)
        if experts.size == 0:
            experts = np.zeros(1, dtype=np.uint32)
        if layer.size == 0:
            layer = np.zeros(1, dtype=np.uint32)
            token = np.zeros(1, dtype=np.uint32)
        return token, layer, offsets, experts


def GreedyGenerateCachedTrace(model: OlmoeModel, ids: Sequence[int], n_predict: int, norm_topk: bool,
                              trace: RoutingTrace) -> list[int]:
    """Cached generation plus token-major routing records (generate.cc:108-181)."""
    cfg = model.config()
    r = generate_ex(model, ids, n_predict, norm_topk, trace=True)
    trace.n_layers, trace.n_expert = cfg.n_layers, cfg.n_expert
    trace.records = []
    if "sel" in r:
        for t in range(r["sel"].shape[0]):
            for l in range(cfg.n_layers):
                trace.records.append(RoutingRecord(t, l, [int(e) for e in r["sel"][t, l]]))
    return r["tokens"]


class ExpertGroup:
    """The communicator of an expert-parallel job (one process per GPU).

    Rank 0 makes the id with ExpertGroup.new_id(); every rank then calls
    ExpertGroup(id, world, rank) on its device at the same time."""

    ID_BYTES = 128

    @staticmethod
    def new_id() -> bytes:
        buf = (C.c_uint8 * ExpertGroup.ID_BYTES)()
        _check(lib().nh_ep_new_id(buf), "nh_ep_new_id (NCCL not loadable)")
        return bytes(buf)

    def __init__(self, group_id: bytes, world: int, rank: int):
        if len(group_id) != self.ID_BYTES:
            raise ValueError("group id must be 128 bytes")
        buf = (C.c_uint8 * self.ID_BYTES).from_buffer_copy(group_id)
        self._h = lib().nh_ep_create(buf, int(world), int(rank))
        if not self._h:
            raise NhError("nh_ep_create: " + lib().nh_last_error().decode())
        self.world, self.rank = int(world), int(rank)

    @staticmethod
    def shard(n_expert: int, world: int, rank: int) -> tuple[int, int]:
        """(first, count) of the experts rank owns (equal contiguous shares)."""
        per = n_expert // world
        return per * rank, per

    def close(self) -> None:
        if self._h:
            lib().nh_ep_free(self._h)
            self._h = None


def generate_batch_ex(model: OlmoeModel, prompts: Sequence[Sequence[int]], n_predict: int, norm_topk: bool,
                      use_graph: bool = True, ep: Optional[ExpertGroup] = None) -> dict:
    """Batched greedy decode of equal-length prompts; ids per sequence and the
    device time of the chunked prompt prefill and of the decode part.  With
    ep, every rank passes its own sequences (the same count everywhere) at the
    same time."""
    p = np.ascontiguousarray(np.asarray(prompts, dtype=np.int32))
    if p.ndim != 2:
        raise ValueError("prompts must all have the same length")
    n_seq, n_prompt = p.shape
    out = np.zeros((n_seq, n_predict), dtype=np.int32)
    pre, ms = C.c_double(0.0), C.c_double(0.0)
    _check(lib().nh_generate_batch_timed(model._h, None if ep is None else ep._h, _ptr(p, C.c_int32), n_seq,
                                         n_prompt, n_predict, int(norm_topk), int(use_graph), _ptr(out, C.c_int32),
                                         C.byref(pre), C.byref(ms)), "nh_generate_batch")
    return {"tokens": out.tolist(), "prefill_ms": pre.value, "decode_ms": ms.value}


def GreedyGenerateCachedBatch(model: OlmoeModel, prompts: Sequence[Sequence[int]], n_predict: int,
                              norm_topk: bool) -> list[list[int]]:
    """Each sequence's n_predict greedy ids; equal to GreedyGenerateCached on it alone."""
    return generate_batch_ex(model, prompts, n_predict, norm_topk)["tokens"]


class StreamingModel:
    """Non-expert weights in HBM, experts in pinned host memory (streaming_model.h:17-44)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def Load(path: str, pinned_store: bool = True) -> Optional["StreamingModel"]:
        h = lib().nh_stream_model_load(str(path).encode(), int(pinned_store))
        return StreamingModel(h) if h else None

    def config(self) -> OlmoeConfig:
        c = NhConfig()
        _check(lib().nh_stream_model_config(self._h, C.byref(c)), "nh_stream_model_config")
        return OlmoeConfig._from(c)

    def close(self) -> None:
        if self._h:
            lib().nh_stream_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def streaming_generate_ex(model: StreamingModel, ids: Sequence[int], n_predict: int, norm_topk: bool,
                          capacity: int, *, policy: str = "lru", pin_slots: int = 0,
                          usage: np.ndarray | None = None, trace: bool = False) -> dict:
    cfg = model.config()
    prompt = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    n_prompt = int(prompt.size)
    toks = np.zeros(max(n_predict, 1), dtype=np.int32)
    hits = np.zeros(cfg.n_layers, dtype=np.int64)
    misses = np.zeros(cfg.n_layers, dtype=np.int64)
    h2d = C.c_uint64(0)
    n_tok = max(n_prompt + n_predict - 1, 0)
    sel = np.zeros((max(n_tok, 1), cfg.n_layers, cfg.n_expert_used), dtype=np.int32) if trace else None
    u = None
    if policy == "learned_pin":
        u = np.ascontiguousarray(np.asarray(usage, dtype=np.uint64).reshape(cfg.n_layers, cfg.n_expert))
    rc = lib().nh_stream_generate(model._h, _ptr(prompt, C.c_int32) if n_prompt else None, n_prompt, n_predict,
                                  int(norm_topk), capacity, 1 if policy == "learned_pin" else 0, pin_slots,
                                  _ptr(u, C.c_uint64), _ptr(toks, C.c_int32), _ptr(hits, C.c_int64),
                                  _ptr(misses, C.c_int64), C.byref(h2d), _ptr(sel, C.c_int32))
    _check(rc, "nh_stream_generate")
    out = {"tokens": toks[:max(n_predict, 0)].tolist() if n_prompt and n_predict > 0 else [],
           "hits": hits, "misses": misses, "h2d_bytes": h2d.value}
    if trace:
        out["sel"] = sel[:n_tok]
    return out


def streaming_generate_batch_ex(model: StreamingModel, prompts: Sequence[Sequence[int]], n_predict: int,
                                norm_topk: bool, capacity: int, *, policy: str = "lru", pin_slots: int = 0,
                                usage: np.ndarray | None = None, ep: Optional[ExpertGroup] = None) -> dict:
    """Batched streaming decode (StreamingGenerateBatch): ids per sequence,
    per-layer hits/misses (one count per wave's Ensure), H2D bytes, the number
    of slot-pool waves and the decode device time.  With ep, every rank
    passes its own sequences at the same time and streams only its expert
    shard through `capacity` slots per layer; the counts are this rank's."""
    cfg = model.config()
    p = np.ascontiguousarray(np.asarray(prompts, dtype=np.int32))
    if p.ndim != 2:
        raise ValueError("prompts must all have the same length")
    n_seq, n_prompt = p.shape
    toks = np.zeros((n_seq, n_predict), dtype=np.int32)
    hits = np.zeros(cfg.n_layers, dtype=np.int64)
    misses = np.zeros(cfg.n_layers, dtype=np.int64)
    h2d, waves, ms = C.c_uint64(0), C.c_int64(0), C.c_double(0)
    u = None
    if policy == "learned_pin":
        u = np.ascontiguousarray(np.asarray(usage, dtype=np.uint64).reshape(cfg.n_layers, cfg.n_expert))
    _check(lib().nh_stream_generate_batch_ep(model._h, None if ep is None else ep._h, _ptr(p, C.c_int32), n_seq,
                                             n_prompt, n_predict, int(norm_topk), capacity,
                                             1 if policy == "learned_pin" else 0, pin_slots, _ptr(u, C.c_uint64),
                                             _ptr(toks, C.c_int32), _ptr(hits, C.c_int64), _ptr(misses, C.c_int64),
                                             C.byref(h2d), C.byref(waves), C.byref(ms)),
           "nh_stream_generate_batch_ep")
    return {"tokens": toks.tolist(), "hits": hits, "misses": misses, "h2d_bytes": h2d.value, "waves": waves.value,
            "decode_ms": ms.value}


class Tokenizer:
    """GPT-2 byte-level BPE tokenizer of an OLMoE GGUF (tokenizer.h:13-44):
    Encode(text) -> ids, Decode(ids) -> text; the rules are in
    include/nuthatch/tokenizer.h.  Host only."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def Load(path: str) -> Optional["Tokenizer"]:
        h = lib().nh_tokenizer_load(str(path).encode())
        return Tokenizer(h) if h else None

    @staticmethod
    def FromLists(vocab: Sequence[str | bytes], merges: Sequence[str | bytes] = ()) -> "Tokenizer":
        enc = [v.encode() if isinstance(v, str) else bytes(v) for v in vocab]
        mer = [m.encode() if isinstance(m, str) else bytes(m) for m in merges]
        va = (C.c_char_p * max(len(enc), 1))(*enc)
        ma = (C.c_char_p * max(len(mer), 1))(*mer)
        h = lib().nh_tokenizer_from_lists(va, len(enc), ma, len(mer))
        if not h:
            raise NhError("nh_tokenizer_from_lists failed")
        return Tokenizer(h)

    def vocab_size(self) -> int:
        return int(lib().nh_tokenizer_vocab_size(self._h))

    def token(self, id_: int) -> bytes:
        n = lib().nh_tokenizer_token(self._h, int(id_), None, 0)
        buf = C.create_string_buffer(max(n, 1))
        lib().nh_tokenizer_token(self._h, int(id_), buf, n)
        return buf.raw[:n]

    def Encode(self, text: str | bytes) -> list[int]:
        raw = text.encode() if isinstance(text, str) else bytes(text)
        ids = np.empty(max(len(raw), 1), dtype=np.int32)  # every id covers at least one byte
        n = lib().nh_tokenizer_encode(self._h, raw, len(raw), _ptr(ids, C.c_int32), ids.size)
        _check(min(int(n), 0), "nh_tokenizer_encode")
        return ids[:n].tolist()

    def DecodeBytes(self, ids: Sequence[int]) -> bytes:
        a = np.ascontiguousarray(np.asarray(list(ids), dtype=np.int32))
        n = lib().nh_tokenizer_decode(self._h, _ptr(a, C.c_int32), a.size, None, 0)
        _check(min(int(n), 0), "nh_tokenizer_decode")
        buf = C.create_string_buffer(max(n, 1))
        lib().nh_tokenizer_decode(self._h, _ptr(a, C.c_int32), a.size, buf, n)
        return buf.raw[:n]

    def Decode(self, ids: Sequence[int]) -> str:
        """The decoded bytes as text (bytes that are not UTF-8 become U+FFFD)."""
        return self.DecodeBytes(ids).decode("utf-8", errors="replace")

    @staticmethod
    def Split(text: str | bytes) -> list[tuple[int, int]]:
        """Pre-split chunks of the text as [begin, end) byte offsets."""
        raw = text.encode() if isinstance(text, str) else bytes(text)
        n = lib().nh_tokenizer_split(raw, len(raw), None, 0)
        _check(min(int(n), 0), "nh_tokenizer_split")
        b = np.zeros(max(2 * n, 2), dtype=np.int64)
        lib().nh_tokenizer_split(raw, len(raw), _ptr(b, C.c_int64), n)
        return [(int(b[2 * i]), int(b[2 * i + 1])) for i in range(n)]

    def close(self) -> None:
        if self._h:
            lib().nh_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def plan_waves(sel: Sequence[int], n_expert: int, per: int, pinned: Sequence[int] | None = None,
               shard: tuple[int, int] | None = None) -> tuple[list[list[int]], list[int]]:
    """The slot-pool waves of one batched streaming layer (nh_plan_waves):
    (id list per wave, wave of every expert or -1).  shard = (first, count)
    of the experts served here (all by default)."""
    s = np.ascontiguousarray(np.asarray(sel, dtype=np.int32).ravel())
    pin = np.zeros(n_expert, dtype=np.uint8)
    if pinned is not None:
        pin[np.asarray(list(pinned), dtype=np.int64)] = 1
    first, count = shard if shard is not None else (0, n_expert)
    wave_of = np.zeros(n_expert, dtype=np.int32)
    size = np.zeros(n_expert, dtype=np.int32)
    ids = np.zeros(n_expert, dtype=np.int32)
    n = lib().nh_plan_waves(_ptr(s, C.c_int32), int(s.size), n_expert, first, first + count, per,
                            _ptr(pin, C.c_uint8), _ptr(wave_of, C.c_int32), _ptr(size, C.c_int32),
                            _ptr(ids, C.c_int32))
    _check(min(n, 0), "nh_plan_waves")
    waves, k = [], 0
    for w in range(n):
        waves.append(ids[k:k + size[w]].tolist())
        k += int(size[w])
    return waves, wave_of.tolist()


def group_wave_pairs(sel: Sequence[int], k: int, wave_of: Sequence[int], w: int, slot_of: Sequence[int],
                     slots: int) -> tuple[list[int], list[int], list[int], list[int]]:
    """The pairs of wave w grouped by slot (nh_group_wave_pairs): off, cnt per
    slot, then the token row and pick index of every pair in slot order."""
    s = np.ascontiguousarray(np.asarray(sel, dtype=np.int32).ravel())
    wo = np.ascontiguousarray(np.asarray(wave_of, dtype=np.int32))
    so = np.ascontiguousarray(np.asarray(slot_of, dtype=np.int32))
    off = np.zeros(slots, dtype=np.int32)
    cnt = np.zeros(slots, dtype=np.int32)
    act = np.zeros(max(s.size, 1), dtype=np.int32)
    out = np.zeros(max(s.size, 1), dtype=np.int32)
    n = lib().nh_group_wave_pairs(_ptr(s, C.c_int32), int(s.size), k, int(wo.size), _ptr(wo, C.c_int32), w,
                                  _ptr(so, C.c_int32), slots, _ptr(off, C.c_int32), _ptr(cnt, C.c_int32),
                                  _ptr(act, C.c_int32), _ptr(out, C.c_int32))
    _check(min(n, 0), "nh_group_wave_pairs")
    return off.tolist(), cnt.tolist(), act[:n].tolist(), out[:n].tolist()


def StreamingGenerate(model: StreamingModel, ids: Sequence[int], n_predict: int, norm_topk: bool,
                      capacity: int) -> list[int]:
    """Two-phase streaming greedy decode with an LRU slot cache (streaming_forward.cc:228-253)."""
    return streaming_generate_ex(model, ids, n_predict, norm_topk, capacity)["tokens"]


# ------------------------------------------------------------------ traces
def WriteRoutingTrace(trace: RoutingTrace, path: str) -> bool:
    token, layer, offsets, experts = trace.flat()
    return lib().nh_trace_write(str(path).encode(), trace.n_layers, trace.n_expert, len(trace.records),
                                _ptr(token, C.c_uint32), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
                                _ptr(experts, C.c_uint32)) == 0


def _read(path: str, text: int, out: RoutingTrace) -> bool:
    nl, ne, tot = C.c_uint32(), C.c_uint32(), C.c_int64()
    n = lib().nh_trace_read(str(path).encode(), text, C.byref(nl), C.byref(ne), C.byref(tot), 0, 0, None, None,
                            None, None)
    if n < 0:
        return False
    token = np.zeros(max(n, 1), dtype=np.uint32)
    layer = np.zeros(max(n, 1), dtype=np.uint32)
    offsets = np.zeros(n + 1, dtype=np.int64)
    experts = np.zeros(max(tot.value, 1), dtype=np.uint32)
    n2 = lib().nh_trace_read(str(path).encode(), text, C.byref(nl), C.byref(ne), C.byref(tot), n, tot.value,
                             _ptr(token, C.c_uint32), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
                             _ptr(experts, C.c_uint32))
    if n2 != n:
        return False
    out.n_layers, out.n_expert = nl.value, ne.value
    out.records = [RoutingRecord(int(token[i]), int(layer[i]), experts[offsets[i]:offsets[i + 1]].tolist())
                   for i in range(n)]
    return True


def ReadRoutingTrace(path: str, out: RoutingTrace) -> bool:
    return _read(path, 0, out)


def ReadRoutingTraceText(path: str, out: RoutingTrace) -> bool:
    return _read(path, 1, out)


# ------------------------------------------------------------------ policies
@dataclass
class ReplayStats:
    accesses: int = 0
    hits: int = 0
    misses: int = 0

    def hit_rate(self) -> float:
        return self.hits / self.accesses if self.accesses else 0.0


@dataclass
class LruPolicy:
    n_layers: int
    slots_per_layer: int


@dataclass
class OsPageCachePolicy:
    capacity: int


@dataclass
class UsageHistogram:
    counts: np.ndarray  # [n_layers][n_expert] uint64


def BuildUsage(trace: RoutingTrace, n_expert: int | None = None) -> UsageHistogram:
    ne = n_expert or max(trace.n_expert, 1 + max((e for r in trace.records for e in r.experts), default=0))
    c = np.zeros((trace.n_layers, ne), dtype=np.uint64)
    for r in trace.records:
        if r.layer < trace.n_layers:
            for e in r.experts:
                c[r.layer, e] += 1
    return UsageHistogram(c)


@dataclass
class LearnedPinPolicy:
    n_layers: int
    pin_slots: int
    lru_slots: int
    usage: UsageHistogram


def Replay(trace: RoutingTrace, policy) -> ReplayStats:
    token, layer, offsets, experts = trace.flat()
    acc = C.c_int64()
    usage = None
    if isinstance(policy, LruPolicy):
        kind, a, b = 0, policy.slots_per_layer, 0
    elif isinstance(policy, OsPageCachePolicy):
        kind, a, b = 1, policy.capacity, 0
    else:
        kind, a, b = 2, policy.pin_slots, policy.lru_slots
        ne = max(trace.n_expert, policy.usage.counts.shape[1])
        u = np.zeros((trace.n_layers, ne), dtype=np.uint64)
        L = min(trace.n_layers, policy.usage.counts.shape[0])
        u[:L, :policy.usage.counts.shape[1]] = policy.usage.counts[:L]
        usage = np.ascontiguousarray(u)
        n_expert = ne
    n_expert = usage.shape[1] if usage is not None else trace.n_expert
    hits = lib().nh_replay(kind, trace.n_layers, n_expert, len(trace.records), _ptr(layer, C.c_uint32),
                           _ptr(offsets, C.c_int64), _ptr(experts, C.c_uint32), a, b, _ptr(usage, C.c_uint64),
                           C.byref(acc))
    return ReplayStats(acc.value, int(hits), acc.value - int(hits))


def SweepBudgets(trace: RoutingTrace, budgets: Sequence[int]) -> list[tuple]:
    token, layer, offsets, experts = trace.flat()
    b = np.asarray(budgets, dtype=np.uint32)
    out = np.zeros(3 * max(len(b), 1), dtype=np.float64)
    n = lib().nh_sweep_budgets(trace.n_layers, trace.n_expert, len(trace.records), _ptr(layer, C.c_uint32),
                               _ptr(offsets, C.c_int64), _ptr(experts, C.c_uint32), _ptr(b, C.c_uint32), len(b),
                               _ptr(out, C.c_double))
    kept = [x for x in budgets if x != 0]
    return [(kept[i], out[3 * i], out[3 * i + 1], out[3 * i + 2]) for i in range(n)]


def SweepBudgetsCalibrated(calibration: RoutingTrace, trace: RoutingTrace, budgets: Sequence[int]) -> list[tuple]:
    """Out-of-sample sweep: learned pin's usage from `calibration` (e.g. a
    trace written by an earlier run and read back), every policy replaying
    `trace`; rows (budget, learned, lru, os) as SweepBudgets."""
    _, cl, co, ce = calibration.flat()
    _, layer, offsets, experts = trace.flat()
    b = np.asarray(budgets, dtype=np.uint32)
    out = np.zeros(3 * max(len(b), 1), dtype=np.float64)
    n = lib().nh_sweep_budgets_calibrated(
        trace.n_layers, trace.n_expert, len(calibration.records), _ptr(cl, C.c_uint32), _ptr(co, C.c_int64),
        _ptr(ce, C.c_uint32), len(trace.records), _ptr(layer, C.c_uint32), _ptr(offsets, C.c_int64),
        _ptr(experts, C.c_uint32), _ptr(b, C.c_uint32), len(b), _ptr(out, C.c_double))
    if n < 0:
        raise NhError(f"nh_sweep_budgets_calibrated failed with code {n}")
    kept = [x for x in budgets if x != 0]
    return [(kept[i], out[3 * i], out[3 * i + 1], out[3 * i + 2]) for i in range(n)]


def SweepPinRatio(trace: RoutingTrace, budget: int) -> list[tuple]:
    token, layer, offsets, experts = trace.flat()
    out = np.zeros(budget + 1, dtype=np.float64)
    n = lib().nh_sweep_pin_ratio(trace.n_layers, trace.n_expert, len(trace.records), _ptr(layer, C.c_uint32),
                                 _ptr(offsets, C.c_int64), _ptr(experts, C.c_uint32), budget,
                                 _ptr(out, C.c_double))
    return [(p, budget - p, out[p]) for p in range(n)]


# ------------------------------------------------------------------ experts
class ExpertReader:
    """Per-expert byte slices of a GGUF (expert_reader.h:10-43)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def Open(path: str) -> Optional["ExpertReader"]:
        h = lib().nh_expert_reader_open(str(path).encode())
        return ExpertReader(h) if h else None

    def ExpertBytes(self, name: str) -> int:
        return int(lib().nh_expert_reader_bytes(self._h, name.encode()))

    def ReadExpert(self, name: str, idx: int) -> Optional[bytes]:
        n = self.ExpertBytes(name)
        if n == 0:
            return None
        buf = C.create_string_buffer(n)
        if lib().nh_expert_reader_read(self._h, name.encode(), idx, buf) != 0:
            return None
        return buf.raw

    def FailReadsAfter(self, n: int) -> None:
        """Host-side fault injection for tests: after n more successful reads
        every read fails as a short read would; n < 0 turns it off."""
        _check(lib().nh_expert_reader_fail_after(self._h, int(n)), "nh_expert_reader_fail_after")

    def __del__(self):
        try:
            if self._h:
                lib().nh_expert_reader_free(self._h)
        except Exception:
            pass


class ExpertSlotCache:
    """HBM slot pool of one layer (expert_slot_cache.h:16-64)."""

    def __init__(self, handle, reader):
        self._h = handle
        self._reader = reader

    @staticmethod
    def Create(cfg: OlmoeConfig, layer: int, capacity: int, reader: ExpertReader, *, policy: str = "lru",
               pin_slots: int = 0, usage_layer: np.ndarray | None = None) -> Optional["ExpertSlotCache"]:
        c = NhConfig(cfg.n_layers, cfg.n_embd, cfg.n_head, cfg.n_head_kv, cfg.n_ff, cfg.n_expert,
                     cfg.n_expert_used, cfg.n_vocab, cfg.n_ctx_train, cfg.rope_freq_base, cfg.rms_eps)
        u = None if usage_layer is None else np.ascontiguousarray(np.asarray(usage_layer, dtype=np.uint64))
        h = lib().nh_slot_cache_create(C.byref(c), layer, capacity, reader._h, 1 if policy == "learned_pin" else 0,
                                       pin_slots, _ptr(u, C.c_uint64))
        return ExpertSlotCache(h, reader) if h else None

    def Ensure(self, ids: Sequence[int]) -> dict:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        slots = np.zeros(max(a.size, 1), dtype=np.int32)
        _check(lib().nh_slot_cache_ensure(self._h, _ptr(a, C.c_int32), int(a.size), _ptr(slots, C.c_int32)),
               "Ensure")
        return {int(i): int(s) for i, s in zip(a, slots)}

    def hits(self) -> int:
        return int(lib().nh_slot_cache_hits(self._h))

    def misses(self) -> int:
        return int(lib().nh_slot_cache_misses(self._h))

    def slot_bytes(self, which: int, slot: int, nbytes: int) -> bytes:
        buf = C.create_string_buffer(nbytes)
        _check(lib().nh_slot_cache_read_slot(self._h, which, slot, buf, nbytes), "read_slot")
        return buf.raw

    def __del__(self):
        try:
            if self._h:
                lib().nh_slot_cache_free(self._h)
        except Exception:
            pass
