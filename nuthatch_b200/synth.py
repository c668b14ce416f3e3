"""Seeded synthetic OLMoE-shaped GGUF files (libnh_synth.so).

Named workloads (sizes as stated by the benchmark configurations):
  * ``olmoe_1b7b``: 16 layers, n_embd 2048, 16 heads x 128 (MHA), 64 experts
    top-8, expert FFN 1024, vocab 50304, Q4_K_M-like quantisation (Q4_K,
    attn_v/ffn_down Q6_K on odd layers, output Q6_K), weights ~N(0, 0.02),
    norms 1.0, router F32.
  * ``olmoe_1b7b_skew``: the same plus a log-Zipf(s=1.1) router bias baked
    into the weights (column 0 of every token embedding row is the constant
    0.3, whose normalised value feeds column 0 of the router with gain 0.03),
    for the streaming cache-policy workloads.  Random-init weights already
    route in a strongly token-independent way (without any bias the top
    quarter of experts takes ~95% of a 48-token trace's selections), so the
    bias is kept mild; the bench reports the realised skew.
  * ``granite_moe``: 24 layers, n_embd 1024, 16 query heads x 64, 8 KV heads,
    32 experts top-8, expert FFN 512, vocab 49155.
  * ``mini`` / ``mini_f32``: small shapes for parity tests.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
from dataclasses import asdict, dataclass, replace
from pathlib import Path

from .build import LIB as LIB_DIR, build_synth


class _Spec(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_ff", C.c_uint32), ("n_expert", C.c_uint32),
                ("n_expert_used", C.c_uint32), ("n_vocab", C.c_uint32), ("n_ctx_train", C.c_uint32),
                ("rope_freq_base", C.c_float), ("rms_eps", C.c_float), ("weight_std", C.c_float),
                ("seed", C.c_uint64), ("quant", C.c_int32), ("skew_embd", C.c_float),
                ("skew_router", C.c_float), ("skew_zipf_s", C.c_float), ("n_threads", C.c_int32)]


@dataclass(frozen=True)
class SynthSpec:
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    n_vocab: int
    n_ctx_train: int = 4096
    rope_freq_base: float = 10000.0
    rms_eps: float = 1e-5
    weight_std: float = 0.02
    seed: int = 1
    quant: int = 1
    skew_embd: float = 0.0
    skew_router: float = 0.0
    skew_zipf_s: float = 0.0

    def key(self) -> str:
        return hashlib.sha256(repr(sorted(asdict(self).items())).encode()).hexdigest()[:16]


OLMOE_1B7B = SynthSpec(n_layers=16, n_embd=2048, n_head=16, n_head_kv=16, n_ff=1024, n_expert=64,
                       n_expert_used=8, n_vocab=50304, seed=1)
OLMOE_1B7B_SKEW = replace(OLMOE_1B7B, seed=2, skew_embd=0.3, skew_router=0.03, skew_zipf_s=1.1)
GRANITE_MOE = SynthSpec(n_layers=24, n_embd=1024, n_head=16, n_head_kv=8, n_ff=512, n_expert=32,
                        n_expert_used=8, n_vocab=49155, seed=5)
MINI = SynthSpec(n_layers=2, n_embd=512, n_head=4, n_head_kv=4, n_ff=256, n_expert=16, n_expert_used=4,
                 n_vocab=1000, seed=3)
MINI_GQA = SynthSpec(n_layers=3, n_embd=512, n_head=8, n_head_kv=4, n_ff=512, n_expert=8, n_expert_used=8,
                     n_vocab=777, seed=4)
MINI_F32 = replace(MINI, quant=0, seed=6)

NAMED = {"olmoe_1b7b": OLMOE_1B7B, "olmoe_1b7b_skew": OLMOE_1B7B_SKEW, "granite_moe": GRANITE_MOE,
         "mini": MINI, "mini_gqa": MINI_GQA, "mini_f32": MINI_F32}


def write(spec: SynthSpec, path: str | os.PathLike, threads: int = 0) -> Path:
    build_synth()
    lib = C.CDLL(str(LIB_DIR / "libnh_synth.so"))
    lib.nh_synth_write_olmoe.restype = C.c_int
    lib.nh_synth_write_olmoe.argtypes = [C.c_char_p, C.POINTER(_Spec)]
    s = _Spec(spec.n_layers, spec.n_embd, spec.n_head, spec.n_head_kv, spec.n_ff, spec.n_expert,
              spec.n_expert_used, spec.n_vocab, spec.n_ctx_train, spec.rope_freq_base, spec.rms_eps,
              spec.weight_std, spec.seed, spec.quant, spec.skew_embd, spec.skew_router, spec.skew_zipf_s,
              threads)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    rc = lib.nh_synth_write_olmoe(str(tmp).encode(), C.byref(s))
    if rc != 0:
        raise RuntimeError(f"synthetic GGUF writer failed ({rc}) for {path}")
    os.replace(tmp, path)
    return path


def cached(spec: SynthSpec, cache_dir: str | os.PathLike | None = None) -> Path:
    """Writes the model once per spec into a cache directory and returns its path."""
    d = Path(cache_dir or os.environ.get("NUTHATCH_SYNTH_DIR", "/tmp/nuthatch_synth"))
    path = d / f"olmoe_{spec.key()}.gguf"
    if not path.exists():
        write(spec, path)
    return path
