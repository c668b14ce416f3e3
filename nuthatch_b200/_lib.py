"""ctypes bindings of libnuthatch_b200.so (include/nh_api.h, include/nh_kernels.h).

The library is built in-tree by ``python -m nuthatch_b200.build``.  A missing
library is an error: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_PATH = LIB_DIR / "libnuthatch_b200.so"
# The phase-timestamp diagnostic build of the same library, loaded instead
# when NH_PHASE_TRACE_LIB=1 at the first lib() call (nuthatch_b200.phase_trace).
PHASE_TRACE_LIB_PATH = LIB_DIR / "libnuthatch_b200_phase_trace.so"

i32, i64, u32, u64, f32 = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_float
vp, cp = C.c_void_p, C.c_char_p
P = C.POINTER


class NhConfig(C.Structure):
    _fields_ = [("n_layers", u32), ("n_embd", u32), ("n_head", u32), ("n_head_kv", u32), ("n_ff", u32),
                ("n_expert", u32), ("n_expert_used", u32), ("n_vocab", u32), ("n_ctx_train", u32),
                ("rope_freq_base", f32), ("rms_eps", f32)]


class NhDecodeState(C.Structure):
    _fields_ = [("pos", i32), ("n_prompt", i32), ("n_predict", i32), ("n_out", i32), ("token", i32),
                ("error", i32), ("pad0", i32), ("pad1", i32)]


class NhMoeLayer(C.Structure):
    _fields_ = [("state", vp), ("h", vp), ("ffn_norm", vp), ("eps", f32), ("router", vp), ("n_embd", i64),
                ("n_ff", i64), ("n_expert", C.c_int), ("k", C.c_int), ("norm_topk", C.c_int), ("layer", C.c_int),
                ("n_layers", C.c_int), ("gate", vp), ("tg", i32), ("gate_nb2", u64), ("up", vp), ("tu", i32),
                ("up_nb2", u64), ("down", vp), ("td", i32), ("down_nb2", u64), ("sel", vp), ("wts", vp),
                ("trace_sel", vp), ("trace_gap", vp), ("ff", vp), ("dump", vp), ("dump_step_stride", i64),
                ("dump_offset", i64), ("scratch", vp)]


# name -> (restype, argtypes)
SIGNATURES = {
    # nh_api.h
    "nh_version": (cp, []),
    "nh_set_device": (C.c_int, [C.c_int]),
    "nh_last_error": (cp, []),
    "nh_gguf_probe": (C.c_int, [cp, P(NhConfig)]),
    "nh_model_load": (vp, [cp]),
    "nh_model_free": (None, [vp]),
    "nh_model_config": (C.c_int, [vp, P(NhConfig)]),
    "nh_model_tensor": (C.c_int, [vp, cp, P(i64), P(i32), P(vp), P(u64)]),
    "nh_generate": (C.c_int, [vp, C.c_int, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, P(i32), P(i32), P(f32),
                              P(f32), P(f32)]),
    "nh_generate_launches": (C.c_int, [vp]),
    "nh_generate_batch": (C.c_int, [vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(i32),
                                    P(C.c_double)]),
    "nh_generate_timed": (C.c_int, [vp, P(i32), C.c_int, C.c_int, C.c_int, P(i32), P(C.c_double),
                                    P(C.c_double)]),
    "nh_generate_batch_timed": (C.c_int, [vp, vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(i32),
                                          P(C.c_double), P(C.c_double)]),
    "nh_ep_new_id": (C.c_int, [vp]),
    "nh_ep_create": (vp, [vp, C.c_int, C.c_int]),
    "nh_ep_free": (None, [vp]),
    "nh_model_load_expert_shard": (vp, [cp, C.c_uint32, C.c_uint32]),
    "nh_generate_batch_ep": (C.c_int, [vp, vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(i32),
                                       P(C.c_double)]),
    "nh_batch_q8_bytes": (i64, [i64, i64]),
    "nh_batch_attention_scratch_bytes": (i64, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "nh_decode_prepare": (C.c_int, [vp, P(i32), C.c_int, C.c_int]),
    "nh_decode_run": (C.c_int, [vp, C.c_int]),
    "nh_decode_result": (C.c_int, [vp, C.c_int, P(i32)]),
    "nh_model_stream": (vp, [vp]),
    "nh_decode_kernel_loop": (C.c_int, [vp, C.c_int, C.c_int]),
    "nh_stream_model_load": (vp, [cp, C.c_int]),
    "nh_stream_model_free": (None, [vp]),
    "nh_stream_model_config": (C.c_int, [vp, P(NhConfig)]),
    "nh_stream_generate": (C.c_int, [vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(u64),
                                     P(i32), P(i64), P(i64), P(u64), P(i32)]),
    "nh_stream_generate_batch": (C.c_int, [vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_int, P(u64), P(i32), P(i64), P(i64), P(u64), P(i64),
                                           P(C.c_double)]),
    "nh_stream_generate_batch_ep": (C.c_int, [vp, vp, P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_int, P(u64), P(i32), P(i64), P(i64), P(u64), P(i64),
                                              P(C.c_double)]),
    "nh_plan_waves": (C.c_int, [P(i32), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(C.c_uint8), P(i32), P(i32),
                                P(i32)]),
    "nh_group_wave_pairs": (C.c_int, [P(i32), C.c_int, C.c_int, C.c_int, P(i32), C.c_int, P(i32), C.c_int, P(i32),
                                      P(i32), P(i32), P(i32)]),
    "nh_tokenizer_load": (vp, [cp]),
    "nh_tokenizer_from_lists": (vp, [P(C.c_char_p), i64, P(C.c_char_p), i64]),
    "nh_tokenizer_free": (None, [vp]),
    "nh_tokenizer_vocab_size": (i64, [vp]),
    "nh_tokenizer_encode": (i64, [vp, C.c_char_p, i64, P(i32), i64]),
    "nh_tokenizer_decode": (i64, [vp, P(i32), i64, C.c_char_p, i64]),
    "nh_tokenizer_token": (i64, [vp, C.c_int32, C.c_char_p, i64]),
    "nh_tokenizer_split": (i64, [C.c_char_p, i64, P(i64), i64]),
    "nh_replay": (i64, [C.c_int, u32, u32, i64, P(u32), P(i64), P(u32), u32, u32, P(u64), P(i64)]),
    "nh_sweep_budgets": (C.c_int, [u32, u32, i64, P(u32), P(i64), P(u32), P(u32), C.c_int, P(C.c_double)]),
    "nh_sweep_pin_ratio": (C.c_int, [u32, u32, i64, P(u32), P(i64), P(u32), u32, P(C.c_double)]),
    "nh_sweep_budgets_calibrated": (C.c_int, [u32, u32, i64, P(u32), P(i64), P(u32), i64, P(u32), P(i64), P(u32),
                                              P(u32), C.c_int, P(C.c_double)]),
    "nh_trace_write": (C.c_int, [cp, u32, u32, i64, P(u32), P(u32), P(i64), P(u32)]),
    "nh_trace_read": (i64, [cp, C.c_int, P(u32), P(u32), P(i64), i64, i64, P(u32), P(u32), P(i64), P(u32)]),
    "nh_expert_reader_open": (vp, [cp]),
    "nh_expert_reader_free": (None, [vp]),
    "nh_expert_reader_bytes": (u64, [vp, cp]),
    "nh_expert_reader_read": (C.c_int, [vp, cp, C.c_int, vp]),
    "nh_expert_reader_fail_after": (C.c_int, [vp, i64]),
    "nh_slot_cache_create": (vp, [P(NhConfig), C.c_int, C.c_int, vp, C.c_int, C.c_int, P(u64)]),
    "nh_slot_cache_free": (None, [vp]),
    "nh_slot_cache_ensure": (C.c_int, [vp, P(i32), C.c_int, P(i32)]),
    "nh_slot_cache_hits": (i64, [vp]),
    "nh_slot_cache_misses": (i64, [vp]),
    "nh_slot_cache_read_slot": (C.c_int, [vp, C.c_int, C.c_int, vp, u64]),
    # nh_kernels.h
    "nh_device_sm_count": (C.c_int, [C.c_int]),
    "nh_attention_scratch_bytes": (i64, [C.c_int, C.c_int, C.c_int]),
    "nh_argmax_scratch_bytes": (i64, [C.c_int]),
    "nh_router_scratch_bytes": (i64, [C.c_int]),
    "nh_rope_table": (None, [f32, C.c_int, C.c_int, P(f32)]),
    "nh_publish_selection": (C.c_int, [vp, C.c_int, vp, vp, u32, vp]),
    "nh_embed_step": (C.c_int, [vp, vp, vp, i32, i64, i64, vp, vp]),
    "nh_qkv_proj": (C.c_int, [vp, vp, vp, f32, vp, i32, vp, i32, vp, i32, i64, i64, vp, vp, vp, vp]),
    "nh_attention_step": (C.c_int, [vp, vp, vp, vp, vp, vp, f32, C.c_int, C.c_int, C.c_int, vp, f32, vp, vp,
                                    C.c_int, vp, vp, vp]),
    "nh_attention_step_static": (C.c_int, [vp, vp, vp, vp, vp, vp, f32, C.c_int, C.c_int, C.c_int, vp, f32, vp,
                                           vp, C.c_int, vp, vp]),
    "nh_out_proj_residual": (C.c_int, [vp, vp, vp, i32, i64, vp, vp]),
    "nh_router_topk": (C.c_int, [vp, vp, vp, f32, vp, i64, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, C.c_int,
                                 C.c_int, vp, vp]),
    "nh_moe_gate_up": (C.c_int, [vp, vp, vp, f32, vp, C.c_int, vp, i32, u64, vp, i32, u64, i64, i64, vp, vp]),
    "nh_moe_gate_up_prefetch": (C.c_int, [vp, vp, vp, f32, vp, C.c_int, vp, i32, u64, vp, i32, u64, i64, i64, vp,
                                          vp, u64, vp]),
    "nh_moe_down_combine": (C.c_int, [vp, vp, vp, vp, C.c_int, vp, i32, u64, i64, i64, vp, vp, i64, i64, vp]),
    "nh_moe_gate_up_slots": (C.c_int, [vp, vp, vp, f32, vp, C.c_int, vp, i32, u64, vp, i32, u64, i64, i64, vp,
                                       vp, u64, vp]),
    "nh_moe_down_combine_slots": (C.c_int, [vp, vp, vp, vp, C.c_int, vp, i32, u64, i64, i64, vp, vp, i64, i64,
                                            vp]),
    "nh_moe_layer": (C.c_int, [P(NhMoeLayer), vp]),
    "nh_moe_layer_scratch_bytes": (i64, [C.c_int]),
    "nh_lm_head_argmax": (C.c_int, [vp, vp, vp, f32, vp, i32, i64, i64, vp, vp, vp, vp]),
    "nh_prefill_embed": (C.c_int, [vp, C.c_int, vp, i32, i64, i64, vp, vp, vp]),
    "nh_prefill_qk": (C.c_int, [vp, vp, vp, vp, vp, f32, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp,
                                C.c_int, vp, vp]),
    "nh_prefill_attention": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, vp, C.c_int, vp,
                                       vp]),
    "nh_prefill_embed_seqs": (C.c_int, [vp, i64, C.c_int, C.c_int, vp, i32, i64, i64, vp, vp, vp]),
    "nh_prefill_qk_seqs": (C.c_int, [vp, vp, vp, vp, vp, f32, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     vp, vp, vp, C.c_int, vp, vp]),
    "nh_prefill_attention_seqs": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, vp,
                                            C.c_int, vp, vp]),
    "nh_batch_router_trace": (C.c_int, [vp, vp, C.c_int, i64, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, C.c_int,
                                        C.c_int, C.c_int, vp]),
    "nh_gemv": (C.c_int, [vp, vp, i32, i64, i64, vp, vp, f32, vp, vp]),
    "nh_quantize_q8k": (C.c_int, [vp, i64, vp, vp]),
    "nh_dequantize": (C.c_int, [vp, i32, i64, i64, vp, vp]),
    "nh_exp_cw": (C.c_int, [vp, i64, vp, vp]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the native library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        path = PHASE_TRACE_LIB_PATH if os.environ.get("NH_PHASE_TRACE_LIB") == "1" else LIB_PATH
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run `python -m nuthatch_b200.build` "
                               "(there is no non-native implementation)")
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)
