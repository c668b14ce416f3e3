"""The reference tests' model fixture, regenerated here.

The reference writes a tiny all-F32 OLMoE GGUF at test time (dims n_embd 8,
n_head 2, n_ff 4, n_expert 4, n_used 2, n_vocab 16, n_layers 2), filling
every tensor from one running LCG, seed 7:
    seed = seed*1103515245 + 12345   (32-bit signed wrap)
    value = 0.02f * ((seed >> 16) % 100 - 50)   (C truncating %)
(generate_test.cc:19-73, forward_test.cc:18-87, streaming_forward_test.cc:17-68).
This module reproduces that fixture byte for byte in content with gguf-py's
writer (an independent GGUF implementation), so the product's parser and the
oracle are both exercised on a third-party-written file.
"""
from __future__ import annotations

import numpy as np
from gguf import GGUFWriter


class _Lcg:
    def __init__(self, seed: int = 7):
        self.seed = seed

    def next(self) -> np.float32:
        s = (self.seed * 1103515245 + 12345) & 0xFFFFFFFF
        if s >= 1 << 31:
            s -= 1 << 32
        self.seed = s
        q = s >> 16  # arithmetic shift of a signed int
        r = q - 100 * int(q / 100)  # C remainder truncates toward zero
        return np.float32(0.02) * np.float32(r - 50)


def write_tiny_olmoe(path, n_embd=8, n_head=2, n_ff=4, n_expert=4, n_used=2, n_vocab=16, n_layers=2,
                     n_ctx=32) -> str:
    w = GGUFWriter(str(path), "olmoe")
    w.add_uint32("olmoe.block_count", n_layers)
    w.add_uint32("olmoe.embedding_length", n_embd)
    w.add_uint32("olmoe.attention.head_count", n_head)
    w.add_uint32("olmoe.attention.head_count_kv", n_head)
    w.add_uint32("olmoe.feed_forward_length", n_ff)
    w.add_uint32("olmoe.expert_count", n_expert)
    w.add_uint32("olmoe.expert_used_count", n_used)
    w.add_uint32("olmoe.context_length", n_ctx)
    w.add_float32("olmoe.rope.freq_base", 10000.0)
    w.add_float32("olmoe.attention.layer_norm_rms_epsilon", 1e-5)
    lcg = _Lcg(7)

    def add(name, a, b=0, c=0):
        ne = [a] + ([b] if b else []) + ([c] if c else [])
        n = int(np.prod(ne))
        vals = np.array([lcg.next() for _ in range(n)], dtype=np.float32)
        w.add_tensor(name, vals.reshape(list(reversed(ne))))

    add("token_embd.weight", n_embd, n_vocab)
    add("output.weight", n_embd, n_vocab)
    add("output_norm.weight", n_embd)
    for l in range(n_layers):
        b = f"blk.{l}."
        add(b + "attn_norm.weight", n_embd)
        add(b + "attn_q.weight", n_embd, n_embd)
        add(b + "attn_k.weight", n_embd, n_embd)
        add(b + "attn_v.weight", n_embd, n_embd)
        add(b + "attn_output.weight", n_embd, n_embd)
        add(b + "attn_q_norm.weight", n_embd)
        add(b + "attn_k_norm.weight", n_embd)
        add(b + "ffn_norm.weight", n_embd)
        add(b + "ffn_gate_inp.weight", n_embd, n_expert)
        add(b + "ffn_gate_exps.weight", n_embd, n_ff, n_expert)
        add(b + "ffn_up_exps.weight", n_embd, n_ff, n_expert)
        add(b + "ffn_down_exps.weight", n_ff, n_embd, n_expert)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return str(path)


def write_slot_fixture(path, n_embd=8, n_ff=4, n_expert=5) -> str:
    """expert_slot_cache_test.cc:20-41: one layer of F32 expert tensors,
    value base + 0.25*i (gate base 1, up 100, down 500)."""
    w = GGUFWriter(str(path), "olmoe")

    def add(name, a, b, base):
        n = a * b * n_expert
        vals = (np.float32(base) + np.float32(0.25) * np.arange(n, dtype=np.float32)).astype(np.float32)
        w.add_tensor(name, vals.reshape(n_expert, b, a))

    add("blk.0.ffn_gate_exps.weight", n_embd, n_ff, 1.0)
    add("blk.0.ffn_up_exps.weight", n_embd, n_ff, 100.0)
    add("blk.0.ffn_down_exps.weight", n_ff, n_embd, 500.0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return str(path)
