"""A small synthetic Qwen2-layout GGUF model for the GGUF tests: seeded random
ggml blocks (Q4_K_M style: Q6_K for attn_v, ffn_down and the output head,
Q4_K for the other linears), fp32 norm weights, the metadata keys the
runner reads.  No real model file exists on this machine."""
from __future__ import annotations

import numpy as np

from vkflame_b200 import gguf
from vkflame_b200 import synth as S


def make(path, layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1280, vocab=2048, seed=0, d_range=None):
    """d_range: the fp16 block scales' range (default: the synthetic
    generator's U[1e-3, 1e-2]; the GPU test picks small ones so that a chain
    of linears stays finite in fp16)."""
    meta = {"general.architecture": "qwen2", "general.name": "synthetic-test", "qwen2.block_count": layers,
            "qwen2.embedding_length": hidden, "qwen2.feed_forward_length": ffn,
            "qwen2.attention.head_count": heads, "qwen2.attention.head_count_kv": kv_heads,
            "qwen2.rope.freq_base": 1000000.0, "qwen2.attention.layer_norm_rms_epsilon": 1e-6,
            "tokenizer.ggml.tokens": ["<a>", "<b>"]}
    tensors = []
    s = seed

    def q(name, fmt, K, N):
        nonlocal s
        s += 1
        tensors.append((name, (K, N), gguf.VKF_TO_GGML[fmt], S.quant_matrix(fmt, N, K, seed=s, d_range=d_range)))

    rng = np.random.default_rng(seed)
    tensors.append(("token_embd.weight", (hidden, vocab), gguf.GGML_F16,
                    rng.standard_normal((vocab, hidden)).astype(np.float16)))
    for i in range(layers):
        b = f"blk.{i}."
        tensors.append((b + "attn_norm.weight", (hidden,), gguf.GGML_F32, np.ones(hidden, np.float32)))
        q(b + "attn_q.weight", S.Q4_K, hidden, heads * head_dim)
        q(b + "attn_k.weight", S.Q4_K, hidden, kv_heads * head_dim)
        q(b + "attn_v.weight", S.Q6_K, hidden, kv_heads * head_dim)
        q(b + "attn_output.weight", S.Q4_K, heads * head_dim, hidden)
        tensors.append((b + "ffn_norm.weight", (hidden,), gguf.GGML_F32, np.ones(hidden, np.float32)))
        q(b + "ffn_gate.weight", S.Q4_K, hidden, ffn)
        q(b + "ffn_up.weight", S.Q4_K, hidden, ffn)
        q(b + "ffn_down.weight", S.Q6_K, ffn, hidden)
    tensors.append(("output_norm.weight", (hidden,), gguf.GGML_F32, np.ones(hidden, np.float32)))
    q("output.weight", S.Q6_K, hidden, vocab)
    gguf.write(path, meta, tensors)
    return tensors
