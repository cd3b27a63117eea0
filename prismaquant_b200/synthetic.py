"""Synthetic workloads with the shapes of the benchmark models (random-init
weights; there is no checkpoint download).

  * llama_dense_linears: Llama-style dense decoder (8B: 32 layers, hidden 4096,
    intermediate 14336, 32 query / 8 KV heads of 128, lm_head 128256 x 4096)
  * moe_expert_params:   packed experts (Qwen3-30B-A3B-like: 48 layers x 128
    experts, gate_up_proj [128, 1536, 2048], down_proj [128, 2048, 768])
  * fused_sibling_group: q/k/v [4096|1024|1024, 4096] + gate/up [14336, 4096]
  * llama_1b_config:     the 1B dense model of the Fisher probe
"""
from __future__ import annotations

import hashlib

import torch


def llama_dense_linears(n_layers=32, hidden=4096, inter=14336, n_heads=32, n_kv=8, head_dim=128,
                        vocab=128256, lm_head=True):
    out = []
    for i in range(n_layers):
        p = f"model.layers.{i}"
        out += [
            (f"{p}.self_attn.q_proj", (n_heads * head_dim, hidden)),
            (f"{p}.self_attn.k_proj", (n_kv * head_dim, hidden)),
            (f"{p}.self_attn.v_proj", (n_kv * head_dim, hidden)),
            (f"{p}.self_attn.o_proj", (hidden, n_heads * head_dim)),
            (f"{p}.mlp.gate_proj", (inter, hidden)),
            (f"{p}.mlp.up_proj", (inter, hidden)),
            (f"{p}.mlp.down_proj", (hidden, inter)),
        ]
    if lm_head:
        out.append(("lm_head", (vocab, hidden)))
    return out


def moe_expert_params(n_layers=48, n_experts=128, hidden=2048, moe_inter=768):
    out = []
    for i in range(n_layers):
        p = f"model.layers.{i}.mlp.experts"
        out += [(f"{p}.gate_up_proj", (n_experts, 2 * moe_inter, hidden)),
                (f"{p}.down_proj", (n_experts, hidden, moe_inter))]
    return out


def fused_sibling_group():
    p = "model.layers.0"
    return [(f"{p}.self_attn.q_proj", (4096, 4096)), (f"{p}.self_attn.k_proj", (1024, 4096)),
            (f"{p}.self_attn.v_proj", (1024, 4096)), (f"{p}.mlp.gate_proj", (14336, 4096)),
            (f"{p}.mlp.up_proj", (14336, 4096))]


def name_seed(name: str, base: int = 0) -> int:
    return (int.from_bytes(hashlib.sha256(name.encode()).digest()[:6], "little") + base) & 0x7FFFFFFFFFFF


def cuda_weights(shapes, device, std=0.02, base_seed=0, dtype=torch.bfloat16):
    """N(0, std^2) bf16 tensors generated on the device, one seed per name."""
    out = {}
    g = torch.Generator(device=device)
    for name, shape in shapes:
        g.manual_seed(name_seed(name, base_seed))
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        out[name] = w.mul_(std).to(dtype)
    return out


def llama_1b_config(vocab=32000, hidden=2048, inter=8192, n_layers=16, n_heads=16, n_kv=16, max_pos=2048):
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=n_layers,
                       num_attention_heads=n_heads, num_key_value_heads=n_kv, max_position_embeddings=max_pos,
                       torch_dtype="bfloat16", tie_word_embeddings=False)
