"""Drop-in for vla/text_encoder_bf16.py: one SmolVLA text-encoder (Llama-style)
layer on the GPU.

``text_encoder_forward(x, params) -> (out, key, value)`` keeps the reference
signature (vla/text_encoder_bf16.py:480-595): x [SEQ, EMBD], params with
Wq/Wk/Wv/Wo/W_gate/W_up/W_down ([in, out]) and W_norm_1/W_norm_2; key is this
layer's post-RoPE K and value its V, [SEQ, KV_H*64] (as the Allo path returns
them, :494-500).  Defaults are benchmark configuration C0 (RoPE base 1e5,
RMSNorm eps 1e-5); the reference module's RoPE base is 1e4 (:79).
"""
from __future__ import annotations

import torch

from . import device as dev
from ._host import to_device, to_host_like
from .blocks import llama_layer, rope_cs, workspace

BF16 = torch.bfloat16


def text_encoder_forward(x_np, params, *, rope_theta: float = 100_000.0, eps: float = 1e-5):
    s, keep = llama_layer(params, eps)
    x = to_device(x_np).reshape(-1, s.hidden).clone()
    seq = x.shape[0]
    q, kv = s.heads * 64, s.kv_heads * 64
    qkv = torch.empty(seq, q + 2 * kv, dtype=BF16, device=x.device)
    dev.llama_self_layer(s, x, 1, seq, rope_cs(seq, rope_theta), workspace(), qkv_out=qkv)
    return (to_host_like(x, x_np), to_host_like(qkv[:, q:q + kv], x_np), to_host_like(qkv[:, q + kv:], x_np))
