"""Drop-in for vla/action_expert_bf16.py: the SmolVLA action-expert layers.

* ``action_expert_self_forward(x, params) -> out`` (reference :662-728): causal
  self-attention layer; params Wq/Wk/Wv/Wo/W_gate/W_up/W_down/W_norm_1/W_norm_2.
* ``action_expert_cross_forward(x, text_k, text_v, params) -> out``
  (reference :731-803): K/V = text_k . Wk_cross, text_v . Wv_cross, RoPE on Q
  only, no causal mask (optional key padding ``kv_len``).
Defaults: RoPE base 1e4 (reference :95), RMSNorm eps 1e-5.
"""
from __future__ import annotations

import torch

from . import device as dev
from ._host import to_device, to_host_like, weight_kmajor
from .blocks import llama_layer, rope_cs, workspace

BF16 = torch.bfloat16


def action_expert_self_forward(x_np, params, *, rope_theta: float = 10_000.0, eps: float = 1e-5):
    s, keep = llama_layer(params, eps)
    x = to_device(x_np).reshape(-1, s.hidden).clone()
    seq = x.shape[0]
    dev.llama_self_layer(s, x, 1, seq, rope_cs(seq, rope_theta), workspace())
    return to_host_like(x, x_np)


def action_expert_cross_forward(x_np, text_k_np, text_v_np, params, *, rope_theta: float = 10_000.0,
                                eps: float = 1e-5, kv_len=None):
    s, keep = llama_layer(params, eps, cross=True)
    x = to_device(x_np).reshape(-1, s.hidden).clone()
    seq = x.shape[0]
    tk, tv = to_device(text_k_np), to_device(text_v_np)
    tk, tv = tk.reshape(-1, tk.shape[-1]), tv.reshape(-1, tv.shape[-1])
    kv_dim = s.kv_heads * 64
    kv = torch.empty(tk.shape[0], 2 * kv_dim, dtype=BF16, device=x.device)
    dev.gemm(tk, weight_kmajor(params["Wk_cross"]), kv[:, :kv_dim])
    dev.gemm(tv, weight_kmajor(params["Wv_cross"]), kv[:, kv_dim:])
    kl = None if kv_len is None else torch.tensor([int(kv_len)], dtype=torch.int32, device=x.device)
    dev.llama_cross_layer(s, x, 1, seq, rope_cs(seq, rope_theta), kv[:, :kv_dim], kv[:, kv_dim:], tk.shape[0],
                          workspace(), kv_len=kl)
    return to_host_like(x, x_np)
