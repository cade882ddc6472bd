"""Drop-in for vla/llama_block_rope_bf16.py (the 768-wide Llama block with RoPE).

* ``llama_block_rope(x, params) -> (out, key, value)`` (reference :519-615):
  one causal self-attention layer; key is post-RoPE K.
* ``llama_block_rope_cross(key, value, x, params) -> out`` (reference :617-709):
  Q from x with RoPE, the given key rotated by RoPE as well, the given value,
  causal masked softmax as the reference's Allo path applies it (:641-652),
  then the output projection and SwiGLU MLP with residuals.
Defaults follow the reference module constants (RoPE base 1e4, eps 1e-5).
"""
from __future__ import annotations

import torch

from . import _lib
from . import device as dev
from ._host import WEIGHTS, to_device, to_host_like, vector, weight_kmajor
from .blocks import llama_layer, rope_cs, workspace
from .model import interleave_gate_up

BF16 = torch.bfloat16


def llama_block_rope(x_np, params, *, rope_theta: float = 10_000.0, eps: float = 1e-5):
    s, keep = llama_layer(params, eps)
    x = to_device(x_np).reshape(-1, s.hidden).clone()
    seq = x.shape[0]
    q, kv = s.heads * 64, s.kv_heads * 64
    qkv = torch.empty(seq, q + 2 * kv, dtype=BF16, device=x.device)
    dev.llama_self_layer(s, x, 1, seq, rope_cs(seq, rope_theta), workspace(), qkv_out=qkv)
    return (to_host_like(x, x_np), to_host_like(qkv[:, q:q + kv], x_np), to_host_like(qkv[:, q + kv:], x_np))


def llama_block_rope_cross(key, value, x_np, params, *, rope_theta: float = 10_000.0, eps: float = 1e-5):
    H = params["Wq"].shape[0]
    x = to_device(x_np).reshape(-1, H).clone()
    seq = x.shape[0]
    k = to_device(key).clone()
    v = to_device(value)
    cs = rope_cs(max(seq, k.shape[0]), rope_theta)
    q_dim, kv_dim, F = params["Wq"].shape[1], k.shape[1], params["W_gate"].shape[1]
    h = dev.rms_norm(x, vector(params["W_norm_1"]), eps)
    qb = torch.empty(seq, q_dim, dtype=BF16, device=x.device)
    dev.gemm(h, weight_kmajor(params["Wq"]), qb,
             dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=seq, rope_ncols=q_dim))
    dev.rope_(k, kv_dim, k.shape[0], cs)
    att = torch.empty(seq, q_dim, dtype=BF16, device=x.device)
    dev.attention(qb, k, v, att, batch=1, Lq=seq, Lk=k.shape[0], Hq=q_dim // 64, Hkv=kv_dim // 64,
                  q_batch=0, k_batch=0, v_batch=0, o_batch=0, causal=True)
    dev.gemm(att, weight_kmajor(params["Wo"]), x, dev.make_epilogue(residual=x))
    # MLP half: x += down(silu(gate(rms(x))) * up(rms(x)))
    h = dev.rms_norm(x, vector(params["W_norm_2"]), eps)
    mid = torch.empty(seq, F, dtype=BF16, device=x.device)
    w_gu = WEIGHTS.get((params["W_gate"], params["W_up"]), "gate_up", lambda: interleave_gate_up(
        to_device(params["W_gate"]), to_device(params["W_up"]), "cuda"))
    dev.gemm(h, w_gu, mid, dev.make_epilogue(act=_lib.ACT_SWIGLU))
    dev.gemm(mid, weight_kmajor(params["W_down"]), x, dev.make_epilogue(residual=x))
    return to_host_like(x, x_np)
