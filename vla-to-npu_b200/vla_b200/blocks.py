"""Shared machinery of the reference-named block builders: turn a reference
``params`` dict into a libvla_b200 layer struct (weights uploaded once and
cached), and run one block on one sequence."""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import _lib
from . import device as dev
from ._host import WEIGHTS, to_device, vector, weight_kmajor
from .model import interleave_gate_up, rope_table

BF16 = torch.bfloat16
_WS = {}


def workspace() -> dev.Workspace:
    d = torch.cuda.current_device()
    if d not in _WS:
        _WS[d] = dev.Workspace(torch.device("cuda", d))
    return _WS[d]


def llama_layer(params: Dict, eps: float, cross: bool = False) -> Tuple[_lib.LlamaLayer, list]:
    """Layer struct for a text/expert block from reference params ([in, out] weights)."""
    hidden = params["Wq"].shape[0]
    q_dim = params["Wq"].shape[1]
    if cross:
        w_qkv = weight_kmajor(params["Wq"])
        kv_dim = params["Wk_cross"].shape[1]
    else:
        kv_dim = params["Wk"].shape[1]
        w_qkv = WEIGHTS.get((params["Wq"], params["Wk"], params["Wv"]), "qkv_self", lambda: torch.cat(
            [to_device(params["Wq"]), to_device(params["Wk"]), to_device(params["Wv"])], dim=1).t().contiguous())
    w_o = weight_kmajor(params["Wo"])
    w_gu = WEIGHTS.get((params["W_gate"], params["W_up"]), "gate_up", lambda: interleave_gate_up(
        to_device(params["W_gate"]), to_device(params["W_up"]), "cuda"))
    w_down = weight_kmajor(params["W_down"])
    n1, n2 = vector(params["W_norm_1"]), vector(params["W_norm_2"])
    s = _lib.LlamaLayer()
    s.norm1, s.w_qkv, s.w_o, s.norm2, s.w_gu, s.w_down = (t.data_ptr() for t in (n1, w_qkv, w_o, n2, w_gu, w_down))
    s.hidden, s.heads, s.kv_heads, s.head_dim = hidden, q_dim // 64, kv_dim // 64, 64
    s.ffn = params["W_gate"].shape[1]
    s.eps = eps
    return s, [n1, w_qkv, w_o, n2, w_gu, w_down]


def rope_cs(seq: int, theta: float) -> torch.Tensor:
    return WEIGHTS.get(rope_table, f"rope:{seq}:{theta}", lambda: rope_table(seq, 64, theta).cuda())


def vision_layer(params: Dict, eps: float) -> Tuple[_lib.VisionLayer, list]:
    H = params["Wq"].shape[0]
    F = params["W_up"].shape[1]
    zeros_h = WEIGHTS.get(torch, f"zeros:{H}", lambda: torch.zeros(H, dtype=BF16, device="cuda"))
    zeros_f = WEIGHTS.get(torch, f"zeros:{F}", lambda: torch.zeros(F, dtype=BF16, device="cuda"))
    w_qkv = WEIGHTS.get((params["Wq"], params["Wk"], params["Wv"]), "qkv_vision", lambda: torch.cat(
        [to_device(params["Wq"]), to_device(params["Wk"]), to_device(params["Wv"])], dim=1).t().contiguous())

    def bias(key, z):
        return vector(params[key]) if key in params else z

    bsrc = tuple(params[k] for k in ("bq", "bk", "bv") if k in params)
    b_tag = f"bqkv_vision:{H}:" + ",".join(k for k in ("bq", "bk", "bv") if k in params)
    b_qkv = WEIGHTS.get(bsrc + (torch,), b_tag, lambda: torch.cat(
        [bias("bq", zeros_h), bias("bk", zeros_h), bias("bv", zeros_h)]).contiguous())
    keep = [w_qkv, b_qkv, weight_kmajor(params["Wo"]), bias("bo", zeros_h), weight_kmajor(params["W_up"]),
            bias("b_up", zeros_f), weight_kmajor(params["W_down"]), bias("b_down", zeros_h),
            vector(params["W_norm_1"]), vector(params["b_norm_1"]), vector(params["W_norm_2"]),
            vector(params["b_norm_2"])]
    s = _lib.VisionLayer()
    s.w_qkv, s.b_qkv, s.w_o, s.b_o, s.w_fc1, s.b_fc1, s.w_fc2, s.b_fc2 = (t.data_ptr() for t in keep[:8])
    s.ln1_g, s.ln1_b, s.ln2_g, s.ln2_b = (t.data_ptr() for t in keep[8:])
    s.hidden, s.heads, s.head_dim, s.ffn, s.eps = H, H // 64, 64, F, eps
    return s, keep
