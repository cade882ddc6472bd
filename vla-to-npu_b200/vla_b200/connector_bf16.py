"""Drop-in for vla/connector_bf16.py: pixel shuffle (scale 4) + linear without bias.

``connector_block(x, params) -> out`` (reference :136-139): x [1024, 768]
(a 32x32 token grid), params["W"] [12288, 960] ([in, out]); out [64, 960].
The reference's per-row copy regions and 192 K=64 GEMM slices summed in bf16
(:97-133) become one pixel-shuffle kernel and one GEMM with fp32 accumulation.
"""
from __future__ import annotations

import math

import torch

from . import device as dev
from ._host import to_device, to_host_like, weight_kmajor

BF16 = torch.bfloat16


def connector_block(x_np, params, *, scale: int = 4):
    x = to_device(x_np)
    tokens, C = x.shape[-2], x.shape[-1]
    grid = int(math.isqrt(tokens))
    x = x.reshape(-1, C)
    B = x.shape[0] // tokens
    w = weight_kmajor(params["W"])
    shuffled = torch.empty(B * (grid // scale) ** 2, scale * scale * C, dtype=BF16, device=x.device)
    dev.pixel_shuffle(x, B, grid, scale, shuffled)
    out = torch.empty(shuffled.shape[0], w.shape[0], dtype=BF16, device=x.device)
    dev.gemm(shuffled, w, out)
    return to_host_like(out.reshape(*x_np.shape[:-2], -1, w.shape[0]) if B > 1 else out, x_np)
