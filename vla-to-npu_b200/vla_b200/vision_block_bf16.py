"""Drop-in for vla/vision_block_bf16.py: one SigLIP encoder layer on the GPU.

``vision_block(x, params) -> out`` keeps the reference signature
(vla/vision_block_bf16.py:308-420): x [SEQ, EMBD]; params Wq/Wk/Wv/Wo/W_up/W_down
([in, out]), W_norm_1/b_norm_1/W_norm_2/b_norm_2, plus optional biases
bq/bk/bv/bo/b_up/b_down of the real SigLIP layer (vla/vision_block.py:13-25;
absent = zero, as in the reference's MiniVit).  The MLP activation is
GELU-tanh and LayerNorm eps defaults to 1e-6 (benchmark configuration C1;
the reference's bf16 oracle MiniVit uses erf-GELU and eps 1e-5).
"""
from __future__ import annotations

from . import device as dev
from ._host import to_device, to_host_like
from .blocks import vision_layer, workspace


def vision_block(x_np, params, *, eps: float = 1e-6):
    s, keep = vision_layer(params, eps)
    x = to_device(x_np).reshape(-1, s.hidden).clone()
    dev.vision_layer(s, x, 1, x.shape[0], workspace())
    return to_host_like(x, x_np)
