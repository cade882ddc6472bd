"""Drop-in for vla/preprocessing_bf16.py: the SigLIP patch embedding.

``preprocessing_block(img, params) -> out`` (reference :105-109): img
[3, 512, 512] (float), params["kernel"] conv weight [768, 3, 16, 16]; out
[1024, 768] bf16.  The reference's 14,592 per-channel 16x16 conv calls
(:86-103) become an im2col kernel and one GEMM.  Optional params
"b_patch" [768] and "pos_emb" [1024, 768] add the conv bias and learned
position embedding of SiglipVisionEmbeddings (vla/vit_emb.py:43-47).
"""
from __future__ import annotations

import torch

from . import device as dev
from ._host import WEIGHTS, to_device, to_host_like, vector

BF16 = torch.bfloat16


def preprocessing_block(x_fp32, params):
    img = to_device(x_fp32)
    if img.dim() == 3:
        img = img.unsqueeze(0)
    B, C, H, W = img.shape
    ker = params["kernel"]
    D, p = ker.shape[0], ker.shape[-1]
    w = WEIGHTS.get(ker, "patch", lambda: to_device(ker).reshape(D, -1).contiguous())
    tokens = (H // p) * (W // p)
    patches = torch.empty(B * tokens, C * p * p, dtype=BF16, device=img.device)
    dev.patch_im2col(img.contiguous(), p, patches)
    out = torch.empty(B * tokens, D, dtype=BF16, device=img.device)
    bias = vector(params["b_patch"]) if "b_patch" in params else None
    pos = vector(params["pos_emb"]) if "pos_emb" in params else None
    dev.gemm(patches, w, out, dev.make_epilogue(bias=bias, residual=pos, res_row_mod=tokens if pos is not None else 0))
    res = out if B > 1 else out.reshape(tokens, D)
    return to_host_like(res, x_fp32)
