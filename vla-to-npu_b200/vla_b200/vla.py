"""Drop-in for vla/vla.py: the pipeline-level entry points.

* ``vision_encoder(num_layers, x, params)``      reference :185-188
* ``joint_transformer(num_layers, vlm_input, action, vlm_params,
  exp_self_params, exp_cross_params)``           reference :194-212 — layer i
  runs the text layer, then the expert self layer (i even) or the cross
  layer on that text layer's K/V (i odd)
* ``postprocessing(out, out_params)``            reference :218-222 — RMSNorm
  (W_exp_norm) then the out projection (W_action_out)
* ``SmolVLA``                                    the full action-chunk model
  (vision tower, connector, prefix, 16 text layers, 10-step flow-matching
  action expert) as one CUDA graph; see vla_b200.model
"""
from __future__ import annotations

import torch

from . import device as dev
from ._host import to_device, to_host_like, vector, weight_kmajor
from .action_expert_bf16 import action_expert_cross_forward, action_expert_self_forward
from .model import SmolVLA  # noqa: F401
from .text_encoder_bf16 import text_encoder_forward
from .vision_block_bf16 import vision_block

BF16 = torch.bfloat16
SKIP = 2  # cross-attention every SKIP layers (reference :79)


def vision_encoder(num_layers, x, params, *, eps: float = 1e-6):
    for _ in range(num_layers):
        x = vision_block(x, params, eps=eps)
    return x


def joint_transformer(num_layers, vlm_input, action, vlm_params, exp_self_params, exp_cross_params, *,
                      text_rope_theta: float = 100_000.0, expert_rope_theta: float = 10_000.0, eps: float = 1e-5):
    for i in range(num_layers):
        vlm_output, text_k, text_v = text_encoder_forward(vlm_input, vlm_params, rope_theta=text_rope_theta, eps=eps)
        vlm_input = vlm_output
        if i % SKIP == 0:
            action = action_expert_self_forward(action, exp_self_params, rope_theta=expert_rope_theta, eps=eps)
        else:
            action = action_expert_cross_forward(action, text_k, text_v, exp_cross_params,
                                                 rope_theta=expert_rope_theta, eps=eps)
    return action


def postprocessing(out, out_params, *, eps: float = 1e-5):
    x = to_device(out)
    x = x.reshape(-1, x.shape[-1])
    h = dev.rms_norm(x, vector(out_params["W_exp_norm"]), eps)
    w = weight_kmajor(out_params["W_action_out"])
    y = torch.empty(h.shape[0], w.shape[0], dtype=BF16, device=h.device)
    dev.gemm(h, w, y)
    return to_host_like(y, out)
