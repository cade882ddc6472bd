"""Per-op entry points with the reference's harness names.

Each function takes host arrays (numpy, including ``ml_dtypes.bfloat16``, or
torch CPU/CUDA tensors), runs one CUDA kernel of libvla_b200, and returns the
result in the caller's array type.  They stand in for the reference's NPU
modules as its per-op tests call them:

  gemm            Allo GEMM module            gemm/v1_test_tiled_gemm.py:51-157
  rms_norm        rms_norm_960_bf16 / rms_norm_bf16
                                              rms_norm/test_rms_norm_bf16.py:51-81,
                                              vla/tests/test_rms_norm_960_bf16.py:321-356
  layer_norm      layer_norm_bf16 (+ bias)    layer_norm/test_layer_bf16.py:154-187
  rope_apply_packed                           vla/text_encoder_bf16.py:422-475
  softmax         softmax_bf16_32_128 / softmax_float32_seq1024
                                              softmax_bf16/test_softmax_bf16_seq1024.py
  masked_softmax  masked_softmax_128_bf16     vla/tests/test_masked_softmax_128_bf16.py
  gelu            gelu_bf16 (tanh form)       gelu/test_gelu_bf16.py
  silu            silu_*_bf16                 silu/test_silu_bf16.py, vla/tests/test_silu_160_bf16.py
  attention_score transpose_matmul_with_scale attn_score/test_attn_score_bf16.py
"""
from __future__ import annotations

import torch

from . import _lib
from . import device as dev
from ._host import to_device, to_host_like
from .model import rope_table

BF16 = torch.bfloat16


def gemm(A, B):
    """C = A[M, K] @ B[K, N] (bf16 in, fp32 accumulate, bf16 out)."""
    a = to_device(A)
    bt = to_device(B).t().contiguous()
    M, N = a.shape[0], bt.shape[0]
    Np = (N + 15) // 16 * 16
    if Np != N:
        bt = torch.cat([bt, torch.zeros(Np - N, bt.shape[1], dtype=BF16, device=bt.device)])
    Kp = (a.shape[1] + 7) // 8 * 8
    if Kp != a.shape[1]:
        a = torch.nn.functional.pad(a, (0, Kp - a.shape[1]))
        bt = torch.nn.functional.pad(bt, (0, Kp - bt.shape[1]))
    out = torch.empty(M, Np, dtype=BF16, device=a.device)
    dev.gemm(a, bt, out)
    return to_host_like(out[:, :N], A)


def rms_norm(x, weight, eps: float = 1e-5):
    xd = to_device(x)
    shape = xd.shape
    xd = xd.reshape(-1, shape[-1])
    y = dev.rms_norm(xd, to_device(weight), eps)
    return to_host_like(y.reshape(shape), x)


def layer_norm(x, weight, bias, eps: float = 1e-6):
    xd = to_device(x)
    shape = xd.shape
    xd = xd.reshape(-1, shape[-1])
    y = dev.layer_norm(xd, to_device(weight), to_device(bias), eps)
    return to_host_like(y.reshape(shape), x)


def rope_apply_packed(packed_bf16, heads, head_dim=64, max_wavelength=10_000.0, pos_offset=0):
    """RoPE on [seq, heads*head_dim] packed heads; positions pos_offset + row."""
    if head_dim != 64:
        raise _lib.VlaError(_lib.VLA_E_UNSUPPORTED, "rope: head_dim must be 64")
    x = to_device(packed_bf16)
    seq = x.shape[0]
    cs = rope_table(pos_offset + seq, head_dim, max_wavelength)[pos_offset:].contiguous().to(x.device)
    dev.rope_(x, heads * head_dim, seq, cs)
    return to_host_like(x, packed_bf16)


def softmax(scores, scale: float = 1.0):
    x = to_device(scores)
    return to_host_like(dev.softmax(x, scale, -1), scores)


def masked_softmax(scores, row_start: int = 0, scale: float = 1.0):
    """Causal row softmax of a tile whose first row is query row ``row_start``."""
    x = to_device(scores)
    return to_host_like(dev.softmax(x, scale, int(row_start)), scores)


def gelu(x):
    xd = to_device(x)
    return to_host_like(dev.elementwise(_lib.EW_GELU_TANH, xd.reshape(-1, xd.shape[-1])).reshape(xd.shape), x)


def silu(x):
    xd = to_device(x)
    return to_host_like(dev.elementwise(_lib.EW_SILU, xd.reshape(-1, xd.shape[-1])).reshape(xd.shape), x)


def attention_score(q, k, scale: float = 0.125):
    """q[M, D] . k[N, D]^T * scale (the reference's transpose_matmul_with_scale)."""
    qd = to_device(q)
    kd = to_device(k)
    N = kd.shape[0]
    Np = (N + 15) // 16 * 16
    if Np != N:
        kd = torch.cat([kd, torch.zeros(Np - N, kd.shape[1], dtype=BF16, device=kd.device)])
    out = torch.empty(qd.shape[0], Np, dtype=BF16, device=qd.device)
    dev.gemm(qd, kd, out, dev.make_epilogue(alpha=scale))
    return to_host_like(out[:, :N], q)
