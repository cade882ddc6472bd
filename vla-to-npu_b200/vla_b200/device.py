"""Device-level wrappers: torch CUDA tensors in, libvla_b200 kernels launched on
the current torch stream.  These are thin — shape/stride bookkeeping only; all
arithmetic happens in the CUDA kernels.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import Epilogue

BF16 = torch.bfloat16


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _rowmajor(t: torch.Tensor, name: str) -> int:
    """Row stride (elements) of a 2-D tensor with unit column stride."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name}: need a 2-D tensor with unit column stride, got shape {tuple(t.shape)} "
                         f"strides {t.stride()}")
    return t.stride(0)


def make_epilogue(bias=None, residual=None, res_row_mod=0, act=_lib.ACT_NONE, alpha=1.0, rope_cs=None, rope_seq=0,
                  rope_ncols=0, out_grp=0, out_grp_stride=0, euler_x=None, euler_dt=0.0) -> Epilogue:
    e = Epilogue()
    e.bias = None if bias is None else bias.data_ptr()
    e.residual = None if residual is None else residual.data_ptr()
    e.ldr = 0 if residual is None else _rowmajor(residual, "residual")
    e.res_row_mod = res_row_mod
    e.act = act
    e.alpha = alpha
    e.rope_cs = None if rope_cs is None else rope_cs.data_ptr()
    e.rope_seq = rope_seq
    e.rope_ncols = rope_ncols
    e.out_grp = out_grp
    e.out_grp_stride = out_grp_stride
    e.euler_x = None if euler_x is None else euler_x.data_ptr()
    e.ldx = 0 if euler_x is None else _rowmajor(euler_x, "euler_x")
    e.euler_dt = euler_dt
    return e


def gemm(a: torch.Tensor, w_t: torch.Tensor, out: torch.Tensor, epi: Optional[Epilogue] = None, m: Optional[int] = None,
         tile_n: int = 0) -> torch.Tensor:
    """out = epilogue(a @ w_t.T) with a [M, K] and w_t [N, K] (K-major weights)."""
    lda = _rowmajor(a, "a")
    ldb = _rowmajor(w_t, "w_t")
    ldc = _rowmajor(out, "out")
    M = a.shape[0] if m is None else m
    N, K = w_t.shape
    if a.shape[1] != K:
        raise ValueError(f"gemm: a has K={a.shape[1]}, w_t has K={K}")
    ep = ctypes.byref(epi) if epi is not None else None
    if tile_n:
        _lib.call("vla_gemm_bf16_tiled", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, tile_n, _stream())
    else:
        _lib.call("vla_gemm_bf16", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, _stream())
    return out


def sync_check() -> None:
    _lib.call("vla_sync_check")
