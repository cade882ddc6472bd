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
                  rope_ncols=0, out_grp=0, out_grp_stride=0, euler_x=None, euler_dt=0.0, b_static=False) -> Epilogue:
    """``b_static``: B is a weight no earlier work in the stream writes (its first
    tiles may be fetched while the previous kernel drains)."""
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
    e.b_static = 1 if b_static else 0
    # the struct holds raw device addresses: keep the tensors alive with it
    e._keep = (bias, residual, rope_cs, euler_x)
    return e


def gemm(a: torch.Tensor, w_t: torch.Tensor, out: torch.Tensor, epi: Optional[Epilogue] = None, m: Optional[int] = None,
         tile_n: int = 0, ctas: int = 0, splits: Optional[int] = None) -> torch.Tensor:
    """out = epilogue(a @ w_t.T) with a [M, K] and w_t [N, K] (K-major weights).
    ``splits`` (one-CTA tiles only) forces the K split: 1 = none, 2..8 CTAs per tile."""
    lda = _rowmajor(a, "a")
    ldb = _rowmajor(w_t, "w_t")
    ldc = _rowmajor(out, "out")
    M = a.shape[0] if m is None else m
    N, K = w_t.shape
    if a.shape[1] != K:
        raise ValueError(f"gemm: a has K={a.shape[1]}, w_t has K={K}")
    ep = ctypes.byref(epi) if epi is not None else None
    if splits is not None:
        _lib.call("vla_gemm_bf16_split", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, tile_n, splits,
                  _stream())
    elif ctas:
        _lib.call("vla_gemm_bf16_ex", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, tile_n, ctas,
                  _stream())
    elif tile_n:
        _lib.call("vla_gemm_bf16_tiled", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, tile_n, _stream())
    else:
        _lib.call("vla_gemm_bf16", _ptr(a), lda, _ptr(w_t), ldb, _ptr(out), ldc, M, N, K, ep, _stream())
    return out


def sync_check() -> None:
    _lib.call("vla_sync_check")


def rms_norm(x: torch.Tensor, g: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    M, N = x.shape
    _lib.call("vla_rms_norm_bf16", _ptr(x), _rowmajor(x, "x"), _ptr(g), _ptr(out), _rowmajor(out, "out"), M, N, eps,
              _stream())
    return out


def layer_norm(x: torch.Tensor, g: torch.Tensor, b: torch.Tensor, eps: float,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    M, N = x.shape
    _lib.call("vla_layer_norm_bf16", _ptr(x), _rowmajor(x, "x"), _ptr(g), _ptr(b), _ptr(out), _rowmajor(out, "out"),
              M, N, eps, _stream())
    return out


def rope_(x: torch.Tensor, ncols: int, seq: int, cs: torch.Tensor) -> torch.Tensor:
    """In-place RoPE on the first ncols columns (64-wide heads); row m has position m % seq."""
    _lib.call("vla_rope_bf16", _ptr(x), _rowmajor(x, "x"), x.shape[0], ncols, seq, _ptr(cs), _stream())
    return x


def softmax(x: torch.Tensor, scale: float = 1.0, causal_row_start: int = -1,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    M, N = x.shape
    _lib.call("vla_softmax_bf16", _ptr(x), _rowmajor(x, "x"), _ptr(out), _rowmajor(out, "out"), M, N, scale,
              causal_row_start, _stream())
    return out


def elementwise(op: int, x: torch.Tensor, y: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    M, N = x.shape
    _lib.call("vla_elementwise_bf16", op, _ptr(x), _rowmajor(x, "x"), _ptr(y), 0 if y is None else _rowmajor(y, "y"),
              _ptr(out), _rowmajor(out, "out"), M, N, _stream())
    return out


def attention(q, k, v, o, *, batch, Lq, Lk, Hq, Hkv, q_batch, k_batch, v_batch, o_batch, causal=False,
              kv_len: Optional[torch.Tensor] = None, impl: int = 0) -> torch.Tensor:
    """Flash attention over `batch` sequences; q/k/v/o are 2-D row views whose row
    strides are their stride(0); sequence b starts ``*_batch`` elements later."""
    a = _lib.AttentionArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    a.q_row, a.k_row, a.v_row, a.o_row = q.stride(0), k.stride(0), v.stride(0), o.stride(0)
    a.q_batch, a.k_batch, a.v_batch, a.o_batch = q_batch, k_batch, v_batch, o_batch
    a.batch, a.Lq, a.Lk, a.Hq, a.Hkv, a.head_dim = batch, Lq, Lk, Hq, Hkv, 64
    a.causal = 1 if causal else 0
    a.kv_len = None if kv_len is None else kv_len.data_ptr()
    a.scale = 0.125
    a.impl = impl
    _lib.call("vla_attention_bf16", ctypes.byref(a), _stream())
    return o


def pixel_shuffle(x: torch.Tensor, batch: int, grid: int, scale: int, out: torch.Tensor) -> torch.Tensor:
    _lib.call("vla_pixel_shuffle_bf16", _ptr(x), _ptr(out), batch, grid, scale, x.shape[-1], _stream())
    return out


def patch_im2col(img: torch.Tensor, patch: int, out: torch.Tensor) -> torch.Tensor:
    B, C, H, W = img.shape
    _lib.call("vla_patch_im2col_bf16", _ptr(img), _ptr(out), B, C, H, W, patch, _stream())
    return out


def camera_preprocess(frames: torch.Tensor, size: int, out: torch.Tensor, patch: int = 0) -> torch.Tensor:
    """uint8 camera frames [B, H, W, 3] -> bf16 model input in [-1, 1], bilinearly
    resized to size x size: the NCHW image [B, 3, size, size] when ``patch`` is 0,
    else the patch-embedding GEMM operand [B * (size/patch)^2, 3 * patch^2]."""
    if frames.dtype != torch.uint8 or frames.dim() != 4 or frames.shape[3] != 3 or not frames.is_contiguous():
        raise ValueError("camera_preprocess: need contiguous uint8 frames [B, H, W, 3]")
    B, H, W, _ = frames.shape
    _lib.call("vla_camera_preprocess_u8", _ptr(frames), B, H, W, size, patch, 1 if patch else 0, _ptr(out),
              _stream())
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, scale: float, out: torch.Tensor, rows_per_seq: int,
          row_offset: int) -> torch.Tensor:
    B, T = ids.shape
    vocab, H = table.shape
    _lib.call("vla_embed_bf16", _ptr(ids), _ptr(table), vocab, H, B, T, scale, _ptr(out), _rowmajor(out, "out"),
              rows_per_seq, row_offset, _stream())
    return out


def f32_to_bf16(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    M, N = x.shape
    _lib.call("vla_f32_to_bf16", _ptr(x), _rowmajor(x, "x"), _ptr(out), _rowmajor(out, "out"), M, N, _stream())
    return out


class Workspace:
    """Grow-only device scratch buffer shared by the block calls of one model."""

    def __init__(self, device=None):
        self.device = device
        self.buf = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device or "cuda")
        return self.buf


def llama_self_layer(layer: "_lib.LlamaLayer", x: torch.Tensor, batch: int, seq: int, rope_cs: torch.Tensor,
                     ws: Workspace, qkv_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    rows = batch * seq
    nbytes = _lib.load().vla_llama_layer_workspace(ctypes.byref(layer), rows, 0 if qkv_out is not None else 1)
    buf = ws.get(nbytes)
    _lib.call("vla_llama_self_layer_bf16", ctypes.byref(layer), _ptr(x), batch, seq, _ptr(rope_cs), _ptr(qkv_out),
              _ptr(buf), buf.numel(), _stream())
    return x


def llama_cross_layer(layer: "_lib.LlamaLayer", x: torch.Tensor, batch: int, seq: int, rope_cs: torch.Tensor,
                      k: torch.Tensor, v: torch.Tensor, kv_seq: int, ws: Workspace,
                      kv_len: Optional[torch.Tensor] = None) -> torch.Tensor:
    rows = batch * seq
    nbytes = _lib.load().vla_llama_layer_workspace(ctypes.byref(layer), rows, 1)
    buf = ws.get(nbytes)
    if k.stride(0) != v.stride(0):
        raise ValueError("k and v must share a row stride")
    _lib.call("vla_llama_cross_layer_bf16", ctypes.byref(layer), _ptr(x), batch, seq, _ptr(rope_cs), _ptr(k), _ptr(v),
              k.stride(0), kv_seq, _ptr(kv_len), _ptr(buf), buf.numel(), _stream())
    return x


def vision_layer(layer: "_lib.VisionLayer", x: torch.Tensor, batch: int, seq: int, ws: Workspace) -> torch.Tensor:
    rows = batch * seq
    nbytes = _lib.load().vla_vision_layer_workspace(ctypes.byref(layer), rows)
    buf = ws.get(nbytes)
    _lib.call("vla_vision_layer_bf16", ctypes.byref(layer), _ptr(x), batch, seq, _ptr(buf), buf.numel(), _stream())
    return x
