"""ctypes binding of libvla_b200.so (the C ABI declared in include/vla_b200.h).

The library is built in-tree (``make -C vla-to-npu_b200/csrc``).  There is no
CPU or PyTorch fallback: if the shared object is missing or a call fails, a
``VlaError`` is raised.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvla_b200.so")

VLA_OK = 0
VLA_E_INVALID = -1
VLA_E_ALIGN = -2
VLA_E_CUDA = -3
VLA_E_UNSUPPORTED = -4
VLA_E_DEVICE_TIMEOUT = -5
VLA_E_WORKSPACE = -6

ACT_NONE = 0
ACT_GELU_TANH = 1
ACT_SWIGLU = 2
ACT_ROPE = 3
ACT_EULER = 4


class VlaError(RuntimeError):
    """A libvla_b200 call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libvla_b200 error {code}: {msg}")
        self.code = code


class Epilogue(ctypes.Structure):
    """Mirror of ``vla_epilogue`` (include/vla_b200.h)."""

    _fields_ = [
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
        ("res_row_mod", ctypes.c_int32),
        ("act", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("rope_seq", ctypes.c_int32),
        ("rope_cs", ctypes.c_void_p),
        ("rope_ncols", ctypes.c_int32),
        ("out_grp", ctypes.c_int32),
        ("out_grp_stride", ctypes.c_int64),
        ("euler_x", ctypes.c_void_p),
        ("ldx", ctypes.c_int64),
        ("euler_dt", ctypes.c_float),
        ("b_static", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3),
    ]


class AttentionArgs(ctypes.Structure):
    """Mirror of ``vla_attention_args``."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("o", ctypes.c_void_p),
        ("q_row", ctypes.c_int64), ("k_row", ctypes.c_int64), ("v_row", ctypes.c_int64), ("o_row", ctypes.c_int64),
        ("q_batch", ctypes.c_int64), ("k_batch", ctypes.c_int64), ("v_batch", ctypes.c_int64),
        ("o_batch", ctypes.c_int64),
        ("batch", ctypes.c_int32), ("Lq", ctypes.c_int32), ("Lk", ctypes.c_int32), ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("causal", ctypes.c_int32),
        ("kv_len", ctypes.c_void_p), ("scale", ctypes.c_float), ("impl", ctypes.c_int32),
    ]


ATTN_AUTO = 0
ATTN_MMA_SYNC = 1
ATTN_TCGEN05 = 2
ATTN_TCGEN05_SHORT = 3
ATTN_TCGEN05_PIPE = 4


class LlamaLayer(ctypes.Structure):
    """Mirror of ``vla_llama_layer``."""

    _fields_ = [
        ("norm1", ctypes.c_void_p), ("w_qkv", ctypes.c_void_p), ("w_o", ctypes.c_void_p),
        ("norm2", ctypes.c_void_p), ("w_gu", ctypes.c_void_p), ("w_down", ctypes.c_void_p),
        ("hidden", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("ffn", ctypes.c_int32), ("eps", ctypes.c_float),
    ]


class VisionLayer(ctypes.Structure):
    """Mirror of ``vla_vision_layer``."""

    _fields_ = [
        ("ln1_g", ctypes.c_void_p), ("ln1_b", ctypes.c_void_p), ("w_qkv", ctypes.c_void_p),
        ("b_qkv", ctypes.c_void_p), ("w_o", ctypes.c_void_p), ("b_o", ctypes.c_void_p),
        ("ln2_g", ctypes.c_void_p), ("ln2_b", ctypes.c_void_p), ("w_fc1", ctypes.c_void_p),
        ("b_fc1", ctypes.c_void_p), ("w_fc2", ctypes.c_void_p), ("b_fc2", ctypes.c_void_p),
        ("hidden", ctypes.c_int32), ("heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("ffn", ctypes.c_int32), ("eps", ctypes.c_float),
    ]


class ProfileRecord(ctypes.Structure):
    """Mirror of ``vla_profile_record``."""

    _fields_ = [("kind", ctypes.c_int32), ("ms", ctypes.c_float), ("flops", ctypes.c_double),
                ("bytes", ctypes.c_double), ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("tile_n", ctypes.c_int32), ("ctas", ctypes.c_int32)]


KIND_NAMES = ["gemm", "attention", "norm", "rope", "softmax", "elementwise", "layout"]

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F32 = ctypes.c_float

# name -> argtypes; every function returns int status unless listed in _RET.
SIGNATURES = {
    "vla_version": [],
    "vla_last_error": [],
    "vla_sync_check": [],
    "vla_peek_device_error": [ctypes.POINTER(ctypes.c_uint)],
    "vla_test_expired_wait": [_I32, _P],
    "vla_test_exp2_fma": [_P, _P, _I64, _P],
    "vla_abi_sizes": [ctypes.POINTER(ctypes.c_int64), _I32],
    "vla_launch_count": [],
    "vla_set_launch_overlap": [_I32],
    "vla_set_fused_layers": [_I32],
    "vla_profile_start": [_I32],
    "vla_profile_stop": [ctypes.POINTER(ProfileRecord), _I32, ctypes.POINTER(ctypes.c_int32)],
    "vla_gemm_bf16": [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, ctypes.POINTER(Epilogue), _P],
    "vla_gemm_bf16_tiled": [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, ctypes.POINTER(Epilogue), _I32, _P],
    "vla_gemm_bf16_ex": [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, ctypes.POINTER(Epilogue), _I32, _I32, _P],
    "vla_gemm_bf16_split": [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, ctypes.POINTER(Epilogue), _I32, _I32, _P],
    "vla_rms_norm_bf16": [_P, _I64, _P, _P, _I64, _I64, _I64, _F32, _P],
    "vla_layer_norm_bf16": [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _F32, _P],
    "vla_rope_bf16": [_P, _I64, _I64, _I32, _I32, _P, _P],
    "vla_rope_table": [_P, _I32, _I32, ctypes.c_double],
    "vla_softmax_bf16": [_P, _I64, _P, _I64, _I64, _I64, _F32, _I32, _P],
    "vla_elementwise_bf16": [_I32, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _P],
    "vla_attention_bf16": [ctypes.POINTER(AttentionArgs), _P],
    "vla_pixel_shuffle_bf16": [_P, _P, _I32, _I32, _I32, _I32, _P],
    "vla_patch_im2col_bf16": [_P, _P, _I32, _I32, _I32, _I32, _I32, _P],
    "vla_embed_bf16": [_P, _P, _I32, _I32, _I32, _I32, _F32, _P, _I64, _I32, _I32, _P],
    "vla_f32_to_bf16": [_P, _I64, _P, _I64, _I64, _I64, _P],
    "vla_pusht_render_u8": [_P, _I32, _I32, _P, _P],
    "vla_camera_preprocess_u8": [_P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P],
    "vla_llama_layer_workspace": [ctypes.POINTER(LlamaLayer), _I64, _I32],
    "vla_llama_self_layer_bf16": [ctypes.POINTER(LlamaLayer), _P, _I32, _I32, _P, _P, _P, ctypes.c_size_t, _P],
    "vla_llama_cross_layer_bf16": [ctypes.POINTER(LlamaLayer), _P, _I32, _I32, _P, _P, _P, _I64, _I32, _P, _P,
                                   ctypes.c_size_t, _P],
    "vla_vision_layer_workspace": [ctypes.POINTER(VisionLayer), _I64],
    "vla_noalloc_scratch_bytes": [],
    "vla_llama_self_layer_bf16_noalloc": [ctypes.POINTER(LlamaLayer), _P, _I32, _I32, _P, _P, _P],
    "vla_vision_layer_bf16": [ctypes.POINTER(VisionLayer), _P, _I32, _I32, _P, ctypes.c_size_t, _P],
}
_RET = {"vla_last_error": ctypes.c_char_p, "vla_launch_count": ctypes.c_uint64, "vla_llama_layer_workspace": ctypes.c_size_t,
        "vla_vision_layer_workspace": ctypes.c_size_t, "vla_noalloc_scratch_bytes": ctypes.c_size_t}

EW_GELU_TANH = 0
EW_SILU = 1
EW_SILU_MUL = 2
EW_ADD = 3

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise VlaError(VLA_E_UNSUPPORTED, f"{LIB_PATH} not built (run `make -C vla-to-npu_b200/csrc`)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RET.get(name, ctypes.c_int)
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().vla_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc != VLA_OK:
        raise VlaError(rc, last_error())


def call(name: str, *args) -> None:
    """Invoke an entry point and raise ``VlaError`` on a negative status."""
    check(getattr(load(), name)(*args))
