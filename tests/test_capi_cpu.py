"""CPU-only checks of the C ABI: the shared library loads without a GPU, it
exports every function include/vla_b200.h declares, the ctypes struct mirrors
match the C layouts, and host-side validation rejects bad arguments before any
CUDA call."""
import ctypes
import os
import re

import pytest
import torch

from vla_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vla_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vla_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    unbound = [n for n in names if n not in _lib.SIGNATURES]
    assert not unbound, f"declared but without a ctypes signature: {unbound}"


def test_abi_struct_sizes_match_ctypes():
    out = (ctypes.c_int64 * 5)()
    assert _lib.load().vla_abi_sizes(out, 5) == 5
    assert list(out) == [ctypes.sizeof(_lib.Epilogue), ctypes.sizeof(_lib.AttentionArgs),
                         ctypes.sizeof(_lib.LlamaLayer), ctypes.sizeof(_lib.VisionLayer),
                         ctypes.sizeof(_lib.ProfileRecord)]


def test_host_validation_without_gpu():
    lib = _lib.load()
    # null operands are rejected before any CUDA call
    rc = lib.vla_gemm_bf16(None, 64, None, 64, None, 64, 16, 16, 64, None, None)
    assert rc == _lib.VLA_E_INVALID
    assert "null" in _lib.last_error()
    # misaligned stride
    rc = lib.vla_gemm_bf16(ctypes.c_void_p(256), 60, ctypes.c_void_p(256), 64, ctypes.c_void_p(256), 64, 16, 16, 60,
                           None, None)
    assert rc == _lib.VLA_E_ALIGN
    rc = lib.vla_llama_self_layer_bf16(None, None, 1, 1, None, None, None, 0, None)
    assert rc == _lib.VLA_E_INVALID
    a = _lib.AttentionArgs()
    a.head_dim = 128
    assert lib.vla_attention_bf16(ctypes.byref(a), None) == _lib.VLA_E_INVALID
    # a well-formed call except for the kernel choice: unknown impl, and the
    # short-sequence tcgen05 kernel forced on with more than 128 keys
    a = _lib.AttentionArgs()
    a.q = a.k = a.v = a.o = 256
    a.q_row, a.k_row, a.v_row, a.o_row = 960, 320, 320, 960
    a.q_batch, a.k_batch, a.v_batch, a.o_batch = 960 * 50, 320 * 200, 320 * 200, 960 * 50
    a.batch, a.Lq, a.Lk, a.Hq, a.Hkv, a.head_dim = 2, 50, 200, 15, 5, 64
    a.scale = 0.125
    a.impl = 5
    assert lib.vla_attention_bf16(ctypes.byref(a), None) == _lib.VLA_E_INVALID
    assert "impl" in _lib.last_error()
    a.impl = _lib.ATTN_TCGEN05_SHORT
    assert lib.vla_attention_bf16(ctypes.byref(a), None) == _lib.VLA_E_INVALID
    assert "128" in _lib.last_error()


def test_rope_table_host_helper_matches_model_table():
    from vla_b200.model import rope_table
    t = torch.empty(128, 64, dtype=torch.float32)
    _lib.call("vla_rope_table", ctypes.c_void_p(t.data_ptr()), 128, 64, 1e5)
    torch.testing.assert_close(t, rope_table(128, 64, 1e5), atol=2e-6, rtol=1e-5)


def test_workspace_query():
    s = _lib.LlamaLayer()
    s.hidden, s.heads, s.kv_heads, s.head_dim, s.ffn = 960, 15, 5, 64, 2560
    n_with = _lib.load().vla_llama_layer_workspace(ctypes.byref(s), 113, 1)
    n_without = _lib.load().vla_llama_layer_workspace(ctypes.byref(s), 113, 0)
    assert n_with - n_without >= 113 * 1600 * 2
    assert n_without >= 113 * (960 + 960 + 2560) * 2


def test_layer_row_count_bounded_before_size_arithmetic():
    """batch * seq at or above 2^31 rows is rejected before any workspace size is
    computed or any kernel launched (the size products would otherwise wrap)."""
    lib = _lib.load()
    s = _lib.LlamaLayer()
    s.norm1 = s.w_qkv = s.w_o = s.norm2 = s.w_gu = s.w_down = 256
    s.hidden, s.heads, s.kv_heads, s.head_dim, s.ffn, s.eps = 960, 15, 5, 64, 2560, 1e-5
    assert lib.vla_llama_layer_workspace(ctypes.byref(s), 1 << 31, 1) == 2 ** 64 - 1
    before = lib.vla_launch_count()
    big = 1 << 20
    rc = lib.vla_llama_self_layer_bf16(ctypes.byref(s), ctypes.c_void_p(256), big, big, ctypes.c_void_p(256), None,
                                       ctypes.c_void_p(256), 2 ** 63, None)
    assert rc == _lib.VLA_E_INVALID and "2^31" in _lib.last_error()
    rc = lib.vla_llama_cross_layer_bf16(ctypes.byref(s), ctypes.c_void_p(256), big, big, ctypes.c_void_p(256),
                                        ctypes.c_void_p(256), ctypes.c_void_p(256), 320, 113, None,
                                        ctypes.c_void_p(256), 2 ** 63, None)
    assert rc == _lib.VLA_E_INVALID and "2^31" in _lib.last_error()
    rc = lib.vla_llama_self_layer_bf16_noalloc(ctypes.byref(s), ctypes.c_void_p(256), big, big,
                                               ctypes.c_void_p(256), None, None)
    assert rc == _lib.VLA_E_INVALID and "2^31" in _lib.last_error()
    assert lib.vla_launch_count() == before


def test_expired_wait_rejects_bad_limits():
    lib = _lib.load()
    assert lib.vla_test_expired_wait(0, None) == _lib.VLA_E_INVALID
    assert lib.vla_test_expired_wait(2_000_000, None) == _lib.VLA_E_INVALID


def test_weight_cache_follows_in_place_refills():
    """Device copies of reference params are reused while the host array is
    unchanged and refreshed when the caller refills it in place (numpy and torch)."""
    import numpy as np
    from vla_b200._host import _Cache, fingerprint
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    f0 = fingerprint(a)
    a[1, 2] = -1.0
    assert fingerprint(a) != f0
    t = torch.zeros(3, 4)
    g0 = fingerprint(t)
    t.add_(1.0)
    assert fingerprint(t) != g0
    # the cache's own behaviour, with a CPU "device copy"
    c = _Cache()
    made = []

    def make(src):
        made.append(1)
        return torch.as_tensor(np.array(src, copy=True))

    orig = torch.cuda.current_device
    torch.cuda.current_device = lambda: 0
    try:
        x1 = c.get(a, "t", lambda: make(a))
        x2 = c.get(a, "t", lambda: make(a))
        assert x1 is x2 and len(made) == 1
        a[0, 0] = 42.0
        x3 = c.get(a, "t", lambda: make(a))
        assert len(made) == 2 and float(x3[0, 0]) == 42.0
        # composite sources: a change in any of them refreshes the entry
        b = np.ones(4, dtype=np.float32)
        c.get((a, b), "cat", lambda: make(b))
        b[0] = 5.0
        c.get((a, b), "cat", lambda: make(b))
        assert len(made) == 4
    finally:
        torch.cuda.current_device = orig
