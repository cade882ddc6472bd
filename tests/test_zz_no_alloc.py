"""The allocation-free layer entry point, vla_llama_self_layer_bf16_noalloc.

Some callers cannot allocate device memory while they run inference: a
real-time control loop that must not call cudaMalloc between actions, a host
framework or plugin sandbox that owns every device buffer, or a foreign-language
binding without a CUDA allocator.  This entry point serves them: its scratch is a
fixed static array inside the library.  The test calls it through the C ABI and
checks it against the workspace-taking entry point vla_llama_self_layer_bf16 on
the same inputs, bit for bit, on two calls in a row (the shared array keeps the first
call's contents), and checks the size limit.  It lives in its own file, named to be
collected last, and sets up everything it needs, so it passes alone in a fresh
process and after the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _layer_and_inputs():
    from vla_b200 import weights as W
    from vla_b200.configs import TextCfg
    from vla_b200.model import LlamaLayerWeights, rope_table
    cfg = TextCfg()
    lw = LlamaLayerWeights(W.text_block_params(cfg, seed=11), cfg, "cuda")
    x = W.randn((128, cfg.hidden), 11, "noalloc.x").cuda()
    cs = rope_table(128, 64, cfg.rope_theta).cuda()
    return cfg, lw, x, cs


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    from vla_b200 import _lib
    lib = _lib.load()
    cfg, lw, x0, cs = _layer_and_inputs()
    nq = cfg.q_dim + 2 * cfg.kv_dim
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # existing entry point with a caller-provided workspace
    ref = x0.clone()
    ref_qkv = torch.empty(128, nq, dtype=BF, device="cuda")
    ws_bytes = lib.vla_llama_layer_workspace(ctypes.byref(lw.struct), 128, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.vla_llama_self_layer_bf16(ctypes.byref(lw.struct), ctypes.c_void_p(ref.data_ptr()), 1, 128,
                                             ctypes.c_void_p(cs.data_ptr()), ctypes.c_void_p(ref_qkv.data_ptr()),
                                             ctypes.c_void_p(ws.data_ptr()), ws_bytes, stream))

    for call in range(2):
        x = x0.clone()
        qkv = torch.full((128, nq), float("nan"), dtype=BF, device="cuda")
        _lib.check(lib.vla_llama_self_layer_bf16_noalloc(ctypes.byref(lw.struct), ctypes.c_void_p(x.data_ptr()), 1,
                                                         128, ctypes.c_void_p(cs.data_ptr()),
                                                         ctypes.c_void_p(qkv.data_ptr()), stream))
        _lib.check(lib.vla_sync_check())
        # the same kernels on the same inputs: any difference would be leftover
        # contents of the shared array or overlapping scratch regions
        assert torch.equal(x, ref), f"call {call}: layer output differs from the workspace entry point"
        assert torch.equal(qkv, ref_qkv), f"call {call}: q/k/v differ from the workspace entry point"

    # without qkv_out the K/V land in the static array too; the layer output must not change
    x = x0.clone()
    _lib.check(lib.vla_llama_self_layer_bf16_noalloc(ctypes.byref(lw.struct), ctypes.c_void_p(x.data_ptr()), 1, 128,
                                                     ctypes.c_void_p(cs.data_ptr()), None, stream))
    _lib.check(lib.vla_sync_check())
    assert torch.equal(x, ref), "layer output without qkv_out differs from the workspace entry point"


def test_noalloc_rejects_requests_above_the_static_size(cuda):
    from vla_b200 import _lib
    lib = _lib.load()
    cfg, lw, x0, cs = _layer_and_inputs()
    limit = lib.vla_noalloc_scratch_bytes()
    assert limit == 8 << 20
    rows = 4096  # far above the 689 rows the 8 MiB array holds at this width
    assert lib.vla_llama_layer_workspace(ctypes.byref(lw.struct), rows, 1) > limit
    big = torch.zeros(rows, cfg.hidden, dtype=BF, device="cuda")
    before = lib.vla_launch_count()
    rc = lib.vla_llama_self_layer_bf16_noalloc(ctypes.byref(lw.struct), ctypes.c_void_p(big.data_ptr()), 32, 128,
                                               ctypes.c_void_p(cs.data_ptr()), None, None)
    assert rc == _lib.VLA_E_WORKSPACE
    assert "static" in _lib.last_error()
    assert lib.vla_launch_count() == before, "a rejected request must not launch anything"
