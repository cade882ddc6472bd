"""The reference-named entry points (drop-ins for vla/*_bf16.py block builders and
the per-op harnesses) called the way the reference's own __main__ tests call them:
numpy inputs (float32 or ml_dtypes.bfloat16), params in [in, out] layout, numpy
bf16 outputs, gate atol = rtol = 1e-1 against the torch bf16 oracle
(vla/text_encoder_bf16.py:627-629, vla/action_expert_bf16.py:849-851)."""
import ml_dtypes
import numpy as np
import pytest
import torch

from oracle import smolvla_ref as R
from vla_b200 import weights as W
from vla_b200.configs import ExpertCfg, TextCfg, VisionCfg

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
NPBF = ml_dtypes.bfloat16


def _np(params):
    """reference-style params: numpy bf16 arrays"""
    return {k: v.float().numpy().astype(NPBF) for k, v in params.items()}


def _close(ours, ref, tol=1e-1):
    assert isinstance(ours, np.ndarray) and ours.dtype == NPBF
    np.testing.assert_allclose(ours.astype(np.float32), ref.float().numpy(), atol=tol, rtol=tol)


def test_text_encoder_forward(cuda):
    from vla_b200.text_encoder_bf16 import text_encoder_forward
    cfg = TextCfg()
    p = W.text_block_params(cfg, seed=3)
    x = W.randn((128, cfg.hidden), 3, "dropin.x", dtype=torch.float32)
    out, key, value = text_encoder_forward(x.numpy(), _np(p))
    o, k, v = R.text_block(x.to(BF)[None], p, cfg, dt=BF)
    _close(out, o[0])
    _close(value, v[0])
    # post-RoPE K against the fp32 oracle: the reference's bf16 module rounds its RoPE
    # timescale buffer to bf16, which alone moves K by up to ~0.4 at position 127
    _, k32, _ = R.text_block(x.to(BF)[None], p, cfg, dt=torch.float32)
    _close(key, k32[0])


def test_llama_block_rope_768(cuda):
    """The reference's 768-wide block: SEQ 64, EMBD 768, 15/5 heads, FFN 3072, RoPE base 1e4."""
    from vla_b200.llama_block_rope_bf16 import llama_block_rope
    cfg = TextCfg(hidden=768, heads=15, kv_heads=5, ffn=3072, rope_theta=1e4)
    p = W.text_block_params(cfg, seed=4)
    x = W.randn((64, 768), 4, "dropin.x768", dtype=torch.float32)
    out, key, value = llama_block_rope(x.numpy(), _np(p))
    o, k, v = R.text_block(x.to(BF)[None], p, cfg, dt=BF)
    _close(out, o[0])
    _, k32, _ = R.text_block(x.to(BF)[None], p, cfg, dt=torch.float32)
    _close(key, k32[0])


def test_vision_block(cuda):
    from vla_b200.vision_block_bf16 import vision_block
    cfg = VisionCfg()
    p = W.vision_block_params(cfg, seed=5)
    x = W.randn((1024, cfg.hidden), 5, "dropin.xv", dtype=torch.float32)
    out = vision_block(x.numpy().astype(NPBF), _np(p))
    _close(out, R.vision_block(x.to(BF)[None], p, cfg, dt=BF)[0])


def test_action_expert_forward(cuda):
    from vla_b200.action_expert_bf16 import action_expert_cross_forward, action_expert_self_forward
    e, t = ExpertCfg(), TextCfg()
    ps, pc = W.expert_self_params(e, seed=6), W.expert_cross_params(e, t.kv_dim, seed=6, layer=1)
    x = W.randn((50, e.hidden), 6, "dropin.xe", dtype=torch.float32)
    tk = W.randn((113, t.kv_dim), 6, "dropin.tk", dtype=torch.float32)
    tv = W.randn((113, t.kv_dim), 6, "dropin.tv", dtype=torch.float32)
    _close(action_expert_self_forward(x.numpy(), _np(ps)), R.expert_self_block(x.to(BF)[None], ps, e, dt=BF)[0])
    kc, vc = R.expert_cross_kv(tk.to(BF)[None], tv.to(BF)[None], pc, dt=BF)
    ref = R.expert_cross_block(x.to(BF)[None], kc, vc, pc, e, dt=BF)[0]
    _close(action_expert_cross_forward(x.numpy(), tk.numpy(), tv.numpy(), _np(pc)), ref)


def test_connector_and_preprocessing(cuda):
    from vla_b200.connector_bf16 import connector_block
    from vla_b200.preprocessing_bf16 import preprocessing_block
    v = VisionCfg()
    x = W.randn((1024, 768), 7, "dropin.xc", dtype=torch.float32)
    w = W.randn((12288, 960), 7, "dropin.Wc", std=0.02)
    out = connector_block(x.numpy().astype(NPBF), {"W": w.float().numpy().astype(NPBF)})
    ref = R.connector(x.to(BF)[None], w, v, 4, dt=torch.float32)[0]
    _close(out, ref, tol=1e-1)  # reference gate: rtol 1e-1 (vla/connector_bf16.py:153)
    pp = W.patch_embed_params(v, seed=7)
    img = W.uniform((3, 512, 512), 7, "dropin.img", -1.0, 1.0, dtype=torch.float32)
    out = preprocessing_block(img.numpy(), {"kernel": pp["kernel"].float().numpy().astype(NPBF)})
    ref = torch.nn.functional.conv2d(img.to(BF)[None].float(), pp["kernel"].float(), stride=16)
    _close(out, ref.flatten(2).transpose(1, 2)[0])


def test_joint_transformer_and_postprocessing(cuda):
    from vla_b200.vla import joint_transformer, postprocessing
    t, e = TextCfg(), ExpertCfg()
    pt = W.text_block_params(t, seed=8)
    ps, pc = W.expert_self_params(e, seed=8), W.expert_cross_params(e, t.kv_dim, seed=8, layer=1)
    vlm = W.randn((113, t.hidden), 8, "dropin.vlm", dtype=torch.float32)
    act = W.randn((50, e.hidden), 8, "dropin.act", dtype=torch.float32)
    out = joint_transformer(2, vlm.numpy(), act.numpy(), _np(pt), _np(ps), _np(pc))
    # oracle of the same schedule (vla/vla.py:489-504)
    x, a = vlm.to(BF)[None], act.to(BF)[None]
    for i in range(2):
        x, k, v = R.text_block(x, pt, t, dt=BF)
        if i % 2 == 0:
            a = R.expert_self_block(a, ps, e, dt=BF)
        else:
            kc, vc = R.expert_cross_kv(k, v, pc, dt=BF)
            a = R.expert_cross_block(a, kc, vc, pc, e, dt=BF)
    _close(out, a[0])
    post = {"W_exp_norm": np.ones(e.hidden, dtype=NPBF),
            "W_action_out": W.randn((e.hidden, 32), 8, "dropin.wout", std=0.02).float().numpy().astype(NPBF)}
    y = postprocessing(out, post)
    ref = R.linear(R.rms_norm(torch.from_numpy(out.astype(np.float32)), torch.ones(e.hidden), 1e-5),
                   torch.from_numpy(post["W_action_out"].astype(np.float32)))
    _close(y, ref)


def test_per_op_harness_names(cuda):
    from vla_b200 import ops
    g = torch.Generator().manual_seed(9)
    a = (torch.rand(64, 960, generator=g) * 0.1).numpy().astype(NPBF)
    b = (torch.rand(960, 768, generator=g) * 0.1).numpy().astype(NPBF)
    c = ops.gemm(a, b)  # gemm/v1_test_tiled_gemm.py: U[0, 0.1) inputs, atol 1e-1 rtol 1e-2
    np.testing.assert_allclose(c.astype(np.float32), a.astype(np.float32) @ b.astype(np.float32), atol=1e-1,
                               rtol=1e-2)
    x = torch.randn(16, 960, generator=g).numpy().astype(NPBF)
    w = np.ones(960, dtype=NPBF)
    np.testing.assert_allclose(ops.rms_norm(x, w).astype(np.float32),
                               R.rms_norm(torch.from_numpy(x.astype(np.float32)), torch.ones(960), 1e-5).numpy(),
                               atol=1e-1, rtol=2e-2)
    s = torch.randn(8, 128, generator=g).numpy().astype(NPBF)
    ms = ops.masked_softmax(s, row_start=96).astype(np.float32)
    assert np.allclose(ms.sum(-1), 1.0, atol=2e-2) and (ms[0, 97:] == 0).all()
    q = torch.randn(128, 15 * 64, generator=g).numpy().astype(NPBF)
    r = ops.rope_apply_packed(q, heads=15).astype(np.float32)
    ref = R.apply_rope(torch.from_numpy(q.astype(np.float32)).view(1, 128, 15, 64), 1e4).reshape(128, -1).numpy()
    np.testing.assert_allclose(r, ref, atol=2e-2, rtol=1e-2)
    xs = torch.randn(4, 768, generator=g).numpy().astype(NPBF)
    np.testing.assert_allclose(ops.gelu(xs).astype(np.float32),
                               torch.nn.functional.gelu(torch.from_numpy(xs.astype(np.float32)),
                                                        approximate="tanh").numpy(), atol=1e-1, rtol=1e-2)
    np.testing.assert_allclose(ops.silu(xs).astype(np.float32),
                               torch.nn.functional.silu(torch.from_numpy(xs.astype(np.float32))).numpy(), atol=5e-2,
                               rtol=1e-1)
