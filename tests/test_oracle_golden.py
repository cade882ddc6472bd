"""Pin the CPU oracle to the reference: run the oracle on the golden cases and
compare with the outputs the reference's own torch code produced
(tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from oracle import smolvla_ref as R
from vla_b200.configs import VisionCfg

import sys
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from golden_cases import EXP_CFG, LLAMA_CFG, TEXT_CFG, VIT_CFG, case_inputs  # noqa: E402

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_oracle.npz"))
BF = torch.bfloat16


def _cmp(ours: torch.Tensor, key: str, atol=0.0, rtol=0.0):
    ref = torch.from_numpy(GOLD[key]).reshape(ours.shape)
    torch.testing.assert_close(ours.float(), ref, atol=atol, rtol=rtol)


def test_text_block_reference_semantics():
    """Reference class as written: RoPE base 1e4, nn.RMSNorm(eps=None) — which torch
    evaluates in fp32 with the fp32 epsilon even for bf16 input — and K/V
    recomputed from ln_1(residual)."""
    inp = case_inputs("text_ref")
    cfg = TEXT_CFG.__class__(**{**TEXT_CFG.__dict__, "eps": torch.finfo(torch.float32).eps, "rope_theta": 1e4})
    out, k, v = R.text_block(inp["args"][0], inp["params"], cfg, dt=BF, kv_export="recompute")
    _cmp(out, "text_ref.bf16.0")
    _cmp(k, "text_ref.bf16.1")
    _cmp(v, "text_ref.bf16.2")


def test_text_block_c0_params():
    inp = case_inputs("text_c0")
    cfg = TEXT_CFG.__class__(**{**TEXT_CFG.__dict__, "eps": 1e-5, "rope_theta": 1e5})
    out, k, v = R.text_block(inp["args"][0], inp["params"], cfg, dt=BF, kv_export="recompute")
    _cmp(out, "text_c0.bf16.0")
    _cmp(k, "text_c0.bf16.1")
    _cmp(v, "text_c0.bf16.2")


def test_expert_self_block():
    inp = case_inputs("exp_self")
    out = R.expert_self_block(inp["args"][0], inp["params"], EXP_CFG, dt=BF)
    _cmp(out, "exp_self.bf16")


def test_expert_cross_block():
    inp = case_inputs("exp_cross")
    x, tk, tv = inp["args"]
    kc, vc = R.expert_cross_kv(tk.to(BF), tv.to(BF), inp["params"], dt=BF)
    out = R.expert_cross_block(x, kc, vc, inp["params"], EXP_CFG, dt=BF)
    _cmp(out, "exp_cross.bf16")


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_minivit_block(mode):
    """MiniVit: zero attention biases, no MLP bias, LayerNorm eps 1e-5, erf GELU; torch's
    nn.MultiheadAttention computes the attention (fused kernel), so fp32 agrees to
    rounding and bf16 to one bf16 ulp of the probabilities."""
    inp = case_inputs("minivit")
    p = {k: v for k, v in inp["params"].items() if not k.startswith("b") or k.startswith("b_norm")}
    cfg = VisionCfg(hidden=VIT_CFG.hidden, heads=VIT_CFG.heads, head_dim=64, ffn=VIT_CFG.ffn, eps=1e-5)
    dt = torch.float32 if mode == "f32" else BF
    out = R.vision_block(inp["args"][0], p, cfg, dt=dt, gelu="none")
    if mode == "f32":
        _cmp(out, "minivit.f32", atol=2e-5, rtol=2e-5)
    else:
        _cmp(out, "minivit.bf16", atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_siglip_embeddings(mode):
    inp = case_inputs("siglip_emb")
    cfg = VisionCfg(hidden=128, image=64, patch=16)
    dt = torch.float32 if mode == "f32" else BF
    out = R.patch_embed(inp["args"][0], inp["params"], cfg, dt=dt)
    _cmp(out, f"siglip_emb.{mode}", atol=1e-5 if mode == "f32" else 0.0, rtol=1e-5 if mode == "f32" else 0.0)


def test_connector_pixel_shuffle():
    inp = case_inputs("con_ref")
    cfg = VisionCfg()
    out = R.connector(inp["x"][None].float(), inp["params"]["W"].float(), cfg, scale=4)
    _cmp(out[0], "con_ref", atol=1e-3, rtol=1e-4)


def test_masked_softmax_cpu():
    """Reference CPU causal softmax (vla/action_expert_bf16.py:530-538) vs the oracle's
    attention masking rule on the same scores."""
    s = case_inputs("masked_softmax_cpu")["x"].float()
    L = s.shape[0]
    s = s.masked_fill(torch.ones(L, L).triu(1).bool(), float("-inf"))
    p = torch.softmax(s, dim=-1).to(BF)
    _cmp(p, "masked_softmax_cpu", atol=0, rtol=0)


def test_llama_block_rope_self():
    """AttentionExpertBlock (vla/llama_block_rope_bf16.py:60-131), the torch twin of
    llama_block_rope, against the oracle's text block with its hyper-parameters."""
    inp = case_inputs("llama_rope")
    out, _, _ = R.text_block(inp["args"][0], inp["params"], LLAMA_CFG, dt=BF)
    _cmp(out, "llama_rope.bf16")


def test_llama_block_rope_cross_pinned_by_self_block():
    """The Allo cross path (vla/llama_block_rope_bf16.py:617-709) given key =
    RMSNorm(x) Wk before RoPE and value = RMSNorm(x) Wv computes exactly the self
    block, so the reference's AttentionExpertBlock output pins the restatement."""
    inp = case_inputs("llama_rope")
    x, p = inp["args"][0], inp["params"]
    h = R.rms_norm(x.to(BF), p["W_norm_1"], LLAMA_CFG.eps, BF)
    key, value = R.linear(h, p["Wk"], dt=BF), R.linear(h, p["Wv"], dt=BF)
    out = R.llama_block_rope_cross(key, value, x, p, LLAMA_CFG, dt=BF)
    _cmp(out, "llama_rope.bf16")


def test_cross_attention_block():
    """CrossAttentionBlock (vla/llama_block_rope_bf16.py:133-180): context through
    ln_1 and k_proj / v_proj, no RoPE, no mask."""
    inp = case_inputs("cross_attn")
    x, ctx = inp["args"]
    out = R.cross_attention_block(x, ctx, inp["params"], LLAMA_CFG, dt=BF)
    _cmp(out, "cross_attn.bf16")


@pytest.mark.parametrize("seed", [0, 3, 99])
def test_pusht_physics_matches_reference_env(seed):
    """vla_b200.pusht.PushTBatch restates simulation/pusht_env.py's physics; on the
    reference environment's own trajectories (reset from the seed, 150 steps of
    pushes with contact) it reproduces every state, and batching environments
    changes nothing."""
    from vla_b200.pusht import PushTBatch
    acts = GOLD[f"pusht.{seed}.actions"]
    ref = GOLD[f"pusht.{seed}.states"]
    env = PushTBatch(1, seed)
    got = [env.state()[0]] + [env.step(a[None])[0] for a in acts]
    np.testing.assert_allclose(np.array(got), ref, atol=1e-6, rtol=0)
    # three environments at once, this seed in the middle
    envs = PushTBatch(3, [seed + 7, seed, seed + 11])
    got3 = [envs.state()[1]] + [envs.step(np.stack([a * 0.5, a, -a]))[1] for a in acts]
    np.testing.assert_allclose(np.array(got3), ref, atol=1e-6, rtol=0)
