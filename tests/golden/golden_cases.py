"""Golden cases shared by make_golden.py (which runs the reference's own torch
code on them) and tests/test_oracle_golden.py (which runs the oracle on them).

Shapes are reduced so the stored outputs stay small; the structure (GQA 3:1,
head_dim 64, SwiGLU, half-split RoPE) is the reference's.  ``consts`` are the
module-level constants the reference classes read.
"""
from __future__ import annotations

import torch

from vla_b200 import weights as W
from vla_b200.configs import ExpertCfg, TextCfg, VisionCfg

TEXT_CONSTS = dict(SEQ=24, EMBD=192, Q_H=6, KV_H=2, HEAD_DIM=64, FFN_HID=320, BATCH=1)
EXP_CONSTS = dict(SEQ=20, TEXT_SEQ=24, EMBD=144, Q_H=6, KV_H=2, HEAD_DIM=64, KV_DIM=128, FFN_HID=256, BATCH=1)
LLAMA_CONSTS = dict(SEQ=20, EMBD=128, Q_H=6, KV_H=2, HEAD_DIM=64, FFN_HID=512, BATCH=1)
VIT_CONSTS = dict(SEQ=40, EMBD=128, N_HEAD=2, HEAD_DIM=64, FFN_HID=512, BATCH=1)

TEXT_CFG = TextCfg(hidden=192, heads=6, kv_heads=2, head_dim=64, ffn=320)
EXP_CFG = ExpertCfg(hidden=144, heads=6, kv_heads=2, head_dim=64, ffn=256)
LLAMA_CFG = TextCfg(hidden=128, heads=6, kv_heads=2, head_dim=64, ffn=512, eps=1e-5, rope_theta=1e4)
VIT_CFG = VisionCfg(hidden=128, heads=2, head_dim=64, ffn=512)

CASES = {
    # reference class exactly as written: RoPE base 1e4, RMSNorm eps = dtype epsilon
    "text_ref": dict(kind="text", consts=TEXT_CONSTS),
    # benchmark C0 hyper-parameters patched onto the reference class
    "text_c0": dict(kind="text", consts=TEXT_CONSTS, patch={"ln_1.eps": 1e-5, "ln_2.eps": 1e-5}, rope_theta=1e5),
    "exp_self": dict(kind="expert_self", consts=EXP_CONSTS, patch={"ln_1.eps": 1e-5, "ln_2.eps": 1e-5}),
    "exp_cross": dict(kind="expert_cross", consts=EXP_CONSTS, patch={"ln_1.eps": 1e-5, "ln_2.eps": 1e-5}),
    "minivit": dict(kind="minivit", consts=VIT_CONSTS),
    # vla/llama_block_rope_bf16.py: the torch twin of llama_block_rope (AttentionExpertBlock)
    # and the external-context block (CrossAttentionBlock)
    "llama_rope": dict(kind="llama_rope", consts=LLAMA_CONSTS, patch={"ln_1.eps": 1e-5, "ln_2.eps": 1e-5}),
    "cross_attn": dict(kind="cross_attn", consts=LLAMA_CONSTS, patch={"ln_1.eps": 1e-5, "ln_2.eps": 1e-5}),
    "siglip_emb": dict(kind="siglip_emb", consts=dict(EMBED=128, IMAGE=64, PATCH=16)),
    "con_ref": dict(kind="con_ref", consts={}),
    "masked_softmax_cpu": dict(kind="masked_softmax_cpu", consts=dict(SEQ=32)),
    # simulation/pusht_env.py module constants
    "pusht": dict(kind="pusht", consts=dict(WORKSPACE=512, EE_RADIUS=15, BLOCK_W=80, BLOCK_H=30, PUSH_COEFF=0.15,
                                            FRICTION=0.7)),
}

SEED = 1234


def case_inputs(name: str) -> dict:
    kind = CASES[name]["kind"]
    if kind == "text":
        c = TEXT_CONSTS
        p = W.text_block_params(TEXT_CFG, seed=SEED)
        x = W.randn((1, c["SEQ"], c["EMBD"]), SEED, "golden.text.x", dtype=torch.float32)
        return {"params": p, "args": [x]}
    if kind == "expert_self":
        c = EXP_CONSTS
        p = W.expert_self_params(EXP_CFG, seed=SEED)
        x = W.randn((1, c["SEQ"], c["EMBD"]), SEED, "golden.exp.x", dtype=torch.float32)
        return {"params": p, "args": [x]}
    if kind == "expert_cross":
        c = EXP_CONSTS
        p = W.expert_cross_params(EXP_CFG, text_kv_dim=c["KV_DIM"], seed=SEED, layer=1)
        x = W.randn((1, c["SEQ"], c["EMBD"]), SEED, "golden.exp.x", dtype=torch.float32)
        tk = W.randn((1, c["TEXT_SEQ"], c["KV_DIM"]), SEED, "golden.exp.tk", dtype=torch.float32)
        tv = W.randn((1, c["TEXT_SEQ"], c["KV_DIM"]), SEED, "golden.exp.tv", dtype=torch.float32)
        return {"params": p, "args": [x, tk, tv]}
    if kind in ("llama_rope", "cross_attn"):
        c = LLAMA_CONSTS
        p = W.text_block_params(LLAMA_CFG, seed=SEED, layer=7)
        x = W.randn((1, c["SEQ"], c["EMBD"]), SEED, "golden.llama.x", dtype=torch.float32)
        if kind == "llama_rope":
            return {"params": p, "args": [x]}
        ctx = W.randn((1, 24, c["EMBD"]), SEED, "golden.llama.ctx", dtype=torch.float32)
        return {"params": p, "args": [x, ctx]}
    if kind == "minivit":
        c = VIT_CONSTS
        p = W.vision_block_params(VIT_CFG, seed=SEED)
        x = W.randn((1, c["SEQ"], c["EMBD"]), SEED, "golden.vit.x", dtype=torch.float32)
        return {"params": p, "args": [x]}
    if kind == "siglip_emb":
        cfg = VisionCfg(hidden=128, image=64, patch=16)
        p = W.patch_embed_params(cfg, seed=SEED)
        p = dict(p, b_patch=W.randn((cfg.hidden,), SEED, "golden.patch.b", std=0.01))
        img = W.uniform((1, 3, 64, 64), SEED, "golden.img", -1.0, 1.0, dtype=torch.float32)
        return {"params": p, "args": [img]}
    if kind == "con_ref":
        x = W.randn((1024, 768), SEED, "golden.con.x")
        w = W.randn((12288, 960), SEED, "golden.con.W", std=0.02)
        return {"params": {"W": w}, "x": x}
    if kind == "pusht":
        return {"params": {}, "seeds": [0, 3, 99], "steps": 150}
    if kind == "masked_softmax_cpu":
        x = W.randn((32, 32), SEED, "golden.msm.x", std=2.0)
        return {"params": {}, "x": x}
    raise ValueError(kind)
