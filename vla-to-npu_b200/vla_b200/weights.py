"""Seeded synthetic weights and inputs for the SmolVLA hot path.

Real SmolVLA checkpoints are not available, so every benchmark and parity
test runs on random weights drawn here, N(0, 0.02) for matrices, N(0, 0.01)
for biases, ones for norm gains (the benchmark configurations).  Parameters
come back as bf16 CPU tensors in the reference's layout: linear weights are
[in_features, out_features] (reference: ``params["Wq"] = W.T``,
vla/text_encoder_bf16.py:602), norm gains are vectors, and the dictionary keys
are the reference's (``Wq, Wk, Wv, Wo, W_gate, W_up, W_down, W_norm_1,
W_norm_2, Wk_cross, Wv_cross, b_norm_*, W, kernel, W_exp_norm, W_action_out``).

Each tensor is drawn from its own generator, seeded from (seed, name, layer),
so a tensor does not depend on which other tensors were drawn before it.
"""
from __future__ import annotations

import zlib
from typing import Dict

import torch

from .configs import ExpertCfg, PrefixCfg, SmolVLACfg, TextCfg, VisionCfg

BF16 = torch.bfloat16


def _gen(seed: int, name: str, layer: int = 0) -> torch.Generator:
    s = (seed * 1_000_003 + zlib.crc32(name.encode()) * 7919 + layer * 104_729) % (2**63 - 1)
    return torch.Generator(device="cpu").manual_seed(s)


def randn(shape, seed: int, name: str, layer: int = 0, std: float = 1.0, dtype=BF16) -> torch.Tensor:
    t = torch.randn(*shape, generator=_gen(seed, name, layer), dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


def uniform(shape, seed: int, name: str, lo: float, hi: float, layer: int = 0, dtype=BF16) -> torch.Tensor:
    t = torch.rand(*shape, generator=_gen(seed, name, layer), dtype=torch.float32)
    return (t * (hi - lo) + lo).to(dtype)


def _w(shape, seed, name, layer, std=0.02):
    return randn(shape, seed, name, layer, std=std)


def text_block_params(cfg: TextCfg = TextCfg(), seed: int = 0, layer: int = 0) -> Dict[str, torch.Tensor]:
    H, Q, KV, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn
    p = {
        "Wq": _w((H, Q), seed, "text.Wq", layer),
        "Wk": _w((H, KV), seed, "text.Wk", layer),
        "Wv": _w((H, KV), seed, "text.Wv", layer),
        "Wo": _w((Q, H), seed, "text.Wo", layer),
        "W_gate": _w((H, F), seed, "text.W_gate", layer),
        "W_up": _w((H, F), seed, "text.W_up", layer),
        "W_down": _w((F, H), seed, "text.W_down", layer),
        "W_norm_1": torch.ones(H, dtype=BF16),
        "W_norm_2": torch.ones(H, dtype=BF16),
    }
    return p


def vision_block_params(cfg: VisionCfg = VisionCfg(), seed: int = 0, layer: int = 0) -> Dict[str, torch.Tensor]:
    H, F = cfg.hidden, cfg.ffn
    p = {
        "Wq": _w((H, H), seed, "vis.Wq", layer),
        "Wk": _w((H, H), seed, "vis.Wk", layer),
        "Wv": _w((H, H), seed, "vis.Wv", layer),
        "Wo": _w((H, H), seed, "vis.Wo", layer),
        "W_up": _w((H, F), seed, "vis.W_up", layer),
        "W_down": _w((F, H), seed, "vis.W_down", layer),
        "bq": _w((H,), seed, "vis.bq", layer, 0.01),
        "bk": _w((H,), seed, "vis.bk", layer, 0.01),
        "bv": _w((H,), seed, "vis.bv", layer, 0.01),
        "bo": _w((H,), seed, "vis.bo", layer, 0.01),
        "b_up": _w((F,), seed, "vis.b_up", layer, 0.01),
        "b_down": _w((H,), seed, "vis.b_down", layer, 0.01),
        "W_norm_1": torch.ones(H, dtype=BF16),
        "b_norm_1": torch.zeros(H, dtype=BF16),
        "W_norm_2": torch.ones(H, dtype=BF16),
        "b_norm_2": torch.zeros(H, dtype=BF16),
    }
    return p


def patch_embed_params(cfg: VisionCfg = VisionCfg(), seed: int = 0) -> Dict[str, torch.Tensor]:
    return {
        # conv weight [out, in, kh, kw] as in the reference's params["kernel"] (vla/vla.py:401)
        "kernel": _w((cfg.hidden, cfg.channels, cfg.patch, cfg.patch), seed, "vis.patch", 0),
        "b_patch": torch.zeros(cfg.hidden, dtype=BF16),  # C2 states no conv bias
        "pos_emb": _w((cfg.tokens, cfg.hidden), seed, "vis.pos", 0),
        "W_post_norm": torch.ones(cfg.hidden, dtype=BF16),
        "b_post_norm": torch.zeros(cfg.hidden, dtype=BF16),
    }


def connector_params(cfg: SmolVLACfg = SmolVLACfg(), seed: int = 0) -> Dict[str, torch.Tensor]:
    k = cfg.vision.hidden * cfg.connector.scale ** 2
    return {"W": _w((k, cfg.connector.out), seed, "connector.W", 0)}


def expert_self_params(cfg: ExpertCfg = ExpertCfg(), seed: int = 0, layer: int = 0) -> Dict[str, torch.Tensor]:
    H, Q, KV, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn
    return {
        "Wq": _w((H, Q), seed, "exp.Wq", layer),
        "Wk": _w((H, KV), seed, "exp.Wk", layer),
        "Wv": _w((H, KV), seed, "exp.Wv", layer),
        "Wo": _w((Q, H), seed, "exp.Wo", layer),
        "W_gate": _w((H, F), seed, "exp.W_gate", layer),
        "W_up": _w((H, F), seed, "exp.W_up", layer),
        "W_down": _w((F, H), seed, "exp.W_down", layer),
        "W_norm_1": torch.ones(H, dtype=BF16),
        "W_norm_2": torch.ones(H, dtype=BF16),
    }


def expert_cross_params(cfg: ExpertCfg = ExpertCfg(), text_kv_dim: int = 320, seed: int = 0,
                        layer: int = 0) -> Dict[str, torch.Tensor]:
    H, Q, KV, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn
    return {
        "Wq": _w((H, Q), seed, "exp.Wq", layer),
        "Wk_cross": _w((text_kv_dim, KV), seed, "exp.Wk_cross", layer),
        "Wv_cross": _w((text_kv_dim, KV), seed, "exp.Wv_cross", layer),
        "Wo": _w((Q, H), seed, "exp.Wo", layer),
        "W_gate": _w((H, F), seed, "exp.W_gate", layer),
        "W_up": _w((H, F), seed, "exp.W_up", layer),
        "W_down": _w((F, H), seed, "exp.W_down", layer),
        "W_norm_1": torch.ones(H, dtype=BF16),
        "W_norm_2": torch.ones(H, dtype=BF16),
    }


def smolvla_params(cfg: SmolVLACfg = SmolVLACfg(), seed: int = 0) -> dict:
    """Every weight of the full model, grouped by stage."""
    t, v, e, pf = cfg.text, cfg.vision, cfg.expert, cfg.prefix
    return {
        "patch": patch_embed_params(v, seed),
        "vision": [vision_block_params(v, seed, i) for i in range(v.layers)],
        "connector": connector_params(cfg, seed),
        "embed": _w((pf.vocab, t.hidden), seed, "text.embed", 0, std=1.0 / (t.hidden ** 0.5)),
        "W_state": _w((pf.state_dim, t.hidden), seed, "state.W", 0),
        "text": [text_block_params(t, seed, i) for i in range(t.layers)],
        "expert": [
            expert_self_params(e, seed, i) if i % 2 == 0 else expert_cross_params(e, t.kv_dim, seed, i)
            for i in range(e.layers)
        ],
        "W_action_in": _w((e.action_dim, e.hidden), seed, "exp.W_action_in", 0),
        "W_exp_norm": torch.ones(e.hidden, dtype=BF16),
        "W_action_out": _w((e.hidden, e.action_dim), seed, "exp.W_action_out", 0),
    }


def observation_batch(cfg: SmolVLACfg, batch: int, seed: int = 1) -> dict:
    """Synthetic observations: image U(-1, 1), token ids U[0, vocab),
    state N(0, 1), and the flow-matching start noise x0 ~ N(0, 1)."""
    v, pf, e = cfg.vision, cfg.prefix, cfg.expert
    g = _gen(seed, "obs.ids")
    return {
        "images": uniform((batch, v.channels, v.image, v.image), seed, "obs.image", -1.0, 1.0),
        "token_ids": torch.randint(0, pf.vocab, (batch, pf.text_tokens), generator=g, dtype=torch.int64).to(torch.int32),
        "state": randn((batch, pf.state_dim), seed, "obs.state"),
        "noise": randn((batch, e.chunk, e.action_dim), seed, "obs.noise", dtype=torch.float32),
    }
