"""Shape/hyper-parameter configurations of the SmolVLA hot path.

The numbers follow the benchmark configurations C0–C4 (text block, SigLIP
block, vision tower + connector, action expert, end-to-end).  Where they
differ from the reference's module-level constants, the reference value is
noted:

* text block: vla/text_encoder_bf16.py:43-49 (SEQ 128, EMBD 960, 15/5 heads,
  head_dim 64, FFN 2560); the reference RoPE base is 10,000
  (vla/text_encoder_bf16.py:79), C0 uses 100,000; the reference RMSNorm uses
  torch's dtype-epsilon default, C0 uses 1e-5.
* SigLIP block: vla/vision_block.py:4-30 (biases, LayerNorm eps 1e-6,
  GELU-tanh); the reference's bf16 oracle MiniVit (vla/vision_block_bf16.py:57-79)
  has zero biases, eps 1e-5 and erf-GELU.
* action expert: vla/action_expert_bf16.py:48-56 uses 32 tokens and width 768;
  C3 uses 50 tokens and width 720, 16 layers, 10 Euler steps.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class TextCfg:
    hidden: int = 960
    heads: int = 15
    kv_heads: int = 5
    head_dim: int = 64
    ffn: int = 2560
    eps: float = 1e-5
    rope_theta: float = 100_000.0
    layers: int = 16

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


@dataclass(frozen=True)
class VisionCfg:
    hidden: int = 768
    heads: int = 12
    head_dim: int = 64
    ffn: int = 3072
    eps: float = 1e-6
    layers: int = 12
    image: int = 512
    patch: int = 16
    channels: int = 3

    @property
    def grid(self) -> int:
        return self.image // self.patch

    @property
    def tokens(self) -> int:
        return self.grid * self.grid

    @property
    def patch_dim(self) -> int:
        return self.channels * self.patch * self.patch


@dataclass(frozen=True)
class ConnectorCfg:
    scale: int = 4
    out: int = 960


@dataclass(frozen=True)
class ExpertCfg:
    hidden: int = 720
    heads: int = 15
    kv_heads: int = 5
    head_dim: int = 64
    ffn: int = 2048
    eps: float = 1e-5
    rope_theta: float = 10_000.0
    layers: int = 16
    chunk: int = 50
    action_dim: int = 32
    steps: int = 10
    # sinusoidal time embedding periods (restated from the SmolVLA paper's
    # flow-matching head: log-spaced periods between these bounds)
    min_period: float = 4e-3
    max_period: float = 4.0

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


@dataclass(frozen=True)
class PrefixCfg:
    image_tokens: int = 64
    text_tokens: int = 48
    state_tokens: int = 1
    vocab: int = 49152
    state_dim: int = 32
    embed_scale_sqrt_hidden: bool = True  # reference: lang_emb * sqrt(hidden) (vla/vla.py:173)

    @property
    def length(self) -> int:
        return self.image_tokens + self.text_tokens + self.state_tokens


@dataclass(frozen=True)
class SmolVLACfg:
    text: TextCfg = field(default_factory=TextCfg)
    vision: VisionCfg = field(default_factory=VisionCfg)
    connector: ConnectorCfg = field(default_factory=ConnectorCfg)
    expert: ExpertCfg = field(default_factory=ExpertCfg)
    prefix: PrefixCfg = field(default_factory=PrefixCfg)


def tiny_cfg() -> SmolVLACfg:
    """A scaled-down model with the same structure, for fast parity tests.

    Head dim stays 64 and every width keeps the kernels' alignment rules."""
    return SmolVLACfg(
        text=TextCfg(hidden=192, heads=6, kv_heads=2, head_dim=64, ffn=320, layers=4),
        vision=VisionCfg(hidden=128, heads=2, head_dim=64, ffn=256, layers=2, image=128, patch=16),
        connector=ConnectorCfg(scale=4, out=192),
        expert=ExpertCfg(hidden=144, heads=6, kv_heads=2, head_dim=64, ffn=256, layers=4, chunk=50, steps=3),
        prefix=PrefixCfg(image_tokens=4, text_tokens=12, state_tokens=1, vocab=1000, state_dim=32),
    )
