"""Parity metrics shared by the GPU tests.

The acceptance rule (benchmark north star): against the fp32 oracle on
identical seeded inputs, the CUDA path's max-abs and relative-L2 errors must be
no worse than those of the reference's own bf16 path (the oracle run with
dt=bfloat16), up to a small slack for rounding-order noise, and the result
must also pass the reference's own block gate (atol = rtol = 1e-1,
vla/text_encoder_bf16.py:627-629).
"""
from __future__ import annotations

import torch

SLACK_REL = 1.10   # ours may exceed the reference bf16 path's error by 10 %
SLACK_ABS = 1e-3   # ... plus this absolute allowance for near-exact cases


def errors(x: torch.Tensor, ref: torch.Tensor):
    x = x.detach().float().cpu()
    ref = ref.detach().float().cpu()
    d = x - ref
    max_abs = d.abs().max().item()
    rel_l2 = (d.norm() / ref.norm().clamp_min(1e-30)).item()
    return max_abs, rel_l2


def check(ours: torch.Tensor, ref32: torch.Tensor, ref_bf16: torch.Tensor, name: str = "", gate_tol: float = 1e-1,
          slack_rel: float = SLACK_REL, slack_abs: float = SLACK_ABS) -> dict:
    ours_abs, ours_rel = errors(ours, ref32)
    bf_abs, bf_rel = errors(ref_bf16, ref32)
    rep = dict(name=name, ours_max_abs=ours_abs, ours_rel_l2=ours_rel, refbf16_max_abs=bf_abs, refbf16_rel_l2=bf_rel)
    print(f"[parity] {name}: ours max|d|={ours_abs:.4g} relL2={ours_rel:.4g} | reference-bf16 max|d|={bf_abs:.4g} "
          f"relL2={bf_rel:.4g}")
    assert ours_rel <= bf_rel * slack_rel + slack_abs, f"{name}: rel-L2 {ours_rel:.4g} worse than reference bf16 {bf_rel:.4g}"
    assert ours_abs <= bf_abs * slack_rel + slack_abs, f"{name}: max-abs {ours_abs:.4g} worse than reference bf16 {bf_abs:.4g}"
    torch.testing.assert_close(ours.detach().float().cpu(), ref32.detach().float().cpu(), atol=gate_tol, rtol=gate_tol)
    return rep
