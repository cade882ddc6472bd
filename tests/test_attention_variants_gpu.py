"""The attention kernels' environment-selected variants, run in child processes
(the switches are read once per process): the pipelined short attention with two
softmax warpgroups instead of four (VLA_ATTN_PIPE_GROUPS=2) must give the same
bits, since every query row runs the same arithmetic in either assignment of
M-tiles to groups; the SigLIP attention with every exponential on MUFU.EX2 and
its P.V products issued by the S issuers (VLA_ATTN_POLY8=0, VLA_ATTN_PV_WARP=0)
must agree with the default, which takes a quarter of them
from the FMA-pipe polynomial, within the kernels' test tolerance, and both must
match the fp32 oracle."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Runs the three attention shapes on seeded inputs and saves the outputs (and the
# inputs, for the oracle) to argv[1].
CHILD = r"""
import os, sys
root = sys.argv[2]
sys.path[:0] = [root, os.path.join(root, "vla-to-npu_b200")]
import torch
from vla_b200 import _lib, device as dev
torch.manual_seed(7)
BF = torch.bfloat16
out = {}
def run(name, B, Lq, Lk, Hq, Hkv, causal, kv_len, impl):
    q = torch.randn(B * Lq, Hq * 64).to(BF).cuda()
    k = torch.randn(B * Lk, Hkv * 64).to(BF).cuda()
    v = torch.randn(B * Lk, Hkv * 64).to(BF).cuda()
    o = torch.full((B * Lq, Hq * 64), float("nan"), dtype=BF, device="cuda")
    kl = None if kv_len is None else torch.tensor(kv_len, dtype=torch.int32, device="cuda")
    dev.attention(q, k, v, o, batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64,
                  k_batch=Lk * Hkv * 64, v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, causal=causal,
                  kv_len=kl, impl=impl)
    dev.sync_check()
    out[name] = dict(q=q.cpu(), k=k.cpu(), v=v.cpu(), o=o.cpu())
run("self", 6, 50, 50, 15, 5, True, None, _lib.ATTN_TCGEN05_PIPE)
run("cross", 4, 50, 113, 15, 5, False, [113, 97, 64, 1], _lib.ATTN_TCGEN05_PIPE)
run("text", 2, 113, 113, 15, 5, True, None, _lib.ATTN_TCGEN05_PIPE)
run("siglip", 2, 1024, 1024, 12, 12, False, None, _lib.ATTN_TCGEN05)
torch.save(out, sys.argv[1])
"""


def _child(path, **env):
    # the switches the parent may carry are dropped: the first child is the default
    e = {k: v for k, v in os.environ.items() if not k.startswith("VLA_ATTN_")}
    e.update(env)
    subprocess.run([sys.executable, "-c", CHILD, str(path), ROOT], env=e, check=True, timeout=600)
    return torch.load(path)


def test_attention_env_variants(cuda, tmp_path):
    from oracle import smolvla_ref as R
    base = _child(tmp_path / "default.pt")
    alt = _child(tmp_path / "variant.pt", VLA_ATTN_PIPE_GROUPS="2", VLA_ATTN_POLY8="0", VLA_ATTN_PV_WARP="0")
    for name in ("self", "cross", "text"):
        assert torch.equal(base[name]["o"], alt[name]["o"]), f"{name}: two softmax groups changed the bits"
    s = base["siglip"]
    B, L, H = 2, 1024, 12
    ref = R.attention(s["q"].view(B, L, H, 64), s["k"].view(B, L, H, 64), s["v"].view(B, L, H, 64),
                      causal=False, dt=torch.float32).reshape(B * L, -1)
    for run in (base, alt):
        torch.testing.assert_close(run["siglip"]["o"].float(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(base["siglip"]["o"].float(), alt["siglip"]["o"].float(), atol=2e-2, rtol=2e-2)
