"""tcgen05 GEMM parity against a plain fp32 torch matmul of the same bf16
operands (the reference GEMM tests compare against numpy A@B with
atol=1e-1, rtol=1e-2: gemm/v1_test_tiled_gemm.py:147-156)."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, w_t):
    return a.float() @ w_t.float().T


@pytest.mark.parametrize("tile_n", [32, 64, 96, 128, 160, 192, 224, 256])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 960, 960), (50, 720, 720), (1024, 768, 768), (113, 1600, 960)])
def test_gemm_plain(cuda, tile_n, M, N, K):
    from vla_b200 import device as dev
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dev.gemm(a, w, out, tile_n=tile_n)
    dev.sync_check()
    ref = _ref(a, w)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


def test_gemm_k_tail_small(cuda):
    from vla_b200 import device as dev
    g = torch.Generator().manual_seed(1)
    for (M, N, K) in [(50, 720, 32), (64, 32, 720), (7, 16, 8)]:
        a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
        w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
        out = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
        dev.gemm(a, w, out)
        dev.sync_check()
        torch.testing.assert_close(out.float(), _ref(a, w), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("N", [16, 48, 80, 720, 208])
def test_gemm_16_column_tails(cuda, N):
    """N % 32 == 16: the last 16 columns of each row.  The output buffer has guard
    columns that must stay untouched, and the residual row ends exactly at N."""
    from vla_b200 import device as dev
    g = torch.Generator().manual_seed(N)
    M, K = 77, 96
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    res = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    bias = torch.randn(N, generator=g).to(torch.bfloat16).cuda()
    for tile_n in (32, 96, 192):
        buf = torch.full((M, N + 16), 7.0, dtype=torch.bfloat16, device="cuda")
        out = buf[:, :N]
        dev.gemm(a, w, out, dev.make_epilogue(bias=bias, residual=res), tile_n=tile_n)
        dev.sync_check()
        ref = a.float() @ w.float().T + bias.float() + res.float()
        torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
        assert (buf[:, N:] == 7.0).all(), "columns beyond N were written"


@pytest.mark.parametrize("tile_n", [64, 96, 128, 160, 192, 224, 256])
@pytest.mark.parametrize("M,N,K", [(1024, 768, 768), (1000, 720, 720), (300, 1600, 960), (4096, 256, 64)])
def test_gemm_cta_pair(cuda, tile_n, M, N, K):
    """Two-CTA (cta_group::2) kernel: 256-row tiles split over a CTA pair, each CTA
    staging its own A rows and half of B; M tails leave part of (or all of) the
    second CTA's rows empty; bias + residual epilogue with a 16-column N tail."""
    from vla_b200 import device as dev
    g = torch.Generator().manual_seed(M + N + K + tile_n)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    bias = torch.randn(N, generator=g).to(torch.bfloat16).cuda()
    res = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dev.gemm(a, w, out, dev.make_epilogue(bias=bias, residual=res), tile_n=tile_n, ctas=2)
    dev.sync_check()
    ref = a.float() @ w.float().T + bias.float() + res.float()
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)


def test_gemm_cta_pair_epilogues(cuda):
    """GELU, SwiGLU, RoPE and row-scatter epilogues on the CTA-pair kernel."""
    import torch.nn.functional as F
    from oracle import smolvla_ref as R
    from vla_b200 import _lib, device as dev
    from vla_b200.model import interleave_gate_up, rope_table
    g = torch.Generator().manual_seed(5)
    M, K = 700, 192
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, K, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    out = torch.empty(M, 256, dtype=torch.bfloat16, device="cuda")
    dev.gemm(a.cuda(), w.cuda(), out, dev.make_epilogue(bias=b.cuda(), act=_lib.ACT_GELU_TANH), ctas=2)
    torch.testing.assert_close(out.float().cpu(), F.gelu(a.float() @ w.float().T + b.float(), approximate="tanh"),
                               atol=3e-2, rtol=2e-2)
    wg, wu = (torch.randn(K, 320, generator=g) * 0.05).to(torch.bfloat16), \
        (torch.randn(K, 320, generator=g) * 0.05).to(torch.bfloat16)
    out = torch.empty(M, 320, dtype=torch.bfloat16, device="cuda")
    dev.gemm(a.cuda(), interleave_gate_up(wg, wu, "cuda"), out, dev.make_epilogue(act=_lib.ACT_SWIGLU), ctas=2)
    torch.testing.assert_close(out.float().cpu(), F.silu(a.float() @ wg.float()) * (a.float() @ wu.float()),
                               atol=3e-2, rtol=2e-2)
    wq = (torch.randn(192, K, generator=g) * 0.05).to(torch.bfloat16)
    cs = rope_table(50, 64, 1e4).cuda()
    out = torch.empty(M, 192, dtype=torch.bfloat16, device="cuda")
    dev.gemm(a.cuda(), wq.cuda(), out, dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=50, rope_ncols=128),
             tile_n=64, ctas=2)
    y = a.float() @ wq.float().T
    pos = (torch.arange(M) % 50).float()
    rot = R.apply_rope(y[:, :128].reshape(M, 1, 2, 64), 1e4, positions=pos[:, None]).reshape(M, 128)
    torch.testing.assert_close(out.float().cpu(), torch.cat([rot, y[:, 128:]], 1), atol=3e-2, rtol=2e-2)
    out = torch.zeros(M // 7 * 9, 256, dtype=torch.bfloat16, device="cuda")
    dev.gemm(a.cuda(), w.cuda(), out, dev.make_epilogue(out_grp=7, out_grp_stride=9), ctas=2)
    o = out.view(M // 7, 9, 256).cpu()
    torch.testing.assert_close(o[:, :7].float(), (a.float() @ w.float().T).view(M // 7, 7, 256), atol=3e-2, rtol=2e-2)
    assert o[:, 7:].abs().sum() == 0
    dev.sync_check()


@pytest.mark.gpu
@pytest.mark.parametrize("ctas", [1, 2])
@pytest.mark.parametrize("tile_n", [64, 128, 192, 256])
def test_gemm_rope_tile_widths(cuda, tile_n, ctas):
    """RoPE epilogue (+bias, +residual) where a tile holds several heads and the
    rotated-column boundary (rope_ncols) falls inside a tile."""
    from oracle import smolvla_ref as R
    from vla_b200 import _lib, device as dev
    from vla_b200.model import rope_table
    g = torch.Generator().manual_seed(11)
    M, K, N, nrot, seq = 4200, 160, 448, 320, 50
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g).to(torch.bfloat16)
    cs = rope_table(seq, 64, 1e4).cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    dev.gemm(a.cuda(), w.cuda(), out, dev.make_epilogue(bias=b.cuda(), residual=r.cuda(), act=_lib.ACT_ROPE,
                                                        rope_cs=cs, rope_seq=seq, rope_ncols=nrot),
             tile_n=tile_n, ctas=ctas)
    y = a.float() @ w.float().T + b.float()
    pos = (torch.arange(M) % seq).float()
    rot = R.apply_rope(y[:, :nrot].reshape(M, 1, nrot // 64, 64), 1e4, positions=pos[:, None]).reshape(M, nrot)
    ref = torch.cat([rot, y[:, nrot:]], 1) + r.float()
    torch.testing.assert_close(out.float().cpu(), ref, atol=4e-2, rtol=2e-2)
    dev.sync_check()


@pytest.mark.parametrize("splits", [2, 3, 4, 8])
@pytest.mark.parametrize("tile_n", [32, 64, 128])
@pytest.mark.parametrize("M,N,K", [(50, 720, 2048), (113, 960, 2560), (7, 1600, 720), (300, 256, 960)])
def test_gemm_split_k(cuda, splits, tile_n, M, N, K):
    """K split over a cluster of CTAs, partial tiles summed through distributed
    shared memory: plain product (300 rows: several tiles per cluster in turn).
    Wider tiles leave room for fewer partial slots (64: 5 CTAs, 128: 2); larger
    splits are rejected."""
    from vla_b200 import _lib
    from vla_b200 import device as dev
    if splits > {32: 8, 64: 5, 128: 2}[tile_n]:
        a = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
        w = torch.zeros(N, K, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(_lib.VlaError):
            dev.gemm(a, w, torch.empty(M, N, dtype=torch.bfloat16, device="cuda"), tile_n=tile_n, splits=splits)
        return
    g = torch.Generator().manual_seed(M + N + K + splits)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dev.gemm(a, w, out, tile_n=tile_n, splits=splits)
    dev.sync_check()
    torch.testing.assert_close(out.float(), _ref(a, w), atol=3e-2, rtol=1e-2)


def test_gemm_split_k_epilogues(cuda):
    """Every fused epilogue behind the split-K reduction matches the same GEMM
    without the split (fp32 sums in another order: within a bf16 rounding)."""
    from vla_b200 import _lib
    from vla_b200 import device as dev
    from vla_b200.model import interleave_gate_up, rope_table
    g = torch.Generator().manual_seed(77)
    M, K = 50, 720
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    cases = []
    w = (torch.randn(720, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    res = torch.randn(M, 720, generator=g).to(torch.bfloat16).cuda()
    bias = (torch.randn(720, generator=g) * 0.1).to(torch.bfloat16).cuda()
    cases.append(("bias+gelu+residual", w, 720, lambda: dev.make_epilogue(bias=bias, act=_lib.ACT_GELU_TANH,
                                                                          residual=res)))
    wg, wu = (torch.randn(K, 2048, generator=g) * 0.05), (torch.randn(K, 2048, generator=g) * 0.05)
    wgu = interleave_gate_up(wg, wu, "cuda")
    cases.append(("swiglu", wgu, 2048, lambda: dev.make_epilogue(act=_lib.ACT_SWIGLU)))
    wq = (torch.randn(1600, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    cs = rope_table(50, 64, 1e4).cuda()
    cases.append(("rope", wq, 1600, lambda: dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=50,
                                                               rope_ncols=1280)))
    wo = (torch.randn(32, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    x0 = torch.randn(M, 32, generator=g).cuda()
    for name, wt, ncols, mk in cases:
        outs = []
        for splits in (1, 4):
            out = torch.full((M, ncols), float("nan"), dtype=torch.bfloat16, device="cuda")
            dev.gemm(a, wt, out, mk(), tile_n=32 if name != "rope" else 64, splits=splits)
            dev.sync_check()
            outs.append(out.float())
        torch.testing.assert_close(outs[1], outs[0], atol=2e-2, rtol=1e-2, msg=name)
    # Euler: x += dt * (a @ wo^T) in fp32, C = bf16(x)
    xs, cb = [], []
    for splits in (1, 4):
        x = x0.clone()
        c = torch.empty(M, 32, dtype=torch.bfloat16, device="cuda")
        dev.gemm(a, wo, c, dev.make_epilogue(act=_lib.ACT_EULER, euler_x=x, euler_dt=-0.1), tile_n=32, splits=splits)
        dev.sync_check()
        xs.append(x)
        cb.append(c.float())
    torch.testing.assert_close(xs[1], xs[0], atol=1e-3, rtol=1e-3)
    ref = x0 - 0.1 * (a.float() @ wo.float().T)
    torch.testing.assert_close(xs[1], ref, atol=2e-3, rtol=1e-3)


def test_gemm_split_k_rejects_bad_requests(cuda):
    from vla_b200 import _lib
    from vla_b200 import device as dev
    a = torch.zeros(50, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(50, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.VlaError):
        dev.gemm(a, w, out, tile_n=32, splits=9)
    with pytest.raises(_lib.VlaError):
        dev.gemm(a, w, out, tile_n=32, splits=4)  # 2 k-blocks cannot feed 4 CTAs
    with pytest.raises(_lib.VlaError):
        dev.gemm(a, w, out, tile_n=96, splits=2)


@pytest.mark.parametrize("M,N,K", [(50, 720, 2048), (64, 720, 960), (1, 736, 720), (50, 720, 256), (33, 208, 296),
                                   (50, 96, 1000), (17, 4096, 1088), (50, 1600, 720), (113, 960, 2560),
                                   (100, 736, 720), (128, 1600, 960)])
@pytest.mark.parametrize("epi", ["plain", "bias_res", "swiglu", "rope"])
def test_gemm_skinny(cuda, M, N, K, epi):
    """One row tile (M <= 64 with 64-row copies, M <= 128 with 128-row copies):
    four k-blocks per stage through k-slab TMA boxes (gemm_skinny.cuh),
    with partial last units and K tails that are not whole k-blocks.  Same bits as
    the one-k-block-per-stage kernel (tile width 96 is not a skinny width) and the
    fp32 product within the GEMM tolerance."""
    import torch.nn.functional as F
    from oracle import smolvla_ref as R
    from vla_b200 import _lib, device as dev
    from vla_b200.model import rope_table
    if (epi == "rope" and N % 64) or (epi == "swiglu" and N % 32):
        pytest.skip("RoPE needs N % 64 == 0, SwiGLU N % 32 == 0")
    g = torch.Generator().manual_seed(M * 131 + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    y = a.float() @ w.float().T
    skinny_tile, plain_tile = (64, 192) if epi == "rope" else (32, 96)
    if epi == "plain":
        e, ref, cols = None, y, N
    elif epi == "bias_res":
        b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g).to(torch.bfloat16)
        e, ref, cols = dev.make_epilogue(bias=b.cuda(), residual=r.cuda()), y + b.float() + r.float(), N
    elif epi == "swiglu":
        e, cols = dev.make_epilogue(act=_lib.ACT_SWIGLU), N // 2
        yy = y.view(M, N // 32, 2, 16)
        ref = (F.silu(yy[:, :, 0]) * yy[:, :, 1]).reshape(M, N // 2)
    else:
        cs = rope_table(50, 64, 1e4).cuda()
        nrot = N - 64 if N > 64 else N
        e = dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=50, rope_ncols=nrot)
        pos = (torch.arange(M) % 50).float()
        rot = R.apply_rope(y[:, :nrot].reshape(M, 1, nrot // 64, 64), 1e4, positions=pos[:, None]).reshape(M, nrot)
        ref, cols = torch.cat([rot, y[:, nrot:]], 1), N
    outs = []
    for tile in (skinny_tile, plain_tile):
        out = torch.full((M, cols), float("nan"), dtype=torch.bfloat16, device="cuda")
        dev.gemm(a.cuda(), w.cuda(), out, e, tile_n=tile)
        outs.append(out.cpu())
    dev.sync_check()
    torch.testing.assert_close(outs[0].float(), ref, atol=3e-2, rtol=2e-2)
    if M <= 64 and K > 256 and os.environ.get("VLA_GEMM_SKINNY_DUAL", "1") != "0":
        # two MMA-issuing threads sum the k-slab units into two fp32 accumulators
        # that the epilogue adds: another summation order, at most one bf16 ulp
        torch.testing.assert_close(outs[0].float(), outs[1].float(), rtol=2.0 ** -7, atol=1e-3)
    else:
        assert torch.equal(outs[0], outs[1]), "skinny and one-k-block-per-stage kernels differ"
