"""tcgen05 GEMM parity against a plain fp32 torch matmul of the same bf16
operands (the reference GEMM tests compare against numpy A@B with
atol=1e-1, rtol=1e-2: gemm/v1_test_tiled_gemm.py:147-156)."""
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
