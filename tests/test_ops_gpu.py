"""Per-op CUDA kernels vs the oracle, at the reference harness shapes
(rms_norm/test_rms_norm_bf16.py, layer_norm/test_layer_bf16.py,
softmax_bf16/*, vla/tests/test_masked_softmax_128_bf16.py, gelu/, silu/,
vla/test_rope_fused.py, vla/test_pixel_shuffle.py) and the benchmark shapes."""
import pytest
import torch
import torch.nn.functional as F

from oracle import smolvla_ref as R

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _rand(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(BF)


@pytest.mark.parametrize("M,N", [(16, 960), (128, 960), (50, 720), (7, 768), (3, 4096), (33, 2048)])
def test_rms_norm(cuda, M, N):
    from vla_b200 import device as dev
    x = _rand((M, N), M + N)
    g = _rand((N,), 7, 0.5) + 1
    y = dev.rms_norm(x.cuda(), g.cuda(), 1e-5)
    ref = R.rms_norm(x, g, 1e-5, torch.float32)
    # reference gate for the RMSNorm kernels: rtol 2e-2, atol 1e-1 (vla/tests/test_rms_norm_960_bf16.py:355)
    torch.testing.assert_close(y.float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("M,N", [(16, 768), (1024, 768), (5, 128), (9, 3072)])
def test_layer_norm(cuda, M, N):
    from vla_b200 import device as dev
    x = _rand((M, N), M * 3 + N) * 3 + 0.5
    g = _rand((N,), 1, 0.3) + 1
    b = _rand((N,), 2, 0.1)
    y = dev.layer_norm(x.cuda(), g.cuda(), b.cuda(), 1e-6)
    ref = R.layer_norm(x, g, b, 1e-6, torch.float32)
    torch.testing.assert_close(y.float().cpu(), ref, atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("L,heads,theta", [(128, 15, 1e5), (64, 5, 1e4), (50, 15, 1e4), (113, 20, 1e5)])
def test_rope(cuda, L, heads, theta):
    from vla_b200 import device as dev
    from vla_b200.model import rope_table
    x = _rand((L, heads * 64), L + heads)
    cs = rope_table(L, 64, theta).cuda()
    y = dev.rope_(x.clone().cuda(), heads * 64, L, cs)
    ref = R.apply_rope(x.float().view(1, L, heads, 64), theta).view(L, heads * 64)
    # reference RoPE tolerance is rtol 1e-3 / atol 1e-4 in fp32 (vla/test_rope_fused.py:153); output here is bf16
    torch.testing.assert_close(y.float().cpu(), ref, atol=2e-2, rtol=1e-2)


def test_rope_table_c_matches_torch(cuda):
    import ctypes
    from vla_b200 import _lib
    from vla_b200.model import rope_table
    t = torch.empty(113, 64, dtype=torch.float32)
    _lib.call("vla_rope_table", ctypes.c_void_p(t.data_ptr()), 113, 64, 1e5)
    torch.testing.assert_close(t, rope_table(113, 64, 1e5), atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("rows,cols,row_start", [(8, 128, 0), (8, 128, 96), (32, 128, -1), (4, 1024, -1), (32, 32, 0)])
def test_softmax(cuda, rows, cols, row_start):
    from vla_b200 import device as dev
    s = _rand((rows, cols), rows + cols, 2.0)
    y = dev.softmax(s.cuda(), 1.0, row_start).float().cpu()
    sf = s.float()
    if row_start >= 0:
        mask = torch.arange(cols)[None, :] > (row_start + torch.arange(rows))[:, None]
        sf = sf.masked_fill(mask, float("-inf"))
    ref = torch.softmax(sf, dim=-1)
    # masked_softmax_128 gate: rtol 5e-2, atol 5e-3 (vla/tests/test_masked_softmax_128_bf16.py:265)
    torch.testing.assert_close(y, ref, atol=5e-3, rtol=5e-2)


@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_elementwise(cuda, op):
    from vla_b200 import device as dev
    x = _rand((64, 2560), 3, 3.0)
    y = _rand((64, 2560), 4)
    out = dev.elementwise(op, x.cuda(), y.cuda() if op >= 2 else None).float().cpu()
    xf, yf = x.float(), y.float()
    ref = [F.gelu(xf, approximate="tanh"), F.silu(xf), F.silu(xf) * yf, xf + yf][op]
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("B,grid,scale,C", [(1, 32, 4, 768), (3, 8, 4, 128), (2, 16, 2, 64)])
def test_pixel_shuffle(cuda, B, grid, scale, C):
    from vla_b200 import device as dev
    x = _rand((B, grid * grid, C), B + grid)
    out = torch.empty(B * (grid // scale) ** 2, scale * scale * C, dtype=BF, device="cuda")
    dev.pixel_shuffle(x.reshape(-1, C).cuda(), B, grid, scale, out)
    ref = R.pixel_shuffle(x, grid, scale).reshape(out.shape)
    assert torch.equal(out.cpu(), ref)


def test_im2col_matches_conv(cuda):
    from vla_b200 import device as dev
    img = _rand((2, 3, 64, 48), 5)
    out = torch.empty(2 * 4 * 3, 3 * 16 * 16, dtype=BF, device="cuda")
    dev.patch_im2col(img.cuda(), 16, out)
    ref = F.unfold(img.float(), 16, stride=16).transpose(1, 2).reshape(out.shape)
    assert torch.equal(out.float().cpu(), ref)


def test_embed_gather(cuda):
    from vla_b200 import device as dev
    table = _rand((1000, 192), 9)
    ids = torch.randint(0, 1000, (3, 12), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    out = torch.zeros(3 * 17, 192, dtype=BF, device="cuda")
    dev.embed(ids.cuda(), table.cuda(), 2.0, out, 17, 4)
    o = out.view(3, 17, 192).cpu()
    ref = (table.float()[ids.long()] * 2.0).to(BF)
    assert torch.equal(o[:, 4:16], ref)
    assert o[:, :4].abs().sum() == 0 and o[:, 16:].abs().sum() == 0


@pytest.mark.parametrize("Lq,Lk,Hq,Hkv,causal,B", [
    (128, 128, 15, 5, True, 1),     # C0 text self-attention
    (113, 113, 15, 5, True, 3),     # C4 prefix (ragged tile)
    (1024, 1024, 12, 12, False, 1),  # C1 SigLIP
    (50, 50, 15, 5, True, 2),       # C3 expert self
    (50, 113, 15, 5, False, 2),     # C3 expert cross
    (1, 7, 2, 1, False, 1),
])
def test_attention(cuda, Lq, Lk, Hq, Hkv, causal, B):
    from vla_b200 import device as dev
    q = _rand((B, Lq, Hq, 64), 1)
    k = _rand((B, Lk, Hkv, 64), 2)
    v = _rand((B, Lk, Hkv, 64), 3)
    o = torch.empty(B * Lq, Hq * 64, dtype=BF, device="cuda")
    dev.attention(q.reshape(B * Lq, -1).cuda(), k.reshape(B * Lk, -1).cuda(), v.reshape(B * Lk, -1).cuda(), o,
                  batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64, k_batch=Lk * Hkv * 64,
                  v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, causal=causal)
    ref = R.attention(q, k, v, causal=causal, dt=torch.float32).reshape(B * Lq, -1)
    torch.testing.assert_close(o.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_attention_key_padding(cuda):
    from vla_b200 import device as dev
    B, Lq, Lk, Hq, Hkv = 3, 50, 128, 15, 5
    q, k, v = _rand((B, Lq, Hq, 64), 4), _rand((B, Lk, Hkv, 64), 5), _rand((B, Lk, Hkv, 64), 6)
    kv_len = torch.tensor([113, 1, 128], dtype=torch.int32)
    o = torch.empty(B * Lq, Hq * 64, dtype=BF, device="cuda")
    dev.attention(q.reshape(B * Lq, -1).cuda(), k.reshape(B * Lk, -1).cuda(), v.reshape(B * Lk, -1).cuda(), o,
                  batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64, k_batch=Lk * Hkv * 64,
                  v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, kv_len=kv_len.cuda())
    ref = R.attention(q, k, v, causal=False, kv_len=kv_len.tolist(), dt=torch.float32).reshape(B * Lq, -1)
    torch.testing.assert_close(o.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_gemm_epilogues(cuda):
    """bias / GELU / residual / SwiGLU / RoPE / Euler / row-scatter epilogues vs fp32 torch."""
    from vla_b200 import _lib, device as dev
    from vla_b200.model import interleave_gate_up, rope_table
    M, K = 200, 192
    a = _rand((M, K), 11)
    # bias + GELU + residual
    w = _rand((256, K), 12, 0.05)
    bias, res = _rand((256,), 13, 0.1), _rand((M, 256), 14)
    out = torch.empty(M, 256, dtype=BF, device="cuda")
    dev.gemm(a.cuda(), w.cuda(), out, dev.make_epilogue(bias=bias.cuda(), act=_lib.ACT_GELU_TANH,
                                                         residual=res.cuda()))
    ref = F.gelu(a.float() @ w.float().T + bias.float(), approximate="tanh") + res.float()
    torch.testing.assert_close(out.float().cpu(), ref, atol=3e-2, rtol=2e-2)
    # SwiGLU with interleaved weights
    wg, wu = _rand((K, 320), 15, 0.05), _rand((K, 320), 16, 0.05)
    wgu = interleave_gate_up(wg, wu, "cuda")
    out = torch.empty(M, 320, dtype=BF, device="cuda")
    dev.gemm(a.cuda(), wgu, out, dev.make_epilogue(act=_lib.ACT_SWIGLU))
    ref = F.silu(a.float() @ wg.float()) * (a.float() @ wu.float())
    torch.testing.assert_close(out.float().cpu(), ref, atol=3e-2, rtol=2e-2)
    # RoPE on the first 2 of 3 heads, positions m % 50
    wq = _rand((192, K), 17, 0.05)
    cs = rope_table(50, 64, 1e4).cuda()
    out = torch.empty(M, 192, dtype=BF, device="cuda")
    dev.gemm(a.cuda(), wq.cuda(), out, dev.make_epilogue(act=_lib.ACT_ROPE, rope_cs=cs, rope_seq=50, rope_ncols=128))
    y = (a.float() @ wq.float().T)
    pos = torch.arange(M) % 50
    rot = R.apply_rope(y[:, :128].reshape(M, 1, 2, 64), 1e4, positions=pos[None, :].float().t()).reshape(M, 128)
    ref = torch.cat([rot, y[:, 128:]], dim=1)
    torch.testing.assert_close(out.float().cpu(), ref, atol=3e-2, rtol=2e-2)
    # Euler: x += dt * (a @ w^T), C = bf16(x)
    w32 = _rand((32, K), 18, 0.05)
    x = torch.randn(M, 32, generator=torch.Generator().manual_seed(19))
    xd = x.clone().cuda()
    out = torch.empty(M, 32, dtype=BF, device="cuda")
    dev.gemm(a.cuda(), w32.cuda(), out, dev.make_epilogue(act=_lib.ACT_EULER, euler_x=xd, euler_dt=-0.1))
    ref = x - 0.1 * (a.float() @ w32.float().T)
    torch.testing.assert_close(xd.cpu(), ref, atol=2e-3, rtol=1e-3)
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=1e-2)
    # output row scatter: rows of group g land at g*7 + r
    out = torch.zeros(M // 4 * 7, 256, dtype=BF, device="cuda")
    dev.gemm(a.cuda(), w.cuda(), out, dev.make_epilogue(out_grp=4, out_grp_stride=7))
    o = out.view(M // 4, 7, 256).cpu()
    ref = (a.float() @ w.float().T).view(M // 4, 4, 256)
    torch.testing.assert_close(o[:, :4].float(), ref, atol=3e-2, rtol=2e-2)
    assert o[:, 4:].abs().sum() == 0


def test_bad_arguments_raise(cuda):
    """Host-side validation: misaligned strides and bad shapes return errors, never launch."""
    from vla_b200 import _lib, device as dev
    a = torch.zeros(16, 60, dtype=BF, device="cuda")
    w = torch.zeros(16, 60, dtype=BF, device="cuda")
    out = torch.zeros(16, 16, dtype=BF, device="cuda")
    with pytest.raises(_lib.VlaError) as e:
        dev.gemm(a, w, out)  # lda 60 is not a multiple of 8
    assert e.value.code == _lib.VLA_E_ALIGN
    a = torch.zeros(16, 64, dtype=BF, device="cuda")
    w = torch.zeros(20, 64, dtype=BF, device="cuda")
    out = torch.zeros(16, 24, dtype=BF, device="cuda")
    with pytest.raises(_lib.VlaError) as e:
        dev.gemm(a, w, out[:, :20])  # N = 20 not a multiple of 16
    assert e.value.code == _lib.VLA_E_INVALID


@pytest.mark.parametrize("Lq,Lk,Hq,Hkv,B,kv_len", [
    (1024, 1024, 12, 12, 2, None),   # SigLIP (C1): 8 query tiles x 8 key tiles
    (200, 300, 4, 4, 2, None),       # ragged query and key tails
    (128, 256, 15, 5, 1, None),      # GQA 3:1
    (50, 113, 15, 5, 3, [113, 60, 1]),  # expert cross shape with key padding
])
def test_attention_tcgen05(cuda, Lq, Lk, Hq, Hkv, B, kv_len):
    """The tcgen05 flash-attention kernel (TMEM accumulators, P from smem, V as an
    MN-major operand) forced on, against the fp32 oracle."""
    from vla_b200 import _lib, device as dev
    q = _rand((B, Lq, Hq, 64), 21)
    k = _rand((B, Lk, Hkv, 64), 22)
    v = _rand((B, Lk, Hkv, 64), 23)
    o = torch.full((B * Lq, Hq * 64), float("nan"), dtype=BF, device="cuda")
    kl = None if kv_len is None else torch.tensor(kv_len, dtype=torch.int32, device="cuda")
    dev.attention(q.reshape(B * Lq, -1).cuda(), k.reshape(B * Lk, -1).cuda(), v.reshape(B * Lk, -1).cuda(), o,
                  batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64, k_batch=Lk * Hkv * 64,
                  v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, kv_len=kl, impl=_lib.ATTN_TCGEN05)
    dev.sync_check()
    ref = R.attention(q, k, v, causal=False, kv_len=kv_len, dt=torch.float32).reshape(B * Lq, -1)
    torch.testing.assert_close(o.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_attention_tcgen05_strided_qkv(cuda):
    """Q/K/V as column views of one fused QKV buffer (the SigLIP layer layout), more
    work items than SMs so each persistent CTA walks several items."""
    from vla_b200 import _lib, device as dev
    B, L, H = 20, 1024, 12
    qkv = _rand((B * L, 3 * H * 64), 24)
    qd = qkv.cuda()
    o = torch.empty(B * L, H * 64, dtype=BF, device="cuda")
    dev.attention(qd[:, :H * 64], qd[:, H * 64:2 * H * 64], qd[:, 2 * H * 64:], o, batch=B, Lq=L, Lk=L, Hq=H,
                  Hkv=H, q_batch=L * 3 * H * 64, k_batch=L * 3 * H * 64, v_batch=L * 3 * H * 64, o_batch=L * H * 64,
                  impl=_lib.ATTN_TCGEN05)
    dev.sync_check()
    x = qkv.view(B, L, 3, H, 64)
    for b in (0, B - 1):
        ref = R.attention(x[b:b + 1, :, 0], x[b:b + 1, :, 1], x[b:b + 1, :, 2], causal=False,
                          dt=torch.float32).reshape(L, -1)
        torch.testing.assert_close(o[b * L:(b + 1) * L].float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("Lq,Lk,Hq,Hkv,causal,B,kv_len", [
    (113, 113, 15, 5, True, 3, None),        # C4 prefix: 3 x 113 stacked rows, causal
    (128, 128, 15, 5, True, 1, None),        # C0 text: 384 stacked rows, 128 keys
    (50, 50, 15, 5, True, 2, None),          # C3 expert self: 64-key variant
    (50, 113, 15, 5, False, 3, [113, 60, 1]),  # C3 expert cross with key padding
    (50, 128, 15, 5, False, 2, [0, 128]),      # a sequence with no keys writes zeros
    (7, 33, 4, 2, False, 1, None),            # ragged: 14 stacked rows, 33 keys
    (300, 97, 2, 2, True, 2, None),           # one head per kv head, 3 row tiles
])
def test_attention_tcgen05_short(cuda, Lq, Lk, Hq, Hkv, causal, B, kv_len):
    """The short-sequence tcgen05 kernel (all keys in one tile, query heads of a
    kv head stacked into 128-row tiles) forced on, against the fp32 oracle."""
    from vla_b200 import _lib, device as dev
    q = _rand((B, Lq, Hq, 64), 31)
    k = _rand((B, Lk, Hkv, 64), 32)
    v = _rand((B, Lk, Hkv, 64), 33)
    o = torch.full((B * Lq, Hq * 64), float("nan"), dtype=BF, device="cuda")
    kl = None if kv_len is None else torch.tensor(kv_len, dtype=torch.int32, device="cuda")
    dev.attention(q.reshape(B * Lq, -1).cuda(), k.reshape(B * Lk, -1).cuda(), v.reshape(B * Lk, -1).cuda(), o,
                  batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64, k_batch=Lk * Hkv * 64,
                  v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, causal=causal, kv_len=kl,
                  impl=_lib.ATTN_TCGEN05_SHORT)
    dev.sync_check()
    ref = R.attention(q, k, v, causal=causal, kv_len=kv_len, dt=torch.float32).reshape(B * Lq, -1)
    if kv_len is not None and 0 in kv_len:
        ref = ref.view(B, Lq, -1)
        ref[[i for i, n in enumerate(kv_len) if n == 0]] = 0.0
        ref = ref.reshape(B * Lq, -1)
    torch.testing.assert_close(o.float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("Lq,Lk,Hq,Hkv,causal,B,kv_len", [
    (113, 113, 15, 5, True, 3, None),        # C4 prefix: 3 x 113 stacked rows, causal
    (128, 128, 15, 5, True, 1, None),        # C0 text: 384 stacked rows, 128 keys
    (50, 50, 15, 5, True, 2, None),          # C3 expert self: 64-key variant
    (50, 113, 15, 5, False, 3, [113, 60, 1]),  # C3 expert cross with key padding
    (50, 128, 15, 5, False, 2, [0, 128]),      # a sequence with no keys writes zeros
    (7, 33, 4, 2, False, 1, None),            # ragged: 14 stacked rows, 33 keys
    (200, 97, 2, 2, True, 2, None),           # one head per kv head, 4 row tiles (2 smem stages)
    (50, 50, 15, 5, True, 400, None),         # 2000 items: every CTA cycles its stages and TMEM slots
])
def test_attention_tcgen05_pipelined(cuda, Lq, Lk, Hq, Hkv, causal, B, kv_len):
    """The pipelined short-sequence kernel (TMA in and out, warp-specialised, items
    in flight) forced on, against the fp32 oracle."""
    from vla_b200 import _lib, device as dev
    q = _rand((B, Lq, Hq, 64), 41)
    k = _rand((B, Lk, Hkv, 64), 42)
    v = _rand((B, Lk, Hkv, 64), 43)
    o = torch.full((B * Lq, Hq * 64), float("nan"), dtype=BF, device="cuda")
    kl = None if kv_len is None else torch.tensor(kv_len, dtype=torch.int32, device="cuda")
    dev.attention(q.reshape(B * Lq, -1).cuda(), k.reshape(B * Lk, -1).cuda(), v.reshape(B * Lk, -1).cuda(), o,
                  batch=B, Lq=Lq, Lk=Lk, Hq=Hq, Hkv=Hkv, q_batch=Lq * Hq * 64, k_batch=Lk * Hkv * 64,
                  v_batch=Lk * Hkv * 64, o_batch=Lq * Hq * 64, causal=causal, kv_len=kl,
                  impl=_lib.ATTN_TCGEN05_PIPE)
    dev.sync_check()
    sel = slice(None) if B <= 8 else [0, 1, B // 2, B - 1]
    ref = R.attention(q[sel], k[sel], v[sel], causal=causal, kv_len=kv_len, dt=torch.float32)
    if kv_len is not None and 0 in kv_len:
        ref[[i for i, n in enumerate(kv_len) if n == 0]] = 0.0
    ours = o.view(B, Lq, -1)[sel].float().cpu()
    torch.testing.assert_close(ours, ref.reshape(ours.shape), atol=2e-2, rtol=2e-2)


def test_attention_tcgen05_pipelined_fused_qkv(cuda):
    """Q/K/V as column views of the layer's fused [rows, Q | K | V] buffer (the
    text / expert self-attention layout), output into a strided view; the result
    matches the mma.sync kernel on the same problem."""
    from vla_b200 import _lib, device as dev
    B, L, Hq, Hkv = 37, 113, 15, 5
    cols = (Hq + 2 * Hkv) * 64
    qkv = _rand((B * L, cols), 44).cuda()
    q, k, v = qkv[:, :Hq * 64], qkv[:, Hq * 64:(Hq + Hkv) * 64], qkv[:, (Hq + Hkv) * 64:]
    outs = {}
    for impl in (_lib.ATTN_TCGEN05_PIPE, _lib.ATTN_MMA_SYNC):
        buf = torch.full((B * L, Hq * 64 + 64), float("nan"), dtype=BF, device="cuda")
        o = buf[:, :Hq * 64]
        dev.attention(q, k, v, o, batch=B, Lq=L, Lk=L, Hq=Hq, Hkv=Hkv, q_batch=L * cols, k_batch=L * cols,
                      v_batch=L * cols, o_batch=L * (Hq * 64 + 64), causal=True, impl=impl)
        dev.sync_check()
        assert torch.isnan(buf[:, Hq * 64:]).all(), "the kernel wrote outside the output view"
        outs[impl] = o.float().cpu()
    torch.testing.assert_close(outs[_lib.ATTN_TCGEN05_PIPE], outs[_lib.ATTN_MMA_SYNC], atol=1e-2, rtol=1e-2)
    x = qkv.view(B, L, cols).cpu()
    for b in (0, B - 1):
        ref = R.attention(x[b:b + 1, :, :Hq * 64].view(1, L, Hq, 64), x[b:b + 1, :, Hq * 64:(Hq + Hkv) * 64].view(
            1, L, Hkv, 64), x[b:b + 1, :, (Hq + Hkv) * 64:].view(1, L, Hkv, 64), causal=True, dt=torch.float32)
        torch.testing.assert_close(outs[_lib.ATTN_TCGEN05_PIPE][b * L:(b + 1) * L], ref.reshape(L, -1), atol=2e-2,
                                   rtol=2e-2)


@pytest.mark.parametrize("B,H,W,S", [(2, 512, 512, 512), (3, 480, 640, 512), (1, 37, 50, 64), (2, 1024, 768, 128)])
def test_camera_preprocess(cuda, B, H, W, S):
    """uint8 HWC camera frames -> bilinear resize (half-pixel centres, no antialias)
    -> [-1, 1] bf16, as the NCHW image and fused with im2col into the patch GEMM
    operand, against torch's interpolate in fp32 on the same frames."""
    from vla_b200 import device as dev
    g = torch.Generator().manual_seed(51 + H)
    frames = torch.randint(0, 256, (B, H, W, 3), generator=g, dtype=torch.uint8)
    x = frames.permute(0, 3, 1, 2).float()
    ref = F.interpolate(x, size=(S, S), mode="bilinear", align_corners=False, antialias=False) * (2.0 / 255.0) - 1.0
    fd = frames.cuda()
    img = torch.empty(B, 3, S, S, dtype=BF, device="cuda")
    dev.camera_preprocess(fd, S, img)
    dev.sync_check()
    # one bf16 rounding of values in [-1, 1]: at most 2^-8 away
    torch.testing.assert_close(img.float().cpu(), ref, atol=2.0 ** -8 + 1e-5, rtol=0)
    if H == W == S:
        assert torch.equal(img.float().cpu(), (x * (2.0 / 255.0) - 1.0).to(BF).float()), "identity resize is exact"
    p = 16
    patches = torch.empty(B * (S // p) ** 2, 3 * p * p, dtype=BF, device="cuda")
    dev.camera_preprocess(fd, S, patches, patch=p)
    ref_patches = torch.empty_like(patches)
    dev.patch_im2col(img, p, ref_patches)
    dev.sync_check()
    assert torch.equal(patches, ref_patches), "fused im2col differs from resize + im2col"


def test_exp2_fma_error_bound(cuda):
    """The FMA-pipe exponential of the SigLIP attention softmax: relative error
    under 1e-4 against exact 2^x over the softmax's argument range (the kernel
    feeds x = s * scale - running max, at most +8 with the lazy rescale), values
    below 2^-126 (no NaN, no wrap-around) for x below -126 and for -inf."""
    import ctypes
    from vla_b200 import _lib
    lib = _lib.load()
    x = torch.cat([torch.linspace(-125.0, 8.0, 1 << 20, dtype=torch.float64),
                   torch.tensor([0.0, -0.0, 1.0, -1.0, 7.999, -1e-7, 1e-7], dtype=torch.float64)]).float().cuda()
    y = torch.empty_like(x)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.vla_test_exp2_fma(x.data_ptr(), y.data_ptr(), x.numel(), stream))
    torch.cuda.synchronize()
    exact = torch.exp2(x.double())
    rel = ((y.double() - exact) / exact).abs()
    assert rel.max().item() < 1e-4, rel.max().item()
    low = torch.tensor([-126.0, -126.5, -127.0, -200.0, -1e30, float("-inf")], device="cuda")
    yl = torch.empty_like(low)
    _lib.check(lib.vla_test_exp2_fma(low.data_ptr(), yl.data_ptr(), low.numel(), stream))
    torch.cuda.synchronize()
    assert torch.isfinite(yl).all() and (yl >= 0).all() and (yl < 2.0 ** -125).all(), yl.tolist()
