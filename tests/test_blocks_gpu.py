"""Block-level parity (benchmark configurations C0-C3) and the full pipeline
(C4 structure) against the oracle: the CUDA path's error versus the fp32 oracle
must not exceed the reference bf16 path's error (tests/parity.py)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import smolvla_ref as R
from parity import check
from vla_b200 import weights as W
from vla_b200.configs import ExpertCfg, SmolVLACfg, TextCfg, VisionCfg, tiny_cfg

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
F32 = torch.float32


def _x(shape, seed, name):
    return W.randn(shape, seed, name, dtype=F32)


@pytest.mark.parametrize("B,L", [(1, 128), (2, 113)])
def test_text_block_c0(cuda, B, L):
    from vla_b200 import device as dev
    from vla_b200.model import LlamaLayerWeights, rope_table
    cfg = TextCfg()
    p = W.text_block_params(cfg, seed=0)
    x = _x((B, L, cfg.hidden), 0, "c0.x").to(BF)
    o32, k32, v32 = R.text_block(x, p, cfg, dt=F32)
    obf, kbf, vbf = R.text_block(x, p, cfg, dt=BF)
    lw = LlamaLayerWeights(p, cfg, "cuda")
    xd = x.reshape(B * L, -1).cuda().contiguous()
    qkv = torch.empty(B * L, cfg.q_dim + 2 * cfg.kv_dim, dtype=BF, device="cuda")
    dev.llama_self_layer(lw.struct, xd, B, L, rope_table(L, 64, cfg.rope_theta).cuda(), dev.Workspace(), qkv_out=qkv)
    dev.sync_check()
    check(xd.view(B, L, -1), o32, obf, f"text block B={B} L={L} out")
    Q, KV = cfg.q_dim, cfg.kv_dim
    check(qkv[:, Q:Q + KV].reshape(B, L, -1), k32, kbf, "text block K (post-RoPE)")
    check(qkv[:, Q + KV:].reshape(B, L, -1), v32, vbf, "text block V")


def test_vision_block_c1(cuda):
    from vla_b200 import device as dev
    from vla_b200.model import VisionLayerWeights
    cfg = VisionCfg()
    p = W.vision_block_params(cfg, seed=0)
    x = _x((1, 1024, cfg.hidden), 0, "c1.x").to(BF)
    o32 = R.vision_block(x, p, cfg, dt=F32)
    obf = R.vision_block(x, p, cfg, dt=BF)
    lw = VisionLayerWeights(p, cfg, "cuda")
    xd = x.reshape(1024, -1).cuda().contiguous()
    dev.vision_layer(lw.struct, xd, 1, 1024, dev.Workspace())
    dev.sync_check()
    check(xd.view(1, 1024, -1), o32, obf, "SigLIP block C1")


@pytest.mark.parametrize("B", [1, 3])
def test_expert_blocks_c3(cuda, B):
    from vla_b200 import device as dev
    from vla_b200.model import LlamaLayerWeights, rope_table
    e, t = ExpertCfg(), TextCfg()
    ps = W.expert_self_params(e, seed=0, layer=0)
    pc = W.expert_cross_params(e, t.kv_dim, seed=0, layer=1)
    x = _x((B, e.chunk, e.hidden), 0, "c3.x").to(BF)
    tk = _x((B, 113, t.kv_dim), 0, "c3.tk").to(BF)
    tv = _x((B, 113, t.kv_dim), 0, "c3.tv").to(BF)
    cs = rope_table(e.chunk, 64, e.rope_theta).cuda()
    ws = dev.Workspace()
    # self layer
    s32 = R.expert_self_block(x, ps, e, dt=F32)
    sbf = R.expert_self_block(x, ps, e, dt=BF)
    lw = LlamaLayerWeights(ps, e, "cuda")
    xd = x.reshape(B * e.chunk, -1).cuda().contiguous()
    dev.llama_self_layer(lw.struct, xd, B, e.chunk, cs, ws)
    dev.sync_check()
    check(xd.view(B, e.chunk, -1), s32, sbf, f"expert self B={B}")
    # cross layer (K/V projections, then cross attention)
    kc32, vc32 = R.expert_cross_kv(tk, tv, pc, dt=F32)
    kcbf, vcbf = R.expert_cross_kv(tk, tv, pc, dt=BF)
    c32 = R.expert_cross_block(x, kc32, vc32, pc, e, dt=F32)
    cbf = R.expert_cross_block(x, kcbf, vcbf, pc, e, dt=BF)
    lw = LlamaLayerWeights(pc, e, "cuda", cross=True)
    kv = torch.empty(B * 113, 2 * e.kv_dim, dtype=BF, device="cuda")
    dev.gemm(tk.reshape(B * 113, -1).cuda(), lw.wk_cross, kv[:, :e.kv_dim])
    dev.gemm(tv.reshape(B * 113, -1).cuda(), lw.wv_cross, kv[:, e.kv_dim:])
    xd = x.reshape(B * e.chunk, -1).cuda().contiguous()
    dev.llama_cross_layer(lw.struct, xd, B, e.chunk, cs, kv[:, :e.kv_dim], kv[:, e.kv_dim:], 113, ws)
    dev.sync_check()
    check(xd.view(B, e.chunk, -1), c32, cbf, f"expert cross B={B}")


def _run_model(cfg, B, seed=0):
    from vla_b200.model import SmolVLA
    params = W.smolvla_params(cfg, seed=seed)
    obs = W.observation_batch(cfg, B, seed=seed + 1)
    m = SmolVLA(cfg, params, "cuda")
    out = m.infer(obs["images"].cuda(), obs["token_ids"].cuda(), obs["state"].cuda(), obs["noise"].cuda(),
                  use_graph=False).clone()
    out_graph = m.infer(obs["images"].cuda(), obs["token_ids"].cuda(), obs["state"].cuda(), obs["noise"].cuda(),
                        use_graph=True).clone()
    from vla_b200 import device as dev
    dev.sync_check()
    return params, obs, m, out, out_graph


def test_pipeline_tiny(cuda):
    """Whole action-chunk inference (vision, connector, prefix, text layers, 10-step
    expert) on the scaled-down model, eager and CUDA-graph replay."""
    cfg = tiny_cfg()
    params, obs, m, out, out_graph = _run_model(cfg, B=3)
    ref32 = R.smolvla_chunk(obs, params, cfg, dt=F32)
    refbf = R.smolvla_chunk(obs, params, cfg, dt=BF)
    check(out, ref32, refbf, "pipeline tiny (eager)")
    assert torch.equal(out, out_graph), "graph replay differs from eager launch"


def test_vision_tower_c2(cuda):
    """Patch embedding + 12 SigLIP layers + post-LN + pixel shuffle + connector (C2)."""
    from vla_b200.model import SmolVLA
    cfg = SmolVLACfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, 1, seed=1)
    m = SmolVLA(cfg, params, "cuda")
    m.load_inputs(obs["images"].cuda(), obs["token_ids"].cuda(), obs["state"].cuda(), obs["noise"].cuda())
    m.vision_tower()
    torch.cuda.synchronize()
    ours = m.prefix.view(1, cfg.prefix.length, -1)[:, :cfg.prefix.image_tokens]
    ref32 = R.vision_tower(obs["images"], params, cfg, dt=F32)
    refbf = R.vision_tower(obs["images"], params, cfg, dt=BF)
    check(ours, ref32, refbf, "vision tower + connector C2", gate_tol=2e-1)


def test_infer_host_stream_matches_per_batch(cuda):
    """The overlapped host API (copies of batch k+1 during compute of batch k,
    double-buffered staging) gives exactly the per-batch results."""
    from vla_b200.model import SmolVLA
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=0)
    m = SmolVLA(cfg, params, "cuda")
    batches, refs = [], []
    for s in range(3):
        obs = W.observation_batch(cfg, 2, seed=10 + s)
        host = tuple(obs[k].pin_memory() for k in ("images", "token_ids", "state", "noise"))
        batches.append(host)
        refs.append(m.infer(*(t.cuda() for t in host)).clone().cpu())
    outs = [torch.empty(2, cfg.expert.chunk, cfg.expert.action_dim).pin_memory() for _ in range(3)]
    m.infer_host_stream(batches, outs)
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)


def test_launch_overlap_is_bit_exact(cuda):
    """Programmatic dependent launch changes only scheduling: the whole pipeline
    (eager and CUDA-graph) gives identical bits with the overlap on and off."""
    from vla_b200 import _lib
    from vla_b200.model import SmolVLA
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, 3, seed=5)
    args = [obs[k].cuda() for k in ("images", "token_ids", "state", "noise")]
    lib = _lib.load()
    outs = {}
    try:
        for ov in (0, 1):
            lib.vla_set_launch_overlap(ov)
            m = SmolVLA(cfg, params, "cuda")
            outs[ov] = (m.infer(*args, use_graph=False).clone(), m.infer(*args, use_graph=True).clone())
    finally:
        lib.vla_set_launch_overlap(1)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[1][0], outs[1][1])


def test_pipeline_camera_frames(cuda):
    """uint8 camera frames [B, H, W, 3] through the model (resize + normalise + im2col
    fused on the GPU) give exactly the actions of the equivalent bf16 images, eager
    and through the streamed host API; frames of another size are resized."""
    from vla_b200.model import SmolVLA
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, 3, seed=9)
    S = cfg.vision.image
    g = torch.Generator().manual_seed(9)
    frames = torch.randint(0, 256, (3, S, S, 3), generator=g, dtype=torch.uint8)
    images = (frames.permute(0, 3, 1, 2).float() * (2.0 / 255.0) - 1.0).to(BF)
    rest = [obs[k].cuda() for k in ("token_ids", "state", "noise")]
    m = SmolVLA(cfg, params, "cuda")
    ref = m.infer(images.cuda(), *rest, use_graph=False).clone()
    out = m.infer(frames.cuda(), *rest, use_graph=False).clone()
    assert torch.equal(out, ref)
    out_g = m.infer(frames.cuda(), *rest, use_graph=True).clone()
    assert torch.equal(out_g, ref)
    host = (frames.pin_memory(), obs["token_ids"].pin_memory(), obs["state"].pin_memory(), obs["noise"].pin_memory())
    outs = [torch.empty(3, cfg.expert.chunk, cfg.expert.action_dim).pin_memory() for _ in range(2)]
    m.infer_host_stream([host, host], outs)
    assert torch.equal(outs[1], ref.cpu())
    # a 96 x 160 camera: resized to S x S on the GPU, against the oracle on torch's resize
    big = torch.randint(0, 256, (3, 96, 160, 3), generator=g, dtype=torch.uint8)
    out_r = m.infer(big.cuda(), *rest, use_graph=False).clone()
    resized = F.interpolate(big.permute(0, 3, 1, 2).float(), size=(S, S), mode="bilinear", align_corners=False,
                            antialias=False) * (2.0 / 255.0) - 1.0
    obs_r = dict(obs, images=resized)
    ref32 = R.smolvla_chunk(obs_r, params, cfg, dt=F32)
    refbf = R.smolvla_chunk(obs_r, params, cfg, dt=BF)
    check(out_r, ref32, refbf, "pipeline tiny from resized camera frames")


def test_infer_overlapped_matches_per_batch(cuda):
    """Consecutive batches overlapped (batch k+1's vision / text half on one stream
    while batch k's expert runs on another, alternating prefix K/V slots) give
    exactly the per-batch results, for bf16 images and for uint8 camera frames."""
    from vla_b200.model import SmolVLA
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=0)
    m = SmolVLA(cfg, params, "cuda")
    for frames in (False, True):
        batches, refs = [], []
        for s in range(5):
            obs = W.observation_batch(cfg, 2, seed=20 + s)
            img = obs["images"]
            if frames:
                g = torch.Generator().manual_seed(30 + s)
                img = torch.randint(0, 256, (2, 96, 112, 3), generator=g, dtype=torch.uint8)
            host = (img.pin_memory(), obs["token_ids"].pin_memory(), obs["state"].pin_memory(),
                    obs["noise"].pin_memory())
            batches.append(host)
            refs.append(m.infer(*(t.cuda() for t in host)).clone().cpu())
        outs = [torch.empty(2, cfg.expert.chunk, cfg.expert.action_dim).pin_memory() for _ in range(5)]
        m.infer_overlapped(batches, outs)
        for o, r in zip(outs, refs):
            assert torch.equal(o, r)


@pytest.mark.parametrize("kind,B,L", [("text", 1, 128), ("text", 2, 113), ("self", 3, 50), ("cross", 3, 50),
                                      ("self", 8, 50)])
def test_fused_layer_matches_seven_launch_layer(cuda, kind, B, L):
    """The single-launch layer (cooperative kernel, grid barriers between its seven
    phases) against the seven-launch layer on the same inputs: the same kernels'
    arithmetic in the same order, so the outputs agree to the last bit or within
    one bf16 rounding of an attention row."""
    from vla_b200 import _lib
    from vla_b200 import device as dev
    from vla_b200.model import LlamaLayerWeights, rope_table
    lib = _lib.load()
    t, e = TextCfg(), ExpertCfg()
    cfg = t if kind == "text" else e
    if kind == "cross":
        p = W.expert_cross_params(e, t.kv_dim, seed=31, layer=1)
    elif kind == "self":
        p = W.expert_self_params(e, seed=31)
    else:
        p = W.text_block_params(t, seed=31)
    lw = LlamaLayerWeights(p, cfg, "cuda", cross=kind == "cross")
    x0 = _x((B * L, cfg.hidden), 31, "fused.x").to(BF).cuda()
    cs = rope_table(L, 64, cfg.rope_theta).cuda()
    kv = _x((B * 113, 2 * e.kv_dim), 31, "fused.kv").to(BF).cuda()
    kv_len = torch.tensor([113, 97, 64][:B], dtype=torch.int32, device="cuda")
    outs = {}
    prev = lib.vla_set_fused_layers(1)
    try:
        for fused in (1, 0):
            lib.vla_set_fused_layers(fused)
            x = x0.clone()
            qkv = torch.empty(B * L, cfg.q_dim + 2 * cfg.kv_dim, dtype=BF, device="cuda")
            if kind == "cross":
                dev.llama_cross_layer(lw.struct, x, B, L, cs, kv[:, :e.kv_dim], kv[:, e.kv_dim:], 113, dev.Workspace(),
                                      kv_len=kv_len)
            else:
                dev.llama_self_layer(lw.struct, x, B, L, cs, dev.Workspace(), qkv_out=qkv)
            dev.sync_check()
            outs[fused] = (x, qkv)
    finally:
        lib.vla_set_fused_layers(prev)
    torch.testing.assert_close(outs[1][0].float(), outs[0][0].float(), atol=2e-2, rtol=1e-2)
    if kind != "cross":
        assert torch.equal(outs[1][1], outs[0][1]), "Q / K / V differ"
    print(f"[fused] {kind} B={B} L={L}: bit-identical output = {torch.equal(outs[1][0], outs[0][0])}")
