"""CPU oracle for the SmolVLA bf16 hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product (vla-to-npu_b200/vla_b200) never calls it.

It restates, in plain PyTorch CPU code, the reference's torch modules that
serve as its own correctness oracle:

* TextEncoderBlock.forward      vla/text_encoder_bf16.py:106-135
* apply_rope (half-split)       vla/text_encoder_bf16.py:92-104
* ActionExpertSelfBlock         vla/action_expert_bf16.py:69-131
* ActionExpertCrossBlock        vla/action_expert_bf16.py:137-207
* CrossAttentionBlock           vla/llama_block_rope_bf16.py:133-180
* llama_block_rope_cross        vla/llama_block_rope_bf16.py:617-709 (the
  Allo cross path: RoPE on Q and on the given key, causal mask)
* MiniVit (block skeleton)      vla/vision_block_bf16.py:57-79, with the real
  SigLIP layer of vla/vision_block.py:4-30 (biases, LayerNorm eps 1e-6,
  GELU-tanh)
* SiglipVisionEmbeddings        vla/vit_emb.py:26-47 (patch conv + pos-emb)
* con_ref (pixel shuffle)       vla/vla.py:434-437
* joint_transformer_ref         vla/vla.py:489-504 (layer schedule)
* postprocessing_ref            vla/vla.py:507-520 (RMSNorm + 768->32)
* create_text_emb               vla/vla.py:169-174 (x sqrt(hidden))

Every function is generic over ``dt``: with ``dt=torch.float32`` it is the
fp32 oracle (bf16 weights upcast); with ``dt=torch.bfloat16`` it reproduces
the reference's own bf16 CPU path (the modules ``.to(torch.bfloat16)`` as in
vla/text_encoder_bf16.py:616-622), which sets the parity floor.

Semantics the reference leaves open are pinned here (and the CUDA path
follows them):

* text layer K/V export: this layer's post-RoPE K and its V, as the Allo path
  returns them (vla/text_encoder_bf16.py:494-500, 595); the torch oracle's
  recomputation from ln_1(residual) (:133-135) is available with
  ``kv_export="recompute"`` for pinning against the reference class;
* RMSNorm / LayerNorm eps are explicit (C0: 1e-5, SigLIP: 1e-6);
* the flow-matching loop, time embedding and action projections are not in
  the reference (vla/vla.py:312 feeds random noise straight into the expert):
  x_{k+1} = x_k + dt * v(x_k, t_k), t_k = 1 - k/steps, dt = -1/steps, v =
  W_out . RMSNorm(expert(x W_in + temb(t))), temb = [sin(2 pi t / p_i),
  cos(2 pi t / p_i)] with log-spaced periods p_i in [4e-3, 4].
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Sequence

import torch
import torch.nn.functional as F

F32 = torch.float32
BF16 = torch.bfloat16


def _c(t: torch.Tensor, dt) -> torch.Tensor:
    return t.to(dt)


def linear(x: torch.Tensor, w_in_out: torch.Tensor, bias: Optional[torch.Tensor] = None, dt=F32) -> torch.Tensor:
    """x @ W with the reference's [in, out] weight layout (nn.Linear on W.T)."""
    return F.linear(_c(x, dt), _c(w_in_out, dt).t(), None if bias is None else _c(bias, dt))


def rms_norm(x, g, eps, dt=F32):
    """nn.RMSNorm(elementwise_affine=True) with an explicit eps
    (vla/text_encoder_bf16.py:73,108; kernel cc/bf16/rms_norm_960_bf16.cc:18-62)."""
    return F.rms_norm(_c(x, dt), (x.shape[-1],), _c(g, dt), eps)


def layer_norm(x, g, b, eps, dt=F32):
    """nn.LayerNorm (vla/vision_block_bf16.py:61; cc/bf16_old/layer_norm_bf16.cc:16-70 + bias region
    vla/vision_block_bf16.py:101-127)."""
    return F.layer_norm(_c(x, dt), (x.shape[-1],), _c(g, dt), _c(b, dt), eps)


def rope_timescale(head_dim: int, theta: float) -> torch.Tensor:
    """theta ** ((2/D) * k), k < D/2, computed in fp32 (vla/text_encoder_bf16.py:80-82)."""
    freq_exponents = (2.0 / head_dim) * torch.arange(head_dim // 2, dtype=F32)
    return theta ** freq_exponents


def rope_cos_sin(seq: int, head_dim: int, theta: float) -> torch.Tensor:
    """[seq, head_dim] fp32 table: cos(pos / ts_k) for k < D/2, then sin(pos / ts_k).
    Same fp32 radians as apply_rope (vla/text_encoder_bf16.py:95-96)."""
    ts = rope_timescale(head_dim, theta)
    radians = torch.arange(seq, dtype=F32)[:, None] / ts[None, :]
    return torch.cat([torch.cos(radians), torch.sin(radians)], dim=-1)


def apply_rope(x: torch.Tensor, theta: float, positions: Optional[torch.Tensor] = None, dt=F32) -> torch.Tensor:
    """Half-split rotary embedding on x [B, L, H, D], computed and RETURNED in fp32
    (vla/text_encoder_bf16.py:92-104: ``x`` is rebound to its fp32 copy before
    ``out.to(x.dtype)``, so the rotated Q/K are never rounded to bf16).  The
    timescale is a registered buffer of the reference module, so
    ``module.to(torch.bfloat16)`` rounds it to bf16; ``dt`` reproduces that
    (vla/text_encoder_bf16.py:83, 95)."""
    B, L, H, D = x.shape
    d_half = D // 2
    ts = rope_timescale(D, theta).to(dt).to(F32)
    if positions is None:
        positions = torch.arange(L, dtype=F32)[None, :].expand(B, -1)
    radians = positions.to(F32)[..., None] / ts[None, None, :]
    radians = radians[..., None, :]
    xf = x.to(F32)
    x1, x2 = xf.split(d_half, dim=-1)
    s, c = torch.sin(radians), torch.cos(radians)
    out = torch.empty_like(xf)
    out[..., :d_half] = x1 * c - x2 * s
    out[..., d_half:] = x2 * c + x1 * s
    return out


def attention(q, k, v, causal: bool, kv_len: Optional[Sequence[int]] = None, dt=F32):
    """Scaled dot-product attention as the reference's torch blocks do it:
    fp32 scores / sqrt(D), -inf mask, fp32 softmax, probabilities cast to the
    working dtype, fp32 P.V, context cast back (vla/text_encoder_bf16.py:117-126).

    q [B, Lq, Hq, D], k/v [B, Lk, Hkv, D]; GQA head h reads kv head
    h * Hkv // Hq (vla/text_encoder_bf16.py:117).  ``kv_len[b]`` masks keys
    >= kv_len[b] (key padding).  Returns [B, Lq, Hq * D] in dt.
    """
    B, Lq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    kv_map = torch.div(torch.arange(Hq) * Hkv, Hq, rounding_mode="floor")
    qh = q.transpose(1, 2).float()
    kh = k.index_select(2, kv_map).transpose(1, 2).float()
    vh = v.index_select(2, kv_map).transpose(1, 2).float()
    scores = torch.matmul(qh, kh.transpose(-2, -1)) / (D ** 0.5)
    if causal:
        scores.masked_fill_(torch.ones(Lq, Lk).triu(1).bool(), float("-inf"))
    if kv_len is not None:
        keys = torch.arange(Lk)
        for b, n in enumerate(kv_len):
            scores[b, :, :, keys >= int(n)] = float("-inf")
    attn = torch.softmax(scores, dim=-1).to(dt)
    ctx = torch.matmul(attn.float(), vh).to(dt)
    return ctx.transpose(1, 2).contiguous().view(B, Lq, Hq * D)


def swiglu_mlp(x, p, dt=F32):
    """down(silu(gate(x)) * up(x)) (vla/text_encoder_bf16.py:131)."""
    return linear(F.silu(linear(x, p["W_gate"], dt=dt)) * linear(x, p["W_up"], dt=dt), p["W_down"], dt=dt)


def text_block(x, p: Dict[str, torch.Tensor], cfg, dt=F32, kv_export: str = "roped"):
    """One Llama-style text decoder block, x [B, L, hidden] -> (out, K, V) with
    K/V [B, L, kv_heads * head_dim] (vla/text_encoder_bf16.py:106-135)."""
    x = _c(x, dt)
    residual = x
    h = rms_norm(x, p["W_norm_1"], cfg.eps, dt)
    B, L, _ = h.shape
    D = cfg.head_dim
    q = linear(h, p["Wq"], dt=dt).view(B, L, cfg.heads, D)
    k = linear(h, p["Wk"], dt=dt).view(B, L, cfg.kv_heads, D)
    v = linear(h, p["Wv"], dt=dt).view(B, L, cfg.kv_heads, D)
    q = apply_rope(q, cfg.rope_theta, dt=dt)
    k = apply_rope(k, cfg.rope_theta, dt=dt)
    ctx = attention(q, k, v, causal=True, dt=dt)
    x = linear(ctx, p["Wo"], dt=dt) + residual
    residual = x
    h = rms_norm(x, p["W_norm_2"], cfg.eps, dt)
    x = swiglu_mlp(h, p, dt) + residual
    if kv_export == "recompute":
        hh = rms_norm(residual, p["W_norm_1"], cfg.eps, dt)
        return x, linear(hh, p["Wk"], dt=dt), linear(hh, p["Wv"], dt=dt)
    return x, k.reshape(B, L, -1).to(dt), v.reshape(B, L, -1)


def vision_block(x, p: Dict[str, torch.Tensor], cfg, dt=F32, gelu: str = "tanh"):
    """SigLIP encoder layer, x [B, S, hidden] (vla/vision_block_bf16.py:67-79 skeleton,
    vla/vision_block.py:13-25 config): pre-LN, biased q/k/v/out projections,
    non-causal softmax attention, pre-LN biased MLP with GELU."""
    x = _c(x, dt)
    residual = x
    h = layer_norm(x, p["W_norm_1"], p["b_norm_1"], cfg.eps, dt)
    B, S, _ = h.shape
    D = cfg.head_dim
    q = linear(h, p["Wq"], p.get("bq"), dt).view(B, S, cfg.heads, D)
    k = linear(h, p["Wk"], p.get("bk"), dt).view(B, S, cfg.heads, D)
    v = linear(h, p["Wv"], p.get("bv"), dt).view(B, S, cfg.heads, D)
    ctx = attention(q, k, v, causal=False, dt=dt)
    x = linear(ctx, p["Wo"], p.get("bo"), dt) + residual
    residual = x
    h = layer_norm(x, p["W_norm_2"], p["b_norm_2"], cfg.eps, dt)
    a = F.gelu(linear(h, p["W_up"], p.get("b_up"), dt), approximate=gelu)
    return linear(a, p["W_down"], p.get("b_down"), dt) + residual


def patch_embed(images, pp, cfg, dt=F32):
    """Conv2d(3, hidden, k=s=patch) + bias, flattened to [B, tokens, hidden], plus the
    learned position embedding (vla/vit_emb.py:43-47; vla/vla.py:396-409)."""
    y = F.conv2d(_c(images, dt), _c(pp["kernel"], dt), _c(pp["b_patch"], dt), stride=cfg.patch)
    y = y.flatten(2).transpose(1, 2)
    return y + _c(pp["pos_emb"], dt)[None]


def pixel_shuffle(x, grid: int, scale: int):
    """[B, grid*grid, C] -> [B, (grid/scale)^2, scale^2 C], the reshape/transpose chain of
    con_ref (vla/vla.py:434-436) generalised from (32, 4, 768)."""
    B, N, C = x.shape
    g2 = grid // scale
    y = x.reshape(B, grid, grid, C).reshape(B, grid, g2, scale * C).transpose(1, 2)
    y = y.reshape(B, g2, g2, scale * scale * C).transpose(1, 2)
    return y.reshape(B, g2 * g2, scale * scale * C)


def connector(x, W, vcfg, scale: int, dt=F32):
    """Pixel shuffle then x @ W without bias (vla/vla.py:434-437; vla/connector_bf16.py:97-139)."""
    return linear(pixel_shuffle(_c(x, dt), vcfg.grid, scale), W, dt=dt)


def vision_tower(images, params, cfg, dt=F32):
    """Patch embed -> vision layers -> post-LayerNorm -> connector: [B, image_tokens, text hidden]."""
    v = cfg.vision
    x = patch_embed(images, params["patch"], v, dt)
    for lp in params["vision"]:
        x = vision_block(x, lp, v, dt)
    x = layer_norm(x, params["patch"]["W_post_norm"], params["patch"]["b_post_norm"], v.eps, dt)
    return connector(x, params["connector"]["W"], v, cfg.connector.scale, dt)


def expert_self_block(x, p, cfg, dt=F32):
    """Causal self-attention expert layer (vla/action_expert_bf16.py:104-131)."""
    x = _c(x, dt)
    residual = x
    h = rms_norm(x, p["W_norm_1"], cfg.eps, dt)
    B, L, _ = h.shape
    D = cfg.head_dim
    q = apply_rope(linear(h, p["Wq"], dt=dt).view(B, L, cfg.heads, D), cfg.rope_theta, dt=dt)
    k = apply_rope(linear(h, p["Wk"], dt=dt).view(B, L, cfg.kv_heads, D), cfg.rope_theta, dt=dt)
    v = linear(h, p["Wv"], dt=dt).view(B, L, cfg.kv_heads, D)
    ctx = attention(q, k, v, causal=True, dt=dt)
    x = linear(ctx, p["Wo"], dt=dt) + residual
    residual = x
    h = rms_norm(x, p["W_norm_2"], cfg.eps, dt)
    return swiglu_mlp(h, p, dt) + residual


def expert_cross_kv(text_k, text_v, p, dt=F32):
    """Cross-attention K/V projections of the text layer's K/V (vla/action_expert_bf16.py:180-181)."""
    return linear(text_k, p["Wk_cross"], dt=dt), linear(text_v, p["Wv_cross"], dt=dt)


def expert_cross_block(x, kc, vc, p, cfg, kv_len=None, dt=F32):
    """Cross-attention expert layer on already-projected K/V [B, Lc, kv_dim]
    (vla/action_expert_bf16.py:169-207): RoPE on Q only, no causal mask,
    optional key padding mask."""
    x = _c(x, dt)
    residual = x
    h = rms_norm(x, p["W_norm_1"], cfg.eps, dt)
    B, L, _ = h.shape
    Lc = kc.shape[1]
    D = cfg.head_dim
    q = apply_rope(linear(h, p["Wq"], dt=dt).view(B, L, cfg.heads, D), cfg.rope_theta, dt=dt)
    k = _c(kc, dt).view(B, Lc, cfg.kv_heads, D)
    v = _c(vc, dt).view(B, Lc, cfg.kv_heads, D)
    ctx = attention(q, k, v, causal=False, kv_len=kv_len, dt=dt)
    x = linear(ctx, p["Wo"], dt=dt) + residual
    residual = x
    h = rms_norm(x, p["W_norm_2"], cfg.eps, dt)
    return swiglu_mlp(h, p, dt) + residual


def cross_attention_block(x, context, p, cfg, dt=F32):
    """CrossAttentionBlock.forward (vla/llama_block_rope_bf16.py:133-180): the
    context is normalised by the same ln_1 as x and projected by k_proj / v_proj;
    no RoPE and no mask; fp32 scores and softmax, probabilities cast to the
    working dtype, fp32 P.V cast back.  ``p`` uses the reference keys
    (Wq, Wk, Wv, Wo, W_gate, W_up, W_down, W_norm_1, W_norm_2)."""
    x = _c(x, dt)
    context = _c(context, dt)
    residual = x
    xn = rms_norm(x, p["W_norm_1"], cfg.eps, dt)
    cn = rms_norm(context, p["W_norm_1"], cfg.eps, dt)
    B, L, _ = xn.shape
    Lc = cn.shape[1]
    D = cfg.head_dim
    q = linear(xn, p["Wq"], dt=dt).view(B, L, cfg.heads, D)
    k = linear(cn, p["Wk"], dt=dt).view(B, Lc, cfg.kv_heads, D)
    v = linear(cn, p["Wv"], dt=dt).view(B, Lc, cfg.kv_heads, D)
    ctx = attention(q, k, v, causal=False, dt=dt)
    x = linear(ctx, p["Wo"], dt=dt) + residual
    residual = x
    h = rms_norm(x, p["W_norm_2"], cfg.eps, dt)
    return swiglu_mlp(h, p, dt) + residual


def llama_block_rope_cross(key, value, x, p, cfg, dt=F32):
    """The Allo cross block (vla/llama_block_rope_bf16.py:617-709): Q = RoPE(RMSNorm(x) Wq),
    the GIVEN key [B, L, kv_dim] is rotated by RoPE at positions 0..L-1 as well
    (:629-630), the given value is used as is, the score is causally masked
    (:641-652, the key sequence has the query's length), then the output
    projection and the SwiGLU MLP with residuals.  Numerics follow the
    reference's torch twin of this block (AttentionExpertBlock,
    vla/llama_block_rope_bf16.py:60-131: RoPE evaluated and returned in fp32,
    fp32 scores and softmax, probabilities and context in the working dtype), so
    that with key = RMSNorm(x) Wk and value = RMSNorm(x) Wv it reproduces that
    module exactly."""
    x = _c(x, dt)
    residual = x
    h = rms_norm(x, p["W_norm_1"], cfg.eps, dt)
    B, L, _ = h.shape
    D = cfg.head_dim
    q = apply_rope(linear(h, p["Wq"], dt=dt).view(B, L, cfg.heads, D), cfg.rope_theta, dt=dt)
    k = apply_rope(_c(key, dt).view(B, L, cfg.kv_heads, D), cfg.rope_theta, dt=dt)
    v = _c(value, dt).view(B, L, cfg.kv_heads, D)
    ctx = attention(q, k, v, causal=True, dt=dt)
    x = linear(ctx, p["Wo"], dt=dt) + residual
    residual = x
    h = rms_norm(x, p["W_norm_2"], cfg.eps, dt)
    return swiglu_mlp(h, p, dt) + residual


def time_embedding(t: float, dim: int, min_period: float, max_period: float) -> torch.Tensor:
    """Sinusoidal embedding of a scalar time: [sin(2 pi t / p_i), cos(2 pi t / p_i)],
    p_i log-spaced in [min_period, max_period], i < dim/2 (fp64 math, fp32 out)."""
    half = dim // 2
    frac = torch.linspace(0.0, 1.0, half, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** frac
    ang = 2.0 * math.pi * t / period
    return torch.cat([torch.sin(ang), torch.cos(ang)]).to(F32)


def prefix_embed(image_tokens, token_ids, state, params, cfg, dt=F32):
    """[image tokens | text embeddings * sqrt(hidden) | state projection]
    (vla/vla.py:169-182, 326; the reference's 15 zero pad rows are not materialised:
    a causal mask makes them invisible to the valid rows)."""
    H = cfg.text.hidden
    emb = _c(params["embed"], dt)[token_ids.long()]
    if cfg.prefix.embed_scale_sqrt_hidden:
        emb = emb * math.sqrt(H)
    st = linear(state, params["W_state"], dt=dt)[:, None, :]
    return torch.cat([_c(image_tokens, dt), _c(emb, dt), st], dim=1)


def expert_velocity(x_t, t, text_kv, params, cfg, dt=F32, kv_len=None):
    """v(x_t, t): in-projection + time embedding, expert layers (even: causal self,
    odd: cross to that layer's projected prefix K/V, keys >= kv_len[b] masked),
    final RMSNorm, out-projection (vla/vla.py:194-222 layer schedule and
    postprocessing)."""
    e = cfg.expert
    temb = time_embedding(t, e.hidden, e.min_period, e.max_period)
    h = linear(x_t, params["W_action_in"], dt=dt) + _c(temb, dt)
    for i, lp in enumerate(params["expert"]):
        if i % 2 == 0:
            h = expert_self_block(h, lp, e, dt)
        else:
            kc, vc = text_kv[i]
            h = expert_cross_block(h, kc, vc, lp, e, kv_len=kv_len, dt=dt)
    h = rms_norm(h, params["W_exp_norm"], e.eps, dt)
    return linear(h, params["W_action_out"], dt=dt)


def smolvla_chunk(obs, params, cfg, dt=F32):
    """Full action-chunk inference for a batch of observations; returns actions
    [B, chunk, action_dim] in fp32 and the per-layer prefix K/V."""
    img = vision_tower(obs["images"], params, cfg, dt)
    x = prefix_embed(img, obs["token_ids"], obs["state"], params, cfg, dt)
    text_kv = {}
    for i, lp in enumerate(params["text"]):
        x, k, v = text_block(x, lp, cfg.text, dt)
        if i % 2 == 1 and i < cfg.expert.layers:
            text_kv[i] = expert_cross_kv(k, v, params["expert"][i], dt)
    return flow_matching(obs["noise"], text_kv, params, cfg, dt)


def flow_matching(noise, text_kv, params, cfg, dt=F32, kv_len=None):
    """Euler integration of the action chunk from x0 = noise [B, chunk, action_dim]:
    x_{k+1} = x_k + dt_k * v(x_k, t_k), t_k = 1 - k/steps, dt_k = -1/steps, the
    state kept in fp32 (not in the reference, whose vla/vla.py:312 feeds noise
    straight into one expert pass)."""
    e = cfg.expert
    xt = noise.to(F32)
    step = -1.0 / e.steps
    for s in range(e.steps):
        t = 1.0 + s * step
        vel = expert_velocity(xt.to(dt), t, text_kv, params, cfg, dt, kv_len=kv_len)
        xt = xt + step * vel.to(F32)
    return xt


def action_expert_chunk(noise, prefix_k, prefix_v, params, cfg, kv_len=None, dt=F32):
    """The action expert on its own (benchmark configuration C3): ``prefix_k`` /
    ``prefix_v`` [layers, B, Lc, text kv_dim] are a cached VLM prefix K/V per text
    layer; each cross layer i projects layer i's K/V by its Wk_cross / Wv_cross
    (vla/action_expert_bf16.py:756-759) and attends to it with keys >= kv_len[b]
    masked; 10 Euler steps as in flow_matching."""
    text_kv = {}
    for i, lp in enumerate(params["expert"]):
        if i % 2 == 1:
            text_kv[i] = expert_cross_kv(_c(prefix_k[i], dt), _c(prefix_v[i], dt), lp, dt)
    return flow_matching(noise, text_kv, params, cfg, dt, kv_len=kv_len)
