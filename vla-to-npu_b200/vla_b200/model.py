"""Device-resident SmolVLA: weights uploaded once in the kernels' layout, every
activation buffer preallocated per batch size, the whole action-chunk forward
captured once into a CUDA graph and replayed.

Pipeline (one action chunk per observation; the reference's orchestration is
vla/vla.py:228-389 with joint_transformer vla/vla.py:194-212):

  images -> im2col -> patch GEMM (+bias, +position embedding)        [B*1024, 768]
         -> 12 SigLIP layers -> post-LayerNorm -> pixel shuffle x4   [B*64, 12288]
         -> connector GEMM, rows scattered into the prefix           [B*113, 960]
  ids    -> embedding gather * sqrt(960) into prefix rows 64..111
  state  -> state GEMM into prefix row 112
  prefix -> 16 causal text layers; odd layer i exports its post-RoPE K/V,
            projected once per chunk by the expert's Wk_cross / Wv_cross
  noise  -> 10 Euler steps of the 16-layer action expert (even: causal
            self-attention over 50 tokens, odd: cross-attention to layer i's
            prefix K/V); velocity = W_out . RMSNorm(h); the out-projection's
            epilogue performs x += dt * v in fp32
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from . import _lib
from . import device as dev
from .configs import ExpertCfg, SmolVLACfg, TextCfg, VisionCfg

BF16 = torch.bfloat16


# ---------------------------------------------------------------------------
# tables computed once on the host
# ---------------------------------------------------------------------------
def rope_table(seq: int, head_dim: int, theta: float) -> torch.Tensor:
    """fp32 [seq, head_dim]: cos(pos / ts_k) | sin(pos / ts_k), ts_k = theta^(2k/D)
    evaluated in fp32 as the reference does (vla/text_encoder_bf16.py:80-96)."""
    ts = theta ** ((2.0 / head_dim) * torch.arange(head_dim // 2, dtype=torch.float32))
    rad = torch.arange(seq, dtype=torch.float32)[:, None] / ts[None, :]
    return torch.cat([torch.cos(rad), torch.sin(rad)], dim=-1).contiguous()


def time_embedding_table(e: ExpertCfg) -> torch.Tensor:
    """[steps, hidden] fp32: row s embeds t_s = 1 - s/steps as
    [sin(2 pi t / p_i), cos(2 pi t / p_i)], p_i log-spaced in [min_period, max_period]."""
    half = e.hidden // 2
    frac = torch.linspace(0.0, 1.0, half, dtype=torch.float64)
    period = e.min_period * (e.max_period / e.min_period) ** frac
    rows = []
    for s in range(e.steps):
        t = 1.0 - s / e.steps
        ang = 2.0 * math.pi * t / period
        rows.append(torch.cat([torch.sin(ang), torch.cos(ang)]))
    return torch.stack(rows).to(torch.float32)


# ---------------------------------------------------------------------------
# weight layout conversion: reference [in, out] -> kernels' K-major [out, in]
# ---------------------------------------------------------------------------
def _kmajor(w_in_out: torch.Tensor, device) -> torch.Tensor:
    return w_in_out.to(BF16).t().contiguous().to(device)


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, device) -> torch.Tensor:
    """[2F, H] with rows [32j, 32j+16) = gate^T rows [16j, 16j+16) and
    [32j+16, 32j+32) = up^T rows [16j, 16j+16) (the SwiGLU epilogue pairing)."""
    g = w_gate.to(BF16).t().contiguous()
    u = w_up.to(BF16).t().contiguous()
    F_, H = g.shape
    assert F_ % 16 == 0
    out = torch.stack([g.view(F_ // 16, 16, H), u.view(F_ // 16, 16, H)], dim=1).reshape(2 * F_, H)
    return out.contiguous().to(device)


class LlamaLayerWeights:
    """One text-decoder or action-expert layer on the device."""

    def __init__(self, p: Dict[str, torch.Tensor], cfg, device, cross: bool = False):
        self.cross = cross
        if cross:
            self.w_qkv = _kmajor(p["Wq"], device)
            self.wk_cross = _kmajor(p["Wk_cross"], device)
            self.wv_cross = _kmajor(p["Wv_cross"], device)
        else:
            self.w_qkv = _kmajor(torch.cat([p["Wq"], p["Wk"], p["Wv"]], dim=1), device)
        self.w_o = _kmajor(p["Wo"], device)
        self.w_gu = interleave_gate_up(p["W_gate"], p["W_up"], device)
        self.w_down = _kmajor(p["W_down"], device)
        self.norm1 = p["W_norm_1"].to(BF16).contiguous().to(device)
        self.norm2 = p["W_norm_2"].to(BF16).contiguous().to(device)
        s = _lib.LlamaLayer()
        s.norm1, s.w_qkv, s.w_o = self.norm1.data_ptr(), self.w_qkv.data_ptr(), self.w_o.data_ptr()
        s.norm2, s.w_gu, s.w_down = self.norm2.data_ptr(), self.w_gu.data_ptr(), self.w_down.data_ptr()
        s.hidden, s.heads, s.kv_heads, s.head_dim, s.ffn = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn
        s.eps = cfg.eps
        self.struct = s


class VisionLayerWeights:
    def __init__(self, p: Dict[str, torch.Tensor], cfg: VisionCfg, device):
        H = cfg.hidden
        z = torch.zeros(H, dtype=BF16)
        self.w_qkv = _kmajor(torch.cat([p["Wq"], p["Wk"], p["Wv"]], dim=1), device)
        self.b_qkv = torch.cat([p.get("bq", z), p.get("bk", z), p.get("bv", z)]).to(BF16).contiguous().to(device)
        self.w_o = _kmajor(p["Wo"], device)
        self.b_o = p.get("bo", z).to(BF16).contiguous().to(device)
        self.w_fc1 = _kmajor(p["W_up"], device)
        self.b_fc1 = p.get("b_up", torch.zeros(cfg.ffn, dtype=BF16)).to(BF16).contiguous().to(device)
        self.w_fc2 = _kmajor(p["W_down"], device)
        self.b_fc2 = p.get("b_down", z).to(BF16).contiguous().to(device)
        self.ln = [p[k].to(BF16).contiguous().to(device) for k in ("W_norm_1", "b_norm_1", "W_norm_2", "b_norm_2")]
        s = _lib.VisionLayer()
        s.ln1_g, s.ln1_b, s.ln2_g, s.ln2_b = (t.data_ptr() for t in self.ln)
        s.w_qkv, s.b_qkv, s.w_o, s.b_o = (self.w_qkv.data_ptr(), self.b_qkv.data_ptr(), self.w_o.data_ptr(),
                                          self.b_o.data_ptr())
        s.w_fc1, s.b_fc1, s.w_fc2, s.b_fc2 = (self.w_fc1.data_ptr(), self.b_fc1.data_ptr(), self.w_fc2.data_ptr(),
                                              self.b_fc2.data_ptr())
        s.hidden, s.heads, s.head_dim, s.ffn, s.eps = H, cfg.heads, cfg.head_dim, cfg.ffn, cfg.eps
        self.struct = s


# ---------------------------------------------------------------------------
# the action expert (benchmark configuration C3; the last stage of the model)
# ---------------------------------------------------------------------------
class ActionExpert:
    """The 16-layer action expert with its flow-matching loop, on the device.

    Even layers: causal self-attention over the chunk; odd layers: cross-attention
    to a cached prefix K/V (the K/V of text layer i, projected once per chunk by
    layer i's Wk_cross / Wv_cross and reused by every Euler step; the reference
    recomputes the projection on every call, vla/action_expert_bf16.py:756-759).
    ``kv_len`` (device int32 [B], optional) masks prefix keys >= kv_len[b]
    (key padding).  Flow matching: x_{k+1} = x_k + dt v(x_k, t_k) with the fp32
    state updated by the out-projection GEMM's epilogue."""

    def __init__(self, cfg: SmolVLACfg, params: dict, device, ws: Optional[dev.Workspace] = None):
        e = cfg.expert
        d = torch.device(device)
        self.cfg, self.device = cfg, d
        self.layers = [LlamaLayerWeights(p, e, d, cross=(i % 2 == 1)) for i, p in enumerate(params["expert"])]
        self.w_in = _kmajor(params["W_action_in"], d)
        self.exp_norm = params["W_exp_norm"].to(BF16).contiguous().to(d)
        self.w_out = _kmajor(params["W_action_out"], d)
        self.temb = time_embedding_table(e).to(BF16).to(d)
        self.rope = rope_table(e.chunk, e.head_dim, e.rope_theta).to(d)
        self.ws = ws if ws is not None else dev.Workspace(d)
        self.cross_index = {}
        for i, lw in enumerate(self.layers):
            if lw.cross:
                self.cross_index[i] = len(self.cross_index)
        self.batch = 0
        self.prefix_len = 0
        self.slot = 0
        self.kv_len: Optional[torch.Tensor] = None

    def allocate(self, batch: int, prefix_len: int) -> None:
        if (batch, prefix_len) == (self.batch, self.prefix_len):
            return
        e, d = self.cfg.expert, self.device
        self.batch, self.prefix_len = batch, prefix_len
        rows_e = batch * e.chunk
        # two sets of projected prefix K/V: the next batch's text layers may fill
        # one while the expert of the current batch reads the other
        self.kv_slots = [torch.empty(len(self.cross_index), batch * prefix_len, 2 * e.kv_dim, dtype=BF16, device=d)
                         for _ in range(2)]
        self.noise_slots = [torch.empty(rows_e, e.action_dim, dtype=torch.float32, device=d) for _ in range(2)]
        self.x_t = torch.empty(rows_e, e.action_dim, dtype=torch.float32, device=d)
        self.x_b = torch.empty(rows_e, e.action_dim, dtype=BF16, device=d)
        self.h = torch.empty(rows_e, e.hidden, dtype=BF16, device=d)
        self.hn = torch.empty(rows_e, e.hidden, dtype=BF16, device=d)
        self.kv_len_buf = torch.full((batch,), prefix_len, dtype=torch.int32, device=d)
        lib = _lib.load()
        import ctypes
        self.ws.get(max(lib.vla_llama_layer_workspace(ctypes.byref(w.struct), rows_e, 1) for w in self.layers))

    @property
    def kv_cross(self) -> torch.Tensor:
        """Projected prefix K/V [cross layers, B * prefix_len, 2 kv_dim] of the current slot."""
        return self.kv_slots[self.slot]

    def project_prefix_kv(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Cross layer ``layer``'s K/V from the prefix K/V [B * prefix_len, text kv_dim]."""
        e = self.cfg.expert
        lw = self.layers[layer]
        kvc = self.kv_cross[self.cross_index[layer]]
        dev.gemm(k, lw.wk_cross, kvc[:, :e.kv_dim], dev.make_epilogue(b_static=True))
        dev.gemm(v, lw.wv_cross, kvc[:, e.kv_dim:], dev.make_epilogue(b_static=True))

    def set_kv_len(self, kv_len: Optional[torch.Tensor]) -> None:
        """Key-padding lengths per observation (None: every prefix key is valid).
        The values are copied into a fixed device buffer, so a captured graph
        picks up new lengths on replay."""
        if kv_len is None:
            self.kv_len = None
            return
        self.kv_len_buf.copy_(kv_len.to(torch.int32), non_blocking=True)
        self.kv_len = self.kv_len_buf

    def run(self) -> torch.Tensor:
        """The Euler loop from the noise already in ``x_t``; returns x_t [B * chunk, action_dim]."""
        e = self.cfg.expert
        B = self.batch
        dev.f32_to_bf16(self.x_t, self.x_b)
        dt = -1.0 / e.steps
        for s in range(e.steps):
            dev.gemm(self.x_b, self.w_in, self.h, dev.make_epilogue(bias=self.temb[s], b_static=True))
            for i, lw in enumerate(self.layers):
                if lw.cross:
                    kvc = self.kv_cross[self.cross_index[i]]
                    dev.llama_cross_layer(lw.struct, self.h, B, e.chunk, self.rope, kvc[:, :e.kv_dim],
                                          kvc[:, e.kv_dim:], self.prefix_len, self.ws, kv_len=self.kv_len)
                else:
                    dev.llama_self_layer(lw.struct, self.h, B, e.chunk, self.rope, self.ws)
            dev.rms_norm(self.h, self.exp_norm, e.eps, out=self.hn)
            dev.gemm(self.hn, self.w_out, self.x_b,
                     dev.make_epilogue(act=_lib.ACT_EULER, euler_x=self.x_t, euler_dt=dt, b_static=True))
        return self.x_t

    def infer(self, noise: torch.Tensor, prefix_k: torch.Tensor, prefix_v: torch.Tensor,
              kv_len: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Benchmark configuration C3: actions [B, chunk, action_dim] fp32 from the noise
        [B, chunk, action_dim] and a cached prefix K/V [layers, B, prefix_len, text kv_dim]
        per text layer (device tensors)."""
        e = self.cfg.expert
        B, Lc = noise.shape[0], prefix_k.shape[2]
        self.allocate(B, Lc)
        for i in self.cross_index:
            self.project_prefix_kv(i, prefix_k[i].reshape(B * Lc, -1), prefix_v[i].reshape(B * Lc, -1))
        self.set_kv_len(kv_len)
        self.x_t.copy_(noise.reshape(B * e.chunk, -1))
        return self.run().view(B, e.chunk, e.action_dim)


# ---------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------
class SmolVLA:
    """SmolVLA action-chunk inference on one GPU (observations along the batch)."""

    def __init__(self, cfg: SmolVLACfg, params: dict, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        d = self.device
        v, t, e, pf = cfg.vision, cfg.text, cfg.expert, cfg.prefix
        assert v.tokens // cfg.connector.scale ** 2 == pf.image_tokens, "pixel shuffle must yield the image tokens"
        pp = params["patch"]
        self.w_patch = pp["kernel"].to(BF16).reshape(v.hidden, -1).contiguous().to(d)  # [hidden, 3*p*p], K-major
        self.b_patch = pp["b_patch"].to(BF16).contiguous().to(d)
        self.pos_emb = pp["pos_emb"].to(BF16).contiguous().to(d)
        self.post_g = pp["W_post_norm"].to(BF16).contiguous().to(d)
        self.post_b = pp["b_post_norm"].to(BF16).contiguous().to(d)
        self.vision = [VisionLayerWeights(p, v, d) for p in params["vision"]]
        self.w_conn = _kmajor(params["connector"]["W"], d)
        self.embed_table = params["embed"].to(BF16).contiguous().to(d)
        self.w_state = _kmajor(params["W_state"], d)
        self.text = [LlamaLayerWeights(p, t, d) for p in params["text"]]
        self.rope_text = rope_table(pf.length, t.head_dim, t.rope_theta).to(d)
        self.ws = dev.Workspace(d)
        # the expert has its own scratch, so that its kernels and the next batch's
        # vision / text kernels can run at the same time (infer_overlapped)
        self.action = ActionExpert(cfg, params, d)
        self.expert = self.action.layers
        self.batch = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.graph_batch = 0
        self.ov_graphs = None
        self.ov_batch = 0
        self.frames_input = False
        self.in_frames: Optional[torch.Tensor] = None

    # -- buffers ----------------------------------------------------------
    def allocate(self, batch: int) -> None:
        if batch == self.batch:
            return
        cfg, d = self.cfg, self.device
        v, t, e, pf = cfg.vision, cfg.text, cfg.expert, cfg.prefix
        self.batch = batch
        B = batch
        self.in_images = torch.empty(B, v.channels, v.image, v.image, dtype=BF16, device=d)
        self.in_frames = None  # uint8 camera frames [B, H, W, 3], allocated when frames are given
        self.frames_input = False
        self.in_ids = torch.empty(B, pf.text_tokens, dtype=torch.int32, device=d)
        self.in_state = torch.empty(B, pf.state_dim, dtype=BF16, device=d)
        self.in_noise = torch.empty(B * e.chunk, e.action_dim, dtype=torch.float32, device=d)
        rows_v = B * v.tokens
        k2 = v.hidden * cfg.connector.scale ** 2
        self.patches = torch.empty(rows_v, v.patch_dim, dtype=BF16, device=d)
        self.x_vis = torch.empty(rows_v, v.hidden, dtype=BF16, device=d)
        self.x_ln = torch.empty(rows_v, v.hidden, dtype=BF16, device=d)
        self.shuffled = torch.empty(B * pf.image_tokens, k2, dtype=BF16, device=d)
        rows_t = B * pf.length
        self.prefix = torch.empty(rows_t, t.hidden, dtype=BF16, device=d)
        self.qkv = torch.empty(rows_t, t.q_dim + 2 * t.kv_dim, dtype=BF16, device=d)
        self.action.allocate(B, pf.length)
        self.x_t = self.action.x_t
        lib = _lib.load()
        import ctypes
        need = max(
            lib.vla_vision_layer_workspace(ctypes.byref(self.vision[0].struct), rows_v) if self.vision else 0,
            lib.vla_llama_layer_workspace(ctypes.byref(self.text[0].struct), rows_t, 0),
        )
        self.ws.get(need)
        self._invalidate()

    # -- stages -----------------------------------------------------------
    def vision_tower(self) -> None:
        cfg = self.cfg
        v, t, pf = cfg.vision, cfg.text, cfg.prefix
        B = self.batch
        if self.frames_input:
            # camera frames: resize + normalisation + im2col in one kernel
            dev.camera_preprocess(self.in_frames, v.image, self.patches, patch=v.patch)
        else:
            dev.patch_im2col(self.in_images, v.patch, self.patches)
        dev.gemm(self.patches, self.w_patch, self.x_vis,
                 dev.make_epilogue(bias=self.b_patch, residual=self.pos_emb, res_row_mod=v.tokens, b_static=True))
        for lw in self.vision:
            dev.vision_layer(lw.struct, self.x_vis, B, v.tokens, self.ws)
        dev.layer_norm(self.x_vis, self.post_g, self.post_b, v.eps, out=self.x_ln)
        dev.pixel_shuffle(self.x_ln, B, v.grid, cfg.connector.scale, self.shuffled)
        # connector rows of observation b land in prefix rows [b*113, b*113 + 64)
        dev.gemm(self.shuffled, self.w_conn, self.prefix,
                 dev.make_epilogue(out_grp=pf.image_tokens, out_grp_stride=pf.length, b_static=True))

    def prefix_tokens(self) -> None:
        t, pf = self.cfg.text, self.cfg.prefix
        scale = math.sqrt(t.hidden) if pf.embed_scale_sqrt_hidden else 1.0
        dev.embed(self.in_ids, self.embed_table, scale, self.prefix, pf.length, pf.image_tokens)
        # state projection -> row 112 of each observation (row stride = prefix length)
        state_rows = self.prefix[pf.image_tokens + pf.text_tokens:].as_strided(
            (self.batch, t.hidden), (pf.length * t.hidden, 1))
        dev.gemm(self.in_state, self.w_state, state_rows, dev.make_epilogue(b_static=True))

    def text_layers(self) -> None:
        t, pf = self.cfg.text, self.cfg.prefix
        Q, KV = t.q_dim, t.kv_dim
        for i, lw in enumerate(self.text):
            dev.llama_self_layer(lw.struct, self.prefix, self.batch, pf.length, self.rope_text, self.ws,
                                 qkv_out=self.qkv)
            if i < len(self.expert) and self.expert[i].cross:
                self.action.project_prefix_kv(i, self.qkv[:, Q:Q + KV], self.qkv[:, Q + KV:Q + 2 * KV])

    def action_expert(self) -> None:
        self.x_t.copy_(self.in_noise)
        self.action.run()

    # -- the two halves of a chunk, for overlapping consecutive batches --------
    def forward_front(self) -> None:
        """Vision tower, prefix, text layers and the expert's prefix K/V projections
        into K/V slot ``self.action.slot``; the batch's noise is parked in the same slot."""
        self.vision_tower()
        self.prefix_tokens()
        self.text_layers()
        self.action.noise_slots[self.action.slot].copy_(self.in_noise)

    def forward_back(self) -> None:
        """The expert's 10 Euler steps on K/V slot ``self.action.slot``."""
        self.x_t.copy_(self.action.noise_slots[self.action.slot])
        self.action.run()

    def forward_device(self) -> torch.Tensor:
        """Launch the whole chunk forward on the current stream from the input buffers."""
        self.vision_tower()
        self.prefix_tokens()
        self.text_layers()
        self.action_expert()
        return self.x_t

    # -- graph ------------------------------------------------------------
    def capture(self) -> None:
        self.forward_device()  # warm-up: sets kernel attributes, touches every buffer
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward_device()
        torch.cuda.synchronize(self.device)
        self.graph = g
        self.graph_batch = self.batch

    def _invalidate(self) -> None:
        self.graph = None
        self.ov_graphs = None

    def replay(self) -> torch.Tensor:
        if self.graph is None or self.graph_batch != self.batch:
            self.capture()
        self.graph.replay()
        return self.x_t

    # -- public API -------------------------------------------------------
    def load_inputs(self, images, token_ids, state, noise, non_blocking: bool = True) -> None:
        """Copy one batch of observations (host or device tensors) into the input buffers."""
        B = images.shape[0]
        self.allocate(B)
        self._image_buffer(images).copy_(images.to(BF16) if images.dtype not in (BF16, torch.uint8) else images,
                                         non_blocking=non_blocking)
        self.in_ids.copy_(token_ids, non_blocking=non_blocking)
        self.in_state.copy_(state.to(BF16) if state.dtype != BF16 else state, non_blocking=non_blocking)
        self.in_noise.copy_(noise.reshape(B * self.cfg.expert.chunk, -1), non_blocking=non_blocking)

    def _image_buffer(self, images: torch.Tensor) -> torch.Tensor:
        """The device buffer an image batch is copied into: uint8 camera frames
        [B, H, W, 3] (any H, W; resized on the GPU) or images [B, 3, S, S] already
        scaled to [-1, 1].  Switching between the two re-captures the graph."""
        frames = images.dtype == torch.uint8
        if frames:
            if images.dim() != 4 or images.shape[3] != 3:
                raise ValueError("uint8 camera frames must be [B, H, W, 3]")
            if self.in_frames is None or self.in_frames.shape != images.shape:
                self.in_frames = torch.empty(images.shape, dtype=torch.uint8, device=self.device)
                self._invalidate()
        if frames != self.frames_input:
            self.frames_input = frames
            self._invalidate()
        return self.in_frames if frames else self.in_images

    def _inputs(self):
        img = self.in_frames if self.frames_input else self.in_images
        return (img, self.in_ids, self.in_state, self.in_noise)

    def infer_host(self, images, token_ids, state, noise, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """End-to-end call from host memory: copy the observations in (pinned host
        buffers give asynchronous copies), replay the chunk graph, copy the actions
        [B, chunk, action_dim] fp32 back to ``out`` (pinned host) and wait for it."""
        self.load_inputs(images, token_ids, state, noise, non_blocking=True)
        res = self.replay()
        if out is None:
            out = torch.empty((self.batch, self.cfg.expert.chunk, self.cfg.expert.action_dim), dtype=torch.float32,
                              pin_memory=True)
        out.view(-1, self.cfg.expert.action_dim).copy_(res, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def infer_host_stream(self, batches, outs) -> list:
        """End-to-end inference over a sequence of host batches with the transfers
        overlapped: batch k+1's observations are copied host->device on a copy
        stream (into one of two device staging sets) while batch k computes, and
        each batch's actions are copied device->host into ``outs[k]`` (pinned)
        right after its chunk graph.  ``batches`` holds (images, token_ids, state,
        noise) tuples of pinned host tensors of one batch size; images are either
        uint8 camera frames [B, H, W, 3] or bf16 images [B, 3, S, S] in [-1, 1].  Returns ``outs``
        after the last copy completed."""
        n = len(batches)
        if n == 0:
            return outs
        B = batches[0][0].shape[0]
        self.allocate(B)
        self._image_buffer(batches[0][0])
        if self.graph is None or self.graph_batch != B:
            self.capture()
        key = (B, tuple(batches[0][0].shape), batches[0][0].dtype)
        if getattr(self, "_stage_key", None) != key:
            self._stage = [[torch.empty_like(t) for t in self._inputs()] for _ in range(2)]
            self._stage_key = key
            self._copy_stream = torch.cuda.Stream(self.device)
        comp = torch.cuda.current_stream(self.device)
        cs = self._copy_stream
        copied = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]

        def h2d(k):
            st = self._stage[k & 1]
            with torch.cuda.stream(cs):
                if k >= 2:
                    cs.wait_event(consumed[k & 1])
                imgs, ids, state, noise = batches[k]
                st[0].copy_(imgs, non_blocking=True)
                st[1].copy_(ids, non_blocking=True)
                st[2].copy_(state, non_blocking=True)
                st[3].copy_(noise.reshape(st[3].shape), non_blocking=True)
                copied[k & 1].record(cs)

        h2d(0)
        for k in range(n):
            if k + 1 < n:
                h2d(k + 1)
            st = self._stage[k & 1]
            comp.wait_event(copied[k & 1])
            for dst, src in zip(self._inputs(), st):
                dst.copy_(src, non_blocking=True)
            consumed[k & 1].record(comp)
            self.graph.replay()
            outs[k].view(-1, self.cfg.expert.action_dim).copy_(self.x_t, non_blocking=True)
        comp.synchronize()
        return outs

    def _capture_halves(self) -> None:
        """CUDA graphs of the two chunk halves for both K/V slots."""
        graphs = []
        for slot in (0, 1):
            self.action.slot = slot
            self.forward_front()  # warm-up
            self.forward_back()
            torch.cuda.synchronize(self.device)
            gf, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(gf):
                self.forward_front()
            with torch.cuda.graph(gb):
                self.forward_back()
            graphs.append((gf, gb))
        self.action.slot = 0
        torch.cuda.synchronize(self.device)
        self.ov_graphs = graphs
        self.ov_batch = self.batch

    def infer_overlapped(self, batches, outs) -> list:
        """Streamed inference that overlaps consecutive batches: batch k+1's vision
        tower, prefix and text layers (front half) run on one stream while batch
        k's 10-step action expert (back half) runs on another, on alternating
        slots of the expert's prefix K/V; host->device copies of batch k+2 run on a
        third.  Same inputs and outputs as infer_host_stream (pinned host
        batches, ``outs[k]`` receives batch k's actions) and the same results."""
        n = len(batches)
        if n == 0:
            return outs
        B = batches[0][0].shape[0]
        self.allocate(B)
        self._image_buffer(batches[0][0])
        if getattr(self, "ov_graphs", None) is None or self.ov_batch != B:
            self._capture_halves()
        key = (B, tuple(batches[0][0].shape), batches[0][0].dtype)
        if getattr(self, "_stage_key", None) != key:
            self._stage = [[torch.empty_like(t) for t in self._inputs()] for _ in range(2)]
            self._stage_key = key
            self._copy_stream = torch.cuda.Stream(self.device)
        if getattr(self, "_ov_streams", None) is None:
            self._ov_streams = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
        sf, sb = self._ov_streams
        cs = self._copy_stream
        main = torch.cuda.current_stream(self.device)
        sf.wait_stream(main)
        sb.wait_stream(main)
        cs.wait_stream(main)
        ev = lambda: torch.cuda.Event()  # noqa: E731
        copied, consumed, front_done, back_done = ([ev(), ev()] for _ in range(4))

        def h2d(k):
            st = self._stage[k & 1]
            with torch.cuda.stream(cs):
                if k >= 2:
                    cs.wait_event(consumed[k & 1])
                imgs, ids, state, noise = batches[k]
                st[0].copy_(imgs, non_blocking=True)
                st[1].copy_(ids, non_blocking=True)
                st[2].copy_(state, non_blocking=True)
                st[3].copy_(noise.reshape(st[3].shape), non_blocking=True)
                copied[k & 1].record(cs)

        h2d(0)
        if n > 1:
            h2d(1)
        for k in range(n):
            slot = k & 1
            with torch.cuda.stream(sf):
                sf.wait_event(copied[slot])
                for dst, src in zip(self._inputs(), self._stage[slot]):
                    dst.copy_(src, non_blocking=True)
                consumed[slot].record(sf)
                if k >= 2:
                    sf.wait_event(back_done[slot])  # the expert of batch k-2 has read this K/V slot
                self.ov_graphs[slot][0].replay()
                front_done[slot].record(sf)
            if k + 2 < n:
                h2d(k + 2)
            with torch.cuda.stream(sb):
                sb.wait_event(front_done[slot])
                self.ov_graphs[slot][1].replay()
                outs[k].view(-1, self.cfg.expert.action_dim).copy_(self.x_t, non_blocking=True)
                back_done[slot].record(sb)
        main.wait_stream(sb)
        main.wait_stream(sf)
        main.synchronize()
        return outs

    def infer(self, images, token_ids, state, noise, use_graph: bool = True) -> torch.Tensor:
        """Action chunks [B, chunk, action_dim] (fp32) for a batch of observations."""
        self.load_inputs(images, token_ids, state, noise)
        out = self.replay() if use_graph else self.forward_device()
        return out.view(self.batch, self.cfg.expert.chunk, self.cfg.expert.action_dim)
