"""Closed-loop PushT on the GPU path: N environments stepped on the host, their
camera frames rasterised on the GPU straight into the model's uint8 input
buffer, one SmolVLA action chunk per environment per model call.

The reference's demo (simulation/demo_cpu.py:423-487) renders each frame with
matplotlib (simulation/pusht_env.py:196-264), feeds it to a CPU torch model and
applies the first two action dimensions as end-effector moves (dx, dy), one per
environment step, re-planning when the chunk is used up.  Here:

* ``PushTBatch`` restates the environment's physics (pusht_env.py:29-194:
  T-shaped block, circular end effector, push impulse + torque on contact,
  velocity damping, workspace clamps) vectorised over N environments, float64
  numpy, with the reference's constants and its reset distribution;
* ``render_frames`` draws the scene of every environment on the GPU
  (``vla_pusht_render_u8``): background, target T outline, block T, end
  effector, as uint8 [N, S, S, 3] frames (the reference's matplotlib styling,
  trail and text overlay are not reproduced);
* ``closed_loop`` runs the loop: render -> SmolVLA.infer (camera frames
  resized / normalised on the GPU) -> actions[:, :, :2] -> physics.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib

WORKSPACE = 512.0
EE_RADIUS = 15.0
BLOCK_W = 80.0
BLOCK_H = 30.0
PUSH_COEFF = 0.15
FRICTION = 0.7


def t_shape(cx, cy, theta):
    """[N, 8, 2] vertices of the T polygon (bar BLOCK_W x BLOCK_H on top, stem of
    half the bar's thickness and 0.4 BLOCK_W below) rotated by theta about its
    centre (pusht_env.py:29-62)."""
    hw, hh = BLOCK_W / 2, BLOCK_H / 2
    sw, sh = BLOCK_H / 2, BLOCK_W * 0.4
    v = np.array([[-hw, hh], [hw, hh], [hw, -hh], [sw, -hh], [sw, -hh - sh], [-sw, -hh - sh], [-sw, -hh],
                  [-hw, -hh]])
    c, s = np.cos(theta)[:, None], np.sin(theta)[:, None]
    x = v[None, :, 0] * c - v[None, :, 1] * s + cx[:, None]
    y = v[None, :, 0] * s + v[None, :, 1] * c + cy[:, None]
    return np.stack([x, y], axis=-1)


def _inside(px, py, verts):
    """Even-odd ray casting per environment (pusht_env.py:65-76)."""
    n = verts.shape[1]
    inside = np.zeros(px.shape, dtype=bool)
    for i in range(n):
        j = (i - 1) % n
        xi, yi = verts[:, i, 0], verts[:, i, 1]
        xj, yj = verts[:, j, 0], verts[:, j, 1]
        with np.errstate(divide="ignore", invalid="ignore"):
            xcross = (xj - xi) * (py - yi) / (yj - yi) + xi
        hit = ((yi > py) != (yj > py)) & (px < xcross)
        inside ^= hit
    return inside


def _overlap(cx, cy, r, verts):
    """Circle / polygon overlap: centre inside, or an edge closer than r
    (pusht_env.py:79-101)."""
    hit = _inside(cx, cy, verts)
    n = verts.shape[1]
    for i in range(n):
        ax, ay = verts[:, i, 0], verts[:, i, 1]
        bx, by = verts[:, (i + 1) % n, 0], verts[:, (i + 1) % n, 1]
        dx, dy = bx - ax, by - ay
        ll = dx * dx + dy * dy
        t = np.clip(((cx - ax) * dx + (cy - ay) * dy) / np.maximum(ll, 1e-8), 0.0, 1.0)
        qx, qy = ax + t * dx, ay + t * dy
        hit |= (ll >= 1e-8) & ((cx - qx) ** 2 + (cy - qy) ** 2 < r * r)
    return hit


class PushTBatch:
    """N PushT environments (pusht_env.py:103-194), vectorised."""

    def __init__(self, n: int, seed=0):
        """Environment i is seeded with seed + i, or with seed[i] for a list."""
        self.n = n
        seeds = list(seed) if isinstance(seed, (list, tuple)) else [seed + i for i in range(n)]
        self.rngs = [np.random.default_rng(s) for s in seeds]
        self.reset()

    def reset(self) -> np.ndarray:
        n = self.n
        self.ee_x = np.full(n, WORKSPACE / 2)
        self.ee_y = np.full(n, WORKSPACE * 0.75)
        draws = np.array([[r.uniform(-50, 50), r.uniform(-50, 50), r.uniform(-0.3, 0.3)] for r in self.rngs])
        self.block_x = WORKSPACE / 2 + draws[:, 0]
        self.block_y = WORKSPACE / 2 + draws[:, 1]
        self.block_theta = draws[:, 2].copy()
        self.block_vx = np.zeros(n)
        self.block_vy = np.zeros(n)
        self.block_vtheta = np.zeros(n)
        self.target = np.array([WORKSPACE / 2, WORKSPACE * 0.35, 0.0])
        self.steps = 0
        return self.state()

    def state(self) -> np.ndarray:
        """[N, 5] float32: ee x, ee y, block x, block y (over WORKSPACE), block theta / pi."""
        return np.stack([self.ee_x / WORKSPACE, self.ee_y / WORKSPACE, self.block_x / WORKSPACE,
                         self.block_y / WORKSPACE, self.block_theta / np.pi], axis=1).astype(np.float32)

    def step(self, action: np.ndarray) -> np.ndarray:
        """action [N, 2] = end-effector (dx, dy)."""
        action = np.asarray(action, dtype=np.float64)
        ox, oy = self.ee_x, self.ee_y
        self.ee_x = np.clip(ox + action[:, 0], EE_RADIUS, WORKSPACE - EE_RADIUS)
        self.ee_y = np.clip(oy + action[:, 1], EE_RADIUS, WORKSPACE - EE_RADIUS)
        mdx, mdy = self.ee_x - ox, self.ee_y - oy
        hit = _overlap(self.ee_x, self.ee_y, EE_RADIUS, t_shape(self.block_x, self.block_y, self.block_theta))
        sx, sy = self.ee_x - self.block_x, self.ee_y - self.block_y
        d = np.maximum(np.sqrt(sx ** 2 + sy ** 2), 1e-6)
        ex = np.clip(self.ee_x + sx / d * 2.0, EE_RADIUS, WORKSPACE - EE_RADIUS)
        ey = np.clip(self.ee_y + sy / d * 2.0, EE_RADIUS, WORKSPACE - EE_RADIUS)
        self.ee_x = np.where(hit, ex, self.ee_x)
        self.ee_y = np.where(hit, ey, self.ee_y)
        self.block_vx = self.block_vx + np.where(hit, mdx * PUSH_COEFF, 0.0)
        self.block_vy = self.block_vy + np.where(hit, mdy * PUSH_COEFF, 0.0)
        rx, ry = self.ee_x - self.block_x, self.ee_y - self.block_y
        self.block_vtheta = self.block_vtheta + np.where(hit, (rx * mdy - ry * mdx) * 0.0001, 0.0)
        self.block_x = self.block_x + self.block_vx
        self.block_y = self.block_y + self.block_vy
        self.block_theta = self.block_theta + self.block_vtheta
        self.block_vx = self.block_vx * FRICTION
        self.block_vy = self.block_vy * FRICTION
        self.block_vtheta = self.block_vtheta * FRICTION
        margin = BLOCK_W / 2 + 10
        self.block_x = np.clip(self.block_x, margin, WORKSPACE - margin)
        self.block_y = np.clip(self.block_y, margin, WORKSPACE - margin)
        self.steps += 1
        return self.state()

    def scene(self) -> np.ndarray:
        """[N, 8] float32 scene of the renderer: ee x, ee y, block x, y, theta, target x, y, theta."""
        t = np.broadcast_to(self.target, (self.n, 3))
        return np.concatenate([np.stack([self.ee_x, self.ee_y, self.block_x, self.block_y, self.block_theta], 1), t],
                              axis=1).astype(np.float32)


def render_frames(scene: torch.Tensor, size: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rasterise [N, 8] float32 scenes (device tensor) into uint8 frames [N, size, size, 3]."""
    n = scene.shape[0]
    if out is None:
        out = torch.empty(n, size, size, 3, dtype=torch.uint8, device=scene.device)
    _lib.call("vla_pusht_render_u8", ctypes.c_void_p(scene.data_ptr()), n, size, ctypes.c_void_p(out.data_ptr()),
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return out


def closed_loop(model, n_envs: int, n_chunks: int, seed: int = 0, token_ids: Optional[torch.Tensor] = None,
                frame_size: int = 512, action_scale: float = 1.0) -> dict:
    """Drive ``n_envs`` PushT environments with ``model`` (a SmolVLA) for
    ``n_chunks`` action chunks each; returns the trajectories and timings."""
    cfg = model.cfg
    e, pf = cfg.expert, cfg.prefix
    dev = model.device
    env = PushTBatch(n_envs, seed)
    g = torch.Generator().manual_seed(seed)
    ids = (token_ids if token_ids is not None
           else torch.randint(0, pf.vocab, (n_envs, pf.text_tokens), generator=g, dtype=torch.int32)).to(dev)
    frames = torch.empty(n_envs, frame_size, frame_size, 3, dtype=torch.uint8, device=dev)
    states, chunk_ms = [env.state()], []
    for _ in range(n_chunks):
        st = np.zeros((n_envs, pf.state_dim), dtype=np.float32)
        st[:, :5] = env.state()
        noise = torch.randn(n_envs, e.chunk, e.action_dim, generator=g)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        render_frames(torch.from_numpy(env.scene()).to(dev), frame_size, frames)
        acts = model.infer(frames, ids, torch.from_numpy(st).to(dev), noise.to(dev))
        b.record()
        acts = acts[:, :, :2].float().cpu().numpy() * action_scale
        chunk_ms.append(a.elapsed_time(b))
        for k in range(e.chunk):
            states.append(env.step(acts[:, k]))
    return {"states": np.stack(states, 1), "chunk_ms": chunk_ms, "frames": frames}


def main(argv=None) -> None:
    """python -m vla_b200.pusht [--envs N] [--chunks K] [--out file.npz]: run the
    closed loop on cuda:0 with the full model (random seeded weights, as the
    reference's demo before tuning) and save the trajectories and last frames."""
    import argparse
    from . import weights as W
    from .configs import SmolVLACfg
    from .model import SmolVLA
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--envs", type=int, default=8)
    ap.add_argument("--chunks", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--action-scale", type=float, default=1.0)
    ap.add_argument("--out", default="pusht_rollout.npz")
    a = ap.parse_args(argv)
    cfg = SmolVLACfg()
    model = SmolVLA(cfg, W.smolvla_params(cfg, seed=a.seed), "cuda:0")
    res = closed_loop(model, a.envs, a.chunks, seed=a.seed, action_scale=a.action_scale)
    np.savez_compressed(a.out, states=res["states"], frames=res["frames"].cpu().numpy(),
                        chunk_ms=np.array(res["chunk_ms"]))
    print(f"{a.envs} environments x {a.chunks} chunks: {np.mean(res['chunk_ms'][1:] or res['chunk_ms']):.2f} ms "
          f"per chunk call (render + inference); saved {a.out}")


if __name__ == "__main__":
    main()
