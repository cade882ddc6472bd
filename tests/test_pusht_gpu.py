"""The closed-loop PushT demo on the GPU path (reference simulation/demo_cpu.py:
423-487): the scene rasteriser against a numpy restatement of its drawing rule,
and whole chunks of the loop (render -> SmolVLA on camera frames -> physics)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _in_t(u, v, grow):
    bar = (np.abs(u) <= 40 + grow) & (np.abs(v) <= 15 + grow)
    stem = (np.abs(u) <= 7.5 + grow) & (v >= -47 - grow) & (v <= 15 + grow)
    return bar | stem


def _render_np(scene, S):
    """numpy restatement of render.cuh's rule (fp32)."""
    n = scene.shape[0]
    out = np.empty((n, S, S, 3), dtype=np.uint8)
    scale = np.float32(512.0 / S)
    c = (np.arange(S, dtype=np.float32) + np.float32(0.5)) * scale
    X, Yr = np.meshgrid(c, c)  # X[r, col] = x of column, Yr[r, col] = (r + 0.5) * scale
    Y = np.float32(512.0) - Yr
    for e in range(n):
        img = np.full((S, S, 3), 240, dtype=np.uint8)

        def frame(cx, cy, th):
            co, si = np.float32(np.cos(th)), np.float32(np.sin(th))
            dx, dy = X - np.float32(cx), Y - np.float32(cy)
            return co * dx + si * dy, co * dy - si * dx

        ee_x, ee_y, bx, by, bt, tx, ty, tt = scene[e]
        u, v = frame(tx, ty, tt)
        img[_in_t(u, v, 1.0) & ~_in_t(u, v, -1.0)] = (144, 238, 144)
        u, v = frame(bx, by, bt)
        inside = _in_t(u, v, 0.0)
        img[inside] = (44, 95, 138)
        img[inside & _in_t(u, v, -1.5)] = (74, 144, 217)
        d2 = (X - np.float32(ee_x)) ** 2 + (Y - np.float32(ee_y)) ** 2
        img[d2 <= 15.0 ** 2] = (204, 68, 68)
        img[d2 <= 13.5 ** 2] = (255, 107, 107)
        out[e] = img
    return out


def test_render_matches_numpy_rule(cuda):
    from vla_b200.pusht import PushTBatch, render_frames
    env = PushTBatch(4, seed=5)
    env.step(np.array([[0, -40.0], [10, -60], [-5, -80.0], [3, -100.0]]))
    scene = env.scene()
    scene[2, 4] = 0.7  # a clearly rotated block
    for S in (512, 96):
        got = render_frames(torch.from_numpy(scene).cuda(), S).cpu().numpy()
        ref = _render_np(scene, S)
        diff = (got != ref).any(-1).mean()
        assert diff < 2e-3, f"{diff:.4%} of pixels differ at S={S}"
        # every layer is present in the first frame
        colours = {tuple(p) for p in got[0].reshape(-1, 3)[::7]}
        for col in ((240, 240, 240), (74, 144, 217), (255, 107, 107)):
            assert col in colours


def test_closed_loop_chunks(cuda):
    from vla_b200 import weights as W
    from vla_b200.configs import tiny_cfg
    from vla_b200.model import SmolVLA
    from vla_b200.pusht import closed_loop
    cfg = tiny_cfg()
    model = SmolVLA(cfg, W.smolvla_params(cfg, seed=0), "cuda")
    res = closed_loop(model, n_envs=3, n_chunks=2, seed=4, frame_size=cfg.vision.image, action_scale=20.0)
    st = res["states"]
    assert st.shape == (3, 1 + 2 * cfg.expert.chunk, 5) and np.isfinite(st).all()
    assert (np.abs(st[:, -1, :2] - st[:, 0, :2]) > 1e-3).any(), "the end effector never moved"
    assert len(res["chunk_ms"]) == 2 and all(t > 0 for t in res["chunk_ms"])
    assert res["frames"].dtype == torch.uint8
