"""Generate golden outputs from the REFERENCE's own torch oracle code.

The reference modules cannot be imported as a whole here: each file imports
the Allo NPU toolchain (and torchtune) and builds NPU kernels at import time.
This script therefore parses the reference sources with ``ast`` and executes
only the pure-PyTorch / numpy oracle definitions it names, in a namespace that
supplies their module-level constants:

  TextEncoderBlock          vla/text_encoder_bf16.py:61-135
  ActionExpertSelfBlock     vla/action_expert_bf16.py:69-131
  ActionExpertCrossBlock    vla/action_expert_bf16.py:137-207
  masked_softmax_cpu        vla/action_expert_bf16.py:530-538
  AttentionExpertBlock      vla/llama_block_rope_bf16.py:60-131
  CrossAttentionBlock       vla/llama_block_rope_bf16.py:133-180
  MiniVit                   vla/vision_block_bf16.py:57-79
  SiglipVisionConfig/Embeddings  vla/vit_emb.py:19-47
  con_ref                   vla/vla.py:434-437
  PushTEnv (+ make_t_shape, point_in_polygon, circle_polygon_overlap)
                            simulation/pusht_env.py:29-194 (physics only;
                            its matplotlib rendering is not executed)

torchtune.modules.MultiHeadAttention is used by TextEncoderBlock only as a
holder of its q/k/v/output projections (the forward never calls it), so a
container stub stands in for it.

Weights and inputs come from vla_b200.weights (seeded, deterministic), so the
tests can regenerate them and need only the outputs stored here.  Run from the
repository root, in the build container where the reference is mounted:

    python tests/golden/make_golden.py /path/to/reference

Output: tests/golden/reference_oracle.npz (small shapes, fp32 outputs).
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vla-to-npu_b200"))
sys.path.insert(0, HERE)

from golden_cases import CASES, case_inputs  # noqa: E402


class _MHAHolder(nn.Module):
    """Stand-in for torchtune.modules.MultiHeadAttention used only as a container."""

    def __init__(self, *, q_proj, k_proj, v_proj, output_proj, **_kw):
        super().__init__()
        self.q_proj, self.k_proj, self.v_proj, self.output_proj = q_proj, k_proj, v_proj, output_proj


def load_defs(path: str, names, consts: dict) -> dict:
    src = open(path).read()
    tree = ast.parse(src)
    ns = {"torch": torch, "nn": nn, "F": F, "np": np, "MultiHeadAttention": _MHAHolder,
          "dataclass": __import__("dataclasses").dataclass,
          "NP_DTYPE": __import__("ml_dtypes").bfloat16}
    ns.update(consts)
    found = set()
    for node in tree.body:
        if isinstance(node, (ast.ClassDef, ast.FunctionDef)) and node.name in names:
            seg = ast.get_source_segment(src, node)
            if node.decorator_list:
                seg = "\n".join("@" + ast.get_source_segment(src, d) for d in node.decorator_list) + "\n" + seg
            exec(compile(seg, path, "exec"), ns)
            found.add(node.name)
    missing = set(names) - found
    if missing:
        raise RuntimeError(f"{path}: definitions not found: {missing}")
    return ns


def _set_linear(lin: nn.Linear, w_in_out: torch.Tensor):
    lin.weight.data = w_in_out.float().t().contiguous()


def run(ref_root: str) -> dict:
    out = {}
    for name, case in CASES.items():
        kind = case["kind"]
        inp = case_inputs(name)
        p = inp["params"]
        c = case["consts"]
        if kind == "text":
            ns = load_defs(os.path.join(ref_root, "vla/text_encoder_bf16.py"), ["TextEncoderBlock"], c)
            m = ns["TextEncoderBlock"]().eval()
            _set_linear(m.attn.q_proj, p["Wq"]); _set_linear(m.attn.k_proj, p["Wk"])
            _set_linear(m.attn.v_proj, p["Wv"]); _set_linear(m.attn.output_proj, p["Wo"])
            _set_linear(m.gate_proj, p["W_gate"]); _set_linear(m.up_proj, p["W_up"])
            _set_linear(m.down_proj, p["W_down"])
            m.ln_1.weight.data = p["W_norm_1"].float(); m.ln_2.weight.data = p["W_norm_2"].float()
        elif kind in ("expert_self", "expert_cross"):
            cls = "ActionExpertSelfBlock" if kind == "expert_self" else "ActionExpertCrossBlock"
            ns = load_defs(os.path.join(ref_root, "vla/action_expert_bf16.py"), [cls], c)
            m = ns[cls]().eval()
            _set_linear(m.q_proj, p["Wq"])
            _set_linear(m.k_proj, p["Wk"] if kind == "expert_self" else p["Wk_cross"])
            _set_linear(m.v_proj, p["Wv"] if kind == "expert_self" else p["Wv_cross"])
            _set_linear(m.o_proj, p["Wo"]); _set_linear(m.gate_proj, p["W_gate"])
            _set_linear(m.up_proj, p["W_up"]); _set_linear(m.down_proj, p["W_down"])
            m.ln_1.weight.data = p["W_norm_1"].float(); m.ln_2.weight.data = p["W_norm_2"].float()
        elif kind in ("llama_rope", "cross_attn"):
            cls = "AttentionExpertBlock" if kind == "llama_rope" else "CrossAttentionBlock"
            ns = load_defs(os.path.join(ref_root, "vla/llama_block_rope_bf16.py"), [cls], c)
            m = ns[cls]().eval()
            a = m.attn if kind == "llama_rope" else m
            _set_linear(a.q_proj, p["Wq"]); _set_linear(a.k_proj, p["Wk"]); _set_linear(a.v_proj, p["Wv"])
            _set_linear(m.attn.output_proj if kind == "llama_rope" else m.o_proj, p["Wo"])
            _set_linear(m.gate_proj, p["W_gate"]); _set_linear(m.up_proj, p["W_up"])
            _set_linear(m.down_proj, p["W_down"])
            m.ln_1.weight.data = p["W_norm_1"].float(); m.ln_2.weight.data = p["W_norm_2"].float()
        elif kind == "minivit":
            ns = load_defs(os.path.join(ref_root, "vla/vision_block_bf16.py"), ["MiniVit"], c)
            torch.manual_seed(0)
            m = ns["MiniVit"]().eval()
            E = c["EMBD"]
            m.attn.in_proj_weight.data = torch.cat([p["Wq"].float().t(), p["Wk"].float().t(), p["Wv"].float().t()], 0)
            m.attn.out_proj.weight.data = p["Wo"].float().t().contiguous()
            _set_linear(m.ffn_up, p["W_up"]); _set_linear(m.ffn_down, p["W_down"])
            m.ln_1.weight.data = p["W_norm_1"].float(); m.ln_1.bias.data = p["b_norm_1"].float()
            m.ln_2.weight.data = p["W_norm_2"].float(); m.ln_2.bias.data = p["b_norm_2"].float()
            assert m.attn.in_proj_bias.abs().sum() == 0 and E == p["Wq"].shape[0]
        elif kind == "siglip_emb":
            ns = load_defs(os.path.join(ref_root, "vla/vit_emb.py"), ["SiglipVisionConfig", "SiglipVisionEmbeddings"], c)
            cfg = ns["SiglipVisionConfig"](num_channels=3, embed_dim=c["EMBED"], image_size=c["IMAGE"],
                                           patch_size=c["PATCH"])
            m = ns["SiglipVisionEmbeddings"](cfg).eval()
            m.patch_embedding.weight.data = p["kernel"].float()
            m.patch_embedding.bias.data = p["b_patch"].float()
            m.position_embedding.weight.data = p["pos_emb"].float()
        elif kind == "con_ref":
            ns = load_defs(os.path.join(ref_root, "vla/vla.py"), ["con_ref"], c)
            x = inp["x"].float().numpy()
            y = ns["con_ref"](x, {"W": p["W"].float().numpy()})
            out[name] = np.asarray(y, dtype=np.float32)
            continue
        elif kind == "pusht":
            ns = load_defs(os.path.join(ref_root, "simulation/pusht_env.py"),
                           ["make_t_shape", "point_in_polygon", "circle_polygon_overlap", "PushTEnv"], c)
            for seed in inp["seeds"]:
                env = ns["PushTEnv"](seed=seed)
                states, actions = [env.get_state()], []
                rng = np.random.default_rng(1000 + seed)
                for t in range(inp["steps"]):
                    # head for the block, then push through it, with noise: plenty of contacts
                    to_b = np.array([env.block_x - env.ee_x, env.block_y - env.ee_y])
                    a = to_b / max(np.linalg.norm(to_b), 1e-6) * 6.0 + rng.normal(0, 0.5, 2)
                    actions.append(a)
                    states.append(env.step(a))
                out[f"{name}.{seed}.actions"] = np.array(actions, dtype=np.float64)
                out[f"{name}.{seed}.states"] = np.array(states, dtype=np.float32)
            continue
        elif kind == "masked_softmax_cpu":
            ns = load_defs(os.path.join(ref_root, "vla/action_expert_bf16.py"), ["masked_softmax_cpu"], c)
            import ml_dtypes
            s = inp["x"].float().numpy().astype(ml_dtypes.bfloat16)
            out[name] = ns["masked_softmax_cpu"](s).astype(np.float32)
            continue
        else:
            raise ValueError(kind)

        for attr, val in case.get("patch", {}).items():
            obj_path, field = attr.rsplit(".", 1)
            obj = m
            for part in obj_path.split("."):
                obj = getattr(obj, part)
            setattr(obj, field, val)
        if case.get("rope_theta") is not None:
            hd = c["HEAD_DIM"]
            m.rope_timescale = case["rope_theta"] ** ((2.0 / hd) * torch.arange(hd // 2, dtype=torch.float32))

        # TextEncoderBlock / ActionExpert*Block hard-cast the attention context to
        # bf16 (vla/text_encoder_bf16.py:126), so they only run as bf16 modules.
        dts = (("bf16", torch.bfloat16),) if kind in ("text", "expert_self", "expert_cross", "llama_rope",
                                                      "cross_attn") else (
            ("f32", torch.float32), ("bf16", torch.bfloat16))
        for dt_name, dt in dts:
            mm = m.to(dt)
            args = [a.to(dt) for a in inp["args"]]
            with torch.no_grad():
                y = mm(*args)
            if isinstance(y, tuple):
                for i, yi in enumerate(y):
                    out[f"{name}.{dt_name}.{i}"] = yi.float().numpy()
            else:
                out[f"{name}.{dt_name}"] = y.float().numpy()
    return out


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VLA_REFERENCE_ROOT", "")
    if not ref or not os.path.isdir(os.path.join(ref, "vla")):
        sys.exit("usage: make_golden.py <reference checkout root>")
    res = run(ref)
    path = os.path.join(HERE, "reference_oracle.npz")
    np.savez_compressed(path, **res)
    print(f"wrote {path}: {len(res)} arrays, {os.path.getsize(path)/1024:.0f} KiB")
