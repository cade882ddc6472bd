"""Weights from safetensors checkpoints into the reference's ``params`` layout.

The reference generates random weights in place (vla/vla.py:229-301: Xavier
``1/sqrt(fan_in)`` matrices, [in, out] layout, ``params["Wq"] = W.T``); a real
deployment loads a trained SmolVLA checkpoint instead.  This module reads and
writes the safetensors container (an 8-byte little-endian header length, a JSON
header mapping each tensor name to dtype / shape / byte range, then the raw
little-endian tensor bytes) with numpy memory maps, and maps tensor names onto
the ``params`` dictionary that ``SmolVLA`` and the block drop-ins take:

* ``naming="params"``: the flat names of this library, e.g. ``text.3.Wq`` or
  ``patch.kernel``, in the params layout ([in, out] linear weights);
* ``naming="smolvla"``: the module names of the SmolVLA checkpoint
  (``model.vlm_with_expert.vlm.model.text_model.layers.3.self_attn.q_proj.weight``
  and so on), torch ``nn.Linear`` layout ([out, in]), transposed on load.

No GPU is touched here: tensors come back as CPU torch tensors (bf16 by
default) and ``SmolVLA(cfg, params)`` uploads them.
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
from typing import Dict, Iterable, Optional

import numpy as np
import torch

from .configs import SmolVLACfg

BF16 = torch.bfloat16

# safetensors dtype tag -> (numpy storage dtype, torch dtype)
_DTYPES = {
    "BF16": (np.uint16, torch.bfloat16),
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64),
    "I32": (np.int32, torch.int32),
    "I64": (np.int64, torch.int64),
    "U8": (np.uint8, torch.uint8),
}
_TAGS = {v[1]: k for k, v in _DTYPES.items()}


class CheckpointError(ValueError):
    pass


def read_safetensors(path: str, names: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """All (or the named) tensors of a safetensors file as CPU torch tensors.
    The file is memory-mapped; each tensor is copied out once."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise CheckpointError(f"{path}: shorter than the 8-byte header length")
        (hlen,) = struct.unpack("<Q", raw)
        if hlen > size - 8:
            raise CheckpointError(f"{path}: header length {hlen} exceeds the file")
        header = json.loads(f.read(hlen).decode("utf-8"))
    base = 8 + hlen
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    want = None if names is None else set(names)
    out = {}
    for name, meta in header.items():
        if name == "__metadata__" or (want is not None and name not in want):
            continue
        tag = meta["dtype"]
        if tag not in _DTYPES:
            raise CheckpointError(f"{path}: tensor {name}: unsupported dtype {tag}")
        npdt, tdt = _DTYPES[tag]
        a, b = meta["data_offsets"]
        shape = tuple(meta["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b - a != count * np.dtype(npdt).itemsize or base + b > size:
            raise CheckpointError(f"{path}: tensor {name}: byte range {a}..{b} does not match shape {shape}")
        arr = np.frombuffer(mm, dtype=npdt, count=count, offset=base + a).reshape(shape).copy()
        t = torch.from_numpy(arr)
        if tdt == torch.bfloat16:
            t = t.view(torch.int16).view(torch.bfloat16) if arr.dtype == np.uint16 else t
        out[name] = t
    if want is not None and want - set(out):
        raise CheckpointError(f"{path}: missing tensors {sorted(want - set(out))[:8]}")
    return out


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None) -> None:
    """Write CPU tensors as a safetensors file (tensors in name order, 8-byte aligned header)."""
    header = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _TAGS:
            raise CheckpointError(f"tensor {name}: unsupported dtype {t.dtype}")
        data = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        header[name] = {"dtype": _TAGS[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = dict(metadata)
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for d in blobs:
            f.write(d)


# ---------------------------------------------------------------------------
# name maps
# ---------------------------------------------------------------------------
_VLM = "model.vlm_with_expert.vlm.model."
_EXP = "model.vlm_with_expert.lm_expert."


def _smolvla_names(cfg: SmolVLACfg) -> Dict[str, tuple]:
    """params path -> (checkpoint name, transpose).  Linear weights are stored
    [out, in] in the checkpoint and [in, out] in params (transpose=True)."""
    m = {
        ("patch", "kernel"): (_VLM + "vision_model.embeddings.patch_embedding.weight", False),
        ("patch", "b_patch"): (_VLM + "vision_model.embeddings.patch_embedding.bias", False),
        ("patch", "pos_emb"): (_VLM + "vision_model.embeddings.position_embedding.weight", False),
        ("patch", "W_post_norm"): (_VLM + "vision_model.post_layernorm.weight", False),
        ("patch", "b_post_norm"): (_VLM + "vision_model.post_layernorm.bias", False),
        ("connector", "W"): (_VLM + "connector.modality_projection.proj.weight", True),
        ("embed",): (_VLM + "text_model.embed_tokens.weight", False),
        ("W_state",): ("model.state_proj.weight", True),
        ("W_action_in",): ("model.action_in_proj.weight", True),
        ("W_action_out",): ("model.action_out_proj.weight", True),
        ("W_exp_norm",): (_EXP + "norm.weight", False),
    }
    vis = {"Wq": ("self_attn.q_proj.weight", True), "Wk": ("self_attn.k_proj.weight", True),
           "Wv": ("self_attn.v_proj.weight", True), "Wo": ("self_attn.out_proj.weight", True),
           "bq": ("self_attn.q_proj.bias", False), "bk": ("self_attn.k_proj.bias", False),
           "bv": ("self_attn.v_proj.bias", False), "bo": ("self_attn.out_proj.bias", False),
           "W_up": ("mlp.fc1.weight", True), "b_up": ("mlp.fc1.bias", False),
           "W_down": ("mlp.fc2.weight", True), "b_down": ("mlp.fc2.bias", False),
           "W_norm_1": ("layer_norm1.weight", False), "b_norm_1": ("layer_norm1.bias", False),
           "W_norm_2": ("layer_norm2.weight", False), "b_norm_2": ("layer_norm2.bias", False)}
    for i in range(cfg.vision.layers):
        for k, (n, tr) in vis.items():
            m[("vision", i, k)] = (f"{_VLM}vision_model.encoder.layers.{i}.{n}", tr)
    llama = {"Wq": ("self_attn.q_proj.weight", True), "Wk": ("self_attn.k_proj.weight", True),
             "Wv": ("self_attn.v_proj.weight", True), "Wo": ("self_attn.o_proj.weight", True),
             "W_gate": ("mlp.gate_proj.weight", True), "W_up": ("mlp.up_proj.weight", True),
             "W_down": ("mlp.down_proj.weight", True), "W_norm_1": ("input_layernorm.weight", False),
             "W_norm_2": ("post_attention_layernorm.weight", False)}
    for i in range(cfg.text.layers):
        for k, (n, tr) in llama.items():
            m[("text", i, k)] = (f"{_VLM}text_model.layers.{i}.{n}", tr)
    for i in range(cfg.expert.layers):
        for k, (n, tr) in llama.items():
            if i % 2 == 1 and k in ("Wk", "Wv"):
                # cross layers project the text layer's K / V: the checkpoint's
                # k_proj / v_proj of those layers take the text kv width as input
                k = k + "_cross"
            m[("expert", i, k)] = (f"{_EXP}layers.{i}.{n}", tr)
    return m


def _with_layers(cfg: SmolVLACfg, text: int, vision: int, expert: int) -> SmolVLACfg:
    return dataclasses.replace(cfg, text=dataclasses.replace(cfg.text, layers=text),
                               vision=dataclasses.replace(cfg.vision, layers=vision),
                               expert=dataclasses.replace(cfg.expert, layers=expert))


def _params_names(cfg: SmolVLACfg) -> Dict[str, tuple]:
    """params path -> (flat name, transpose=False) for this library's own naming."""
    from . import weights as W
    ref = W.smolvla_params(_with_layers(cfg, 0, 0, 0), seed=0)
    m = {}
    for top, v in ref.items():
        if isinstance(v, dict):
            for k in v:
                m[(top, k)] = (f"{top}.{k}", False)
        elif not isinstance(v, list):
            m[(top,)] = (top, False)
    vis_keys = W.vision_block_params(cfg.vision).keys()
    for i in range(cfg.vision.layers):
        for k in vis_keys:
            m[("vision", i, k)] = (f"vision.{i}.{k}", False)
    for i in range(cfg.text.layers):
        for k in W.text_block_params(cfg.text).keys():
            m[("text", i, k)] = (f"text.{i}.{k}", False)
    for i in range(cfg.expert.layers):
        keys = (W.expert_self_params(cfg.expert) if i % 2 == 0 else W.expert_cross_params(cfg.expert)).keys()
        for k in keys:
            m[("expert", i, k)] = (f"expert.{i}.{k}", False)
    return m


def _name_map(cfg: SmolVLACfg, naming: str) -> Dict[str, tuple]:
    if naming == "smolvla":
        return _smolvla_names(cfg)
    if naming == "params":
        return _params_names(cfg)
    raise CheckpointError(f"unknown naming {naming!r} (use 'smolvla' or 'params')")


def params_from_tensors(tensors: Dict[str, torch.Tensor], cfg: SmolVLACfg, naming: str = "smolvla",
                        dtype=BF16) -> dict:
    """Build the ``params`` dictionary (the layout of vla_b200.weights.smolvla_params)
    from named checkpoint tensors.  Optional vision biases absent from the
    checkpoint are left out (the layers then use zero biases); every other
    tensor must be present with the configuration's shape."""
    from . import weights as W
    nm = _name_map(cfg, naming)
    shapes = W.smolvla_params(_with_layers(cfg, min(cfg.text.layers, 1), min(cfg.vision.layers, 1),
                                           min(cfg.expert.layers, 2)), seed=0)
    optional = {"bq", "bk", "bv", "bo", "b_up", "b_down", "b_patch"}
    params = {"patch": {}, "vision": [{} for _ in range(cfg.vision.layers)], "connector": {},
              "text": [{} for _ in range(cfg.text.layers)], "expert": [{} for _ in range(cfg.expert.layers)]}
    for path, (name, transpose) in nm.items():
        if name not in tensors:
            if path[-1] in optional:
                continue
            raise CheckpointError(f"checkpoint lacks {name} (params {'/'.join(map(str, path))})")
        t = tensors[name]
        t = t.t() if transpose else t
        if len(path) == 3:
            want = shapes[path[0]][min(path[1], 1 if path[0] == "expert" and path[1] % 2 else 0)][path[2]].shape
        elif len(path) == 2:
            want = shapes[path[0]][path[1]].shape
        else:
            want = shapes[path[0]].shape
        if tuple(t.shape) != tuple(want):
            raise CheckpointError(f"{name}: shape {tuple(t.shape)} where the configuration needs {tuple(want)}")
        t = t.to(dtype).contiguous()
        if len(path) == 3:
            params[path[0]][path[1]][path[2]] = t
        elif len(path) == 2:
            params[path[0]][path[1]] = t
        else:
            params[path[0]] = t
    return params


def tensors_from_params(params: dict, cfg: SmolVLACfg, naming: str = "params") -> Dict[str, torch.Tensor]:
    """The inverse of params_from_tensors: named tensors ready for write_safetensors."""
    out = {}
    for path, (name, transpose) in _name_map(cfg, naming).items():
        node = params
        try:
            for p in path:
                node = node[p]
        except (KeyError, IndexError):
            continue
        out[name] = (node.t() if transpose else node).contiguous()
    return out


def load_params(path: str, cfg: SmolVLACfg, naming: str = "smolvla", dtype=BF16) -> dict:
    """``params`` for SmolVLA(cfg, params) from a safetensors checkpoint."""
    wanted = {name for name, _ in _name_map(cfg, naming).values()}
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        present = set(json.loads(f.read(hlen).decode("utf-8")))
    return params_from_tensors(read_safetensors(path, names=wanted & present), cfg, naming, dtype)


def save_params(path: str, params: dict, cfg: SmolVLACfg, naming: str = "params") -> None:
    write_safetensors(path, tensors_from_params(params, cfg, naming), metadata={"format": "vla_b200." + naming})
