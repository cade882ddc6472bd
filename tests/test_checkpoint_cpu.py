"""The safetensors weight loader (no GPU): the container format round-trips and
agrees with the safetensors library where it is installed, SmolVLA checkpoint
names map onto the reference's params layout ([in, out] weights, reference
vla/vla.py:229-301) with the right transposes, and malformed or mismatched
checkpoints are rejected with a clear error."""
import os

import pytest
import torch

from vla_b200 import checkpoint as C
from vla_b200 import weights as W
from vla_b200.configs import tiny_cfg


def _flat(params, prefix=""):
    for k, v in (params.items() if isinstance(params, dict) else enumerate(params)):
        if isinstance(v, (dict, list)):
            yield from _flat(v, f"{prefix}{k}.")
        else:
            yield f"{prefix}{k}", v


def test_container_round_trip(tmp_path):
    ts = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.arange(7, dtype=torch.int32),
          "c": torch.randn(2, 2, 2), "d": torch.randint(0, 255, (4,), dtype=torch.uint8)}
    p = str(tmp_path / "x.safetensors")
    C.write_safetensors(p, ts, metadata={"k": "v"})
    back = C.read_safetensors(p)
    assert set(back) == set(ts)
    for k in ts:
        assert back[k].dtype == ts[k].dtype and torch.equal(back[k], ts[k])
    try:
        from safetensors.torch import load_file, save_file
    except ImportError:
        return
    lib = load_file(p)  # our writer, the library's reader
    assert all(torch.equal(lib[k], ts[k]) for k in ts)
    p2 = str(tmp_path / "y.safetensors")
    save_file(ts, p2)  # the library's writer, our reader
    ours = C.read_safetensors(p2)
    assert all(torch.equal(ours[k], ts[k]) for k in ts)


@pytest.mark.parametrize("naming", ["params", "smolvla"])
def test_params_round_trip(tmp_path, naming):
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=3)
    p = str(tmp_path / f"{naming}.safetensors")
    C.save_params(p, params, cfg, naming=naming)
    back = C.load_params(p, cfg, naming=naming)
    a, b = dict(_flat(params)), dict(_flat(back))
    assert set(a) == set(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_smolvla_names_use_linear_layout(tmp_path):
    """Checkpoint linear weights are nn.Linear [out, in]; params hold [in, out]."""
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=4)
    ts = C.tensors_from_params(params, cfg, naming="smolvla")
    q = ts["model.vlm_with_expert.vlm.model.text_model.layers.1.self_attn.q_proj.weight"]
    assert torch.equal(q, params["text"][1]["Wq"].t())
    kc = ts["model.vlm_with_expert.lm_expert.layers.1.self_attn.k_proj.weight"]
    assert torch.equal(kc, params["expert"][1]["Wk_cross"].t())
    assert torch.equal(ts["model.state_proj.weight"], params["W_state"].t())
    conv = ts["model.vlm_with_expert.vlm.model.vision_model.embeddings.patch_embedding.weight"]
    assert torch.equal(conv, params["patch"]["kernel"])  # conv kernels keep their layout


def test_mismatches_are_rejected(tmp_path):
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=5)
    ts = C.tensors_from_params(params, cfg, naming="smolvla")
    name = "model.vlm_with_expert.vlm.model.text_model.layers.0.mlp.down_proj.weight"
    bad = dict(ts)
    bad[name] = bad[name][:, :-16]
    with pytest.raises(C.CheckpointError, match="shape"):
        C.params_from_tensors(bad, cfg, naming="smolvla")
    missing = {k: v for k, v in ts.items() if "layers.2.self_attn.o_proj" not in k or "text_model" not in k}
    with pytest.raises(C.CheckpointError, match="lacks"):
        C.params_from_tensors(missing, cfg, naming="smolvla")
    # vision biases are optional: without them the layers use zero biases
    nob = {k: v for k, v in ts.items()
           if not (k.endswith(".bias") and "encoder.layers" in k and ("self_attn" in k or "mlp" in k))}
    got = C.params_from_tensors(nob, cfg, naming="smolvla")
    assert "bq" not in got["vision"][0] and "W_norm_1" in got["vision"][0]
    p = str(tmp_path / "trunc.safetensors")
    C.write_safetensors(p, {"a": torch.zeros(64)})
    with open(p, "r+b") as f:
        f.truncate(os.path.getsize(p) - 8)
    with pytest.raises(C.CheckpointError):
        C.read_safetensors(p)
