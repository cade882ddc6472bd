"""Host-array plumbing for the reference-compatible entry points.

The reference's block builders and per-op harnesses take numpy arrays
(``ml_dtypes.bfloat16`` or float32) and return numpy bf16 arrays, with
weights in a ``params`` dict ([in, out] layout).  These helpers move such
arrays to the GPU (caching uploaded weights by identity, so that calling a
block repeatedly with the same ``params`` uploads them once) and bring
results back in the caller's array type.
"""
from __future__ import annotations

import weakref
from typing import Any, Callable, Dict, Tuple

import numpy as np
import torch

BF16 = torch.bfloat16


def is_numpy(x) -> bool:
    return isinstance(x, np.ndarray)


def to_device(x, dtype=BF16, device="cuda") -> torch.Tensor:
    """numpy (any float dtype, incl. ml_dtypes.bfloat16) or torch -> contiguous CUDA tensor."""
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=dtype).contiguous()
    a = np.asarray(x)
    if a.dtype.name == "bfloat16":
        t = torch.from_numpy(a.view(np.uint16).astype(np.int16, copy=False)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(device=device).to(dtype).contiguous()


def to_host_like(t: torch.Tensor, like) -> Any:
    """Return a CUDA result as the caller's type: numpy bf16 (ml_dtypes) for numpy
    inputs, a CPU torch tensor for torch inputs."""
    if is_numpy(like):
        import ml_dtypes
        u = t.detach().to(BF16).contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
        return u.view(ml_dtypes.bfloat16)
    return t.detach().cpu()


class _Cache:
    """Device copies of host weights keyed by (id, shape, transform); entries die with
    their host array when it is weak-referenceable, else live for the process."""

    def __init__(self):
        self._d: Dict[Tuple, torch.Tensor] = {}

    def get(self, key_obj, tag: str, make: Callable[[], torch.Tensor]) -> torch.Tensor:
        key = (id(key_obj), tag, getattr(key_obj, "shape", None), torch.cuda.current_device())
        t = self._d.get(key)
        if t is None:
            t = make()
            self._d[key] = t
            try:
                weakref.finalize(key_obj, self._d.pop, key, None)
            except TypeError:
                pass
        return t


WEIGHTS = _Cache()


def weight_kmajor(w_in_out, tag: str = "kmajor") -> torch.Tensor:
    """Reference [in, out] weight -> cached device [out, in] (K-major) bf16."""
    return WEIGHTS.get(w_in_out, tag, lambda: to_device(w_in_out).t().contiguous())


def vector(v, tag: str = "vec") -> torch.Tensor:
    return WEIGHTS.get(v, tag, lambda: to_device(v))
