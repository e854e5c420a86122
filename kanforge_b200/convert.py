"""``.npz`` model files in the reference's format (kanforge/convert.py:108-325).

A file holds the arrays named like ``state_dict`` plus ``__spec__``, a JSON
string ``{"format": 1, "source": ..., "model": spec}``.  Files written by the
reference load here and files written here load in the reference, for the
layer types of the hot path: ``KANLinear``, ``GRKAN``, ``KAN`` and sequences of
those with ``Linear`` layers and standard activations.
"""

from __future__ import annotations

import functools
import json

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from .layers import GRKAN, KAN, KANLinear, rebuild_kan

ACTIVATIONS = ("identity", "silu", "gelu", "gelu_tanh", "tanh", "relu", "sigmoid")


def activation_name(act) -> str | None:
    """Portable name of an activation (None = absent) (convert.py:27-57)."""
    if act is None:
        return None
    if isinstance(act, functools.partial) and getattr(act.func, "__name__", "") == "gelu":
        return "gelu_tanh" if act.keywords.get("approximate", None) in (True, "tanh") else "gelu"
    cls = type(act).__name__.lower()
    fname = getattr(act, "__name__", "").lower()
    for name in (cls, fname):
        if name in ("identity", "_identity"):
            return "identity"
        if name in ("silu", "swish"):
            return "silu"
        if name in ("tanh", "relu", "sigmoid"):
            return name
    if "gelu" in cls or "gelu" in fname:
        approx = getattr(act, "approximate", None)
        return "gelu_tanh" if approx in ("tanh", True) else "gelu"
    raise ValueError(f"cannot convert activation {act!r}")


def make_activation(name: str | None):
    """torch callable for an activation name."""
    if name is None:
        return None
    table = {
        "identity": nn.Identity(),
        "silu": F.silu,
        "gelu": F.gelu,
        "gelu_tanh": functools.partial(F.gelu, approximate="tanh"),
        "tanh": nn.Tanh(),
        "relu": nn.ReLU(),
        "sigmoid": nn.Sigmoid(),
    }
    return table[name]


def _dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).replace("torch.", "")


def _layer_spec(layer: KANLinear):
    opt = layer.options
    spec = {
        "type": "GRKAN" if isinstance(layer, GRKAN) else "KANLinear",
        "in": layer.in_features,
        "out": layer.out_features,
        "basis": layer.basis.config(),
        "bias": bool(opt.bias),
        "base_activation": activation_name(opt.base_activation),
        "groups": opt.groups,
        "edge_scale": bool(opt.edge_scale),
        "edge_dropout": float(opt.edge_dropout),
        "backend": opt.backend,
        "dtype": _dtype_name(layer.coef),
    }
    return spec, {k: v for k, v in layer._export_full().items() if v is not None}


def to_spec(model):
    """(spec, arrays) of a model."""
    arrays: dict[str, np.ndarray] = {}

    def walk(m, prefix):
        if isinstance(m, KANLinear):
            spec, arr = _layer_spec(m)
            arrays.update({prefix + k: v for k, v in arr.items()})
            return spec
        if isinstance(m, KAN):
            return {"type": "KAN", "widths": list(m.widths), "layers": [walk(c, f"{prefix}{k}.") for k, c in enumerate(m)]}
        if isinstance(m, nn.Sequential):
            return {"type": "Sequential", "layers": [walk(c, f"{prefix}{k}.") for k, c in enumerate(m)]}
        if isinstance(m, nn.Linear):
            arrays[prefix + "weight"] = m.weight.detach().cpu().double().numpy()
            if m.bias is not None:
                arrays[prefix + "bias"] = m.bias.detach().cpu().double().numpy()
            return {"type": "Linear", "in": m.in_features, "out": m.out_features, "bias": m.bias is not None,
                    "dtype": _dtype_name(m.weight)}
        return {"type": "Activation", "name": activation_name(m)}

    return walk(model, ""), arrays


class _Lambda(nn.Module):
    def __init__(self, fn):
        super().__init__()
        self.fn = fn

    def forward(self, x):
        return self.fn(x)


def _build(spec, arrays, prefix=""):
    t = spec["type"]
    if t in ("KANLinear", "GRKAN"):
        layer = KANLinear(
            spec["in"], spec["out"], spec["basis"], bias=spec["bias"], base_activation=make_activation(spec["base_activation"]),
            groups=spec["groups"], edge_scale=spec["edge_scale"], edge_dropout=spec["edge_dropout"],
            backend=spec["backend"], dtype=getattr(torch, spec.get("dtype", "float32")),
        )
        state = {k[len(prefix):]: v for k, v in arrays.items() if k.startswith(prefix) and "." not in k[len(prefix):]}
        layer._import_full(state)
        return layer
    if t in ("KAN", "Sequential"):
        children = [_build(c, arrays, f"{prefix}{k}.") for k, c in enumerate(spec["layers"])]
        return rebuild_kan(children) if t == "KAN" else nn.Sequential(*children)
    if t == "Linear":
        lin = nn.Linear(spec["in"], spec["out"], bias=spec["bias"], dtype=getattr(torch, spec.get("dtype", "float32")))
        with torch.no_grad():
            lin.weight.copy_(torch.as_tensor(arrays[prefix + "weight"]))
            if spec["bias"]:
                lin.bias.copy_(torch.as_tensor(arrays[prefix + "bias"]))
        return lin
    if t == "Activation":
        act = make_activation(spec["name"])
        return act if isinstance(act, nn.Module) else _Lambda(act)
    raise ValueError(f"layer type {t!r} is not part of the kanforge_b200 hot path")


def from_spec(spec, arrays):
    return _build(spec, arrays)


def save(model, path) -> None:
    """One ``.npz``: arrays plus the JSON spec (convert.py:313-317)."""
    spec, arrays = to_spec(model)
    np.savez(path, __spec__=np.array(json.dumps({"format": 1, "source": "torch", "model": spec})), **arrays)


def load(path, backend: str = "torch"):
    """Load a file written by ``save`` here or by the reference (convert.py:319-325)."""
    if backend != "torch":
        raise ValueError("kanforge_b200 loads models for torch only")
    with np.load(path, allow_pickle=False) as data:
        meta = json.loads(str(data["__spec__"]))
        arrays = {k: data[k] for k in data.files if k != "__spec__"}
    return from_spec(meta["model"], arrays)
