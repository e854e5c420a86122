"""``.npz`` model files in the reference's format (kanforge/convert.py:108-325).

A file holds the arrays named like ``state_dict`` plus ``__spec__``, a JSON
string ``{"format": 1, "source": ..., "model": spec}``.  Files written by the
reference load here and files written here load in the reference, for the
layer types of the hot path: ``KANLinear``, ``GRKAN``, ``KAN`` and sequences of
those with ``Linear`` layers and standard activations.

Arrays are float64 in the file, as the reference writes them.  ``save`` copies
device tensors to the host in their own dtype (the fewest bytes over PCIe)
and widens them there; writing the file dominates (2.7 GB in 1.56 s for a
4096 x 4096 Chebyshev(12) layer, the same as a per-tensor copy).
``load(..., device=cuda)`` streams the file's float64 arrays through two
alternating 64 MiB pinned buffers to the GPU and narrows each to its
parameter's dtype there: 1.55 s against 5.45 s for loading on the host and
moving the model (same layer), with pinned memory bounded at 128 MiB.
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


STAGING_BYTES = 64 << 20  # each of the two pinned staging buffers of the device copies


class _Staging:
    """Two pinned host buffers that alternate: while one chunk crosses PCIe
    asynchronously on a side stream, the other is copied to or from NumPy."""

    def __init__(self, device: torch.device):
        n = STAGING_BYTES // 8
        self.bufs = [torch.empty(n, dtype=torch.float64, pin_memory=True) for _ in range(2)]
        self.host = [b.numpy() for b in self.bufs]
        self.events: list = [None, None]
        self.stream = torch.cuda.Stream(device)
        self.stream.wait_stream(torch.cuda.current_stream(device))
        self.n = n

    def wait(self, k: int) -> None:
        if self.events[k] is not None:
            self.events[k].synchronize()
            self.events[k] = None

    def record(self, k: int) -> None:
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self.events[k] = ev


def _host_float64(tensors: dict[str, torch.Tensor]) -> dict[str, np.ndarray]:
    """float64 NumPy copies of tensors.  Device tensors cross PCIe in their own
    dtype (a quarter of the float64 bytes for bf16, half for float32) and are
    widened on the host."""
    return {name: t.detach().cpu().to(torch.float64).numpy() for name, t in tensors.items()}


def _device_float64(arrays: dict[str, np.ndarray], device: torch.device) -> dict[str, torch.Tensor]:
    """The arrays as float64 tensors on a CUDA device, streamed through the two
    pinned buffers chunk by chunk."""
    st = _Staging(device)
    out = {}
    k = 0
    for name, arr in arrays.items():
        a = np.ascontiguousarray(arr, dtype=np.float64)
        flat = a.reshape(-1)
        dev = torch.empty(a.size, dtype=torch.float64, device=device)
        for off in range(0, a.size, st.n):
            m = min(st.n, a.size - off)
            st.wait(k)
            st.host[k][:m] = flat[off:off + m]
            with torch.cuda.stream(st.stream):
                dev[off:off + m].copy_(st.bufs[k][:m], non_blocking=True)
            st.record(k)
            k ^= 1
        out[name] = dev.view(a.shape)
    torch.cuda.current_stream(device).wait_stream(st.stream)
    for k in (0, 1):
        st.wait(k)
    return out


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
    own = {**dict(layer.named_parameters(recurse=False)), **dict(layer.named_buffers(recurse=False))}
    return spec, own


def to_spec(model):
    """(spec, arrays) of a model, arrays float64 NumPy (convert.py:141-172)."""
    tensors: dict[str, torch.Tensor] = {}

    def walk(m, prefix):
        if isinstance(m, KANLinear):
            spec, own = _layer_spec(m)
            tensors.update({prefix + k: v for k, v in own.items()})
            return spec
        if isinstance(m, KAN):
            return {"type": "KAN", "widths": list(m.widths), "layers": [walk(c, f"{prefix}{k}.") for k, c in enumerate(m)]}
        if isinstance(m, nn.Sequential):
            return {"type": "Sequential", "layers": [walk(c, f"{prefix}{k}.") for k, c in enumerate(m)]}
        if isinstance(m, nn.Linear):
            tensors[prefix + "weight"] = m.weight
            if m.bias is not None:
                tensors[prefix + "bias"] = m.bias
            return {"type": "Linear", "in": m.in_features, "out": m.out_features, "bias": m.bias is not None,
                    "dtype": _dtype_name(m.weight)}
        return {"type": "Activation", "name": activation_name(m)}

    spec = walk(model, "")
    return spec, _host_float64(tensors)


class _Lambda(nn.Module):
    def __init__(self, fn):
        super().__init__()
        self.fn = fn

    def forward(self, x):
        return self.fn(x)


def _build(spec, arrays, prefix="", device=None):
    t = spec["type"]
    if t in ("KANLinear", "GRKAN"):
        layer = KANLinear(
            spec["in"], spec["out"], spec["basis"], bias=spec["bias"], base_activation=make_activation(spec["base_activation"]),
            groups=spec["groups"], edge_scale=spec["edge_scale"], edge_dropout=spec["edge_dropout"],
            backend=spec["backend"], dtype=getattr(torch, spec.get("dtype", "float32")), device=device,
        )
        state = {k[len(prefix):]: v for k, v in arrays.items() if k.startswith(prefix) and "." not in k[len(prefix):]}
        layer._import_full(state)
        return layer
    if t in ("KAN", "Sequential"):
        children = [_build(c, arrays, f"{prefix}{k}.", device) for k, c in enumerate(spec["layers"])]
        return rebuild_kan(children) if t == "KAN" else nn.Sequential(*children)
    if t == "Linear":
        lin = nn.Linear(spec["in"], spec["out"], bias=spec["bias"], dtype=getattr(torch, spec.get("dtype", "float32")),
                        device=device)
        with torch.no_grad():
            lin.weight.copy_(torch.as_tensor(arrays[prefix + "weight"]))
            if spec["bias"]:
                lin.bias.copy_(torch.as_tensor(arrays[prefix + "bias"]))
        return lin
    if t == "Activation":
        act = make_activation(spec["name"])
        return act if isinstance(act, nn.Module) else _Lambda(act)
    raise ValueError(f"layer type {t!r} is not part of the kanforge_b200 hot path")


def from_spec(spec, arrays, device=None):
    """The model of ``spec`` with ``arrays`` loaded, on ``device`` (default CPU)."""
    device = None if device is None else torch.device(device)
    if device is not None and device.type == "cuda":
        arrays = _device_float64(arrays, device)
    return _build(spec, arrays, device=device)


def save(model, path) -> None:
    """One ``.npz``: arrays plus the JSON spec (convert.py:313-317)."""
    spec, arrays = to_spec(model)
    np.savez(path, __spec__=np.array(json.dumps({"format": 1, "source": "torch", "model": spec})), **arrays)


def load(path, backend: str = "torch", device=None):
    """Load a file written by ``save`` here or by the reference (convert.py:319-325),
    onto ``device`` (default CPU, like the reference)."""
    if backend != "torch":
        raise ValueError("kanforge_b200 loads models for torch only")
    with np.load(path, allow_pickle=False) as data:
        meta = json.loads(str(data["__spec__"]))
        arrays = {k: data[k] for k in data.files if k != "__spec__"}
    return from_spec(meta["model"], arrays, device)
