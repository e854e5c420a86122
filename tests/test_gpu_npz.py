"""``.npz`` model files with device-resident models (reference
kanforge/convert.py:313-325): ``save`` of a CUDA model and ``load(...,
device="cuda")`` move all arrays in one pinned batch and must give back the
same values as the per-tensor CPU path, bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN

import kanforge_b200 as kb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cuda_model_round_trip_bit_exact(tmp_path, dtype):
    torch.manual_seed(0)
    model = kb.KAN([64, 96, 8], kb.BSpline(6, 3), edge_scale=True, device="cuda", dtype=dtype)
    model[0].update_grid(torch.randn(2048, 64, device="cuda").to(dtype))
    kb.save(model, tmp_path / "m.npz")
    with np.load(tmp_path / "m.npz") as data:
        for k, v in model.state_dict().items():
            assert data[k].dtype == np.float64
            assert np.array_equal(data[k], v.detach().double().cpu().numpy()), k
    back = kb.load(tmp_path / "m.npz", device="cuda")
    for k, v in back.state_dict().items():
        assert v.device.type == "cuda" and torch.equal(v, model.state_dict()[k]), k
    cpu = kb.load(tmp_path / "m.npz")
    for k, v in cpu.state_dict().items():
        assert torch.equal(v, back.state_dict()[k].cpu()), k
    x = torch.randn(100, 64, device="cuda").to(dtype)
    assert torch.equal(back(x), model(x))


def test_reference_file_loads_onto_the_gpu():
    ref = kb.load(GOLDEN / "ref_model.npz")
    dev = kb.load(GOLDEN / "ref_model.npz", device="cuda")
    for k, v in ref.state_dict().items():
        assert torch.equal(dev.state_dict()[k].cpu(), v), k
