"""Shared test setup: the ``gpu`` marker, import paths and golden-fixture loaders."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels through the C-ABI")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as data:
        return {k: data[k] for k in data.files}


def golden_cases(data: dict) -> list[str]:
    return sorted({k.split("/")[0] for k in data})


def spec_of(data: dict, case: str) -> dict:
    spec = json.loads(str(data[f"{case}/spec"]))
    if "grid_range" in spec:
        spec["grid_range"] = tuple(spec["grid_range"])
    return spec


def params_of(data: dict, case: str) -> dict:
    pre = f"{case}/param/"
    return {k[len(pre):]: v for k, v in data.items() if k.startswith(pre)}


@pytest.fixture(scope="session")
def golden_bases():
    return load_golden("bases.npz")


@pytest.fixture(scope="session")
def golden_layers():
    return load_golden("layers.npz")


@pytest.fixture(scope="session")
def golden_prims():
    return load_golden("prims.npz")


@pytest.fixture(scope="session")
def golden_init():
    return load_golden("init.npz")
