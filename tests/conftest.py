"""Shared pytest configuration (reference counterpart: tests/conftest.py).

* Puts ``<root>/fused-attention-cuda_b200`` (the ``fused_attn`` package) and ``<root>`` (the
  ``oracle`` checker) on ``sys.path``.
* ``gpu`` marker: skipped automatically when ``torch.cuda.is_available()`` is False.
* ``make_qkv``: the reference's seeded generator (CPU ``torch.randn`` in q, k, v order).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "fused-attention-cuda_b200"
for p in (str(PKG_DIR), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

os.environ.setdefault("MPLBACKEND", "Agg")

GOLDEN_DIR = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200); auto-skipped when no CUDA device is present"
    )


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip_gpu = pytest.mark.skip(reason="no CUDA device (torch.cuda.is_available() is False)")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip_gpu)


@pytest.fixture(scope="session")
def device() -> torch.device:
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


# (B, H, N, D): the reference's GPU shape set (tests/conftest.py:74-80).
GPU_SHAPES = [
    (1, 1, 64, 64),
    (2, 4, 256, 64),
    (1, 2, 512, 128),
    (2, 2, 1024, 64),
    (1, 2, 2048, 64),
]


def shape_id(shape: tuple[int, int, int, int]) -> str:
    b, h, n, d = shape
    return f"B{b}_H{h}_N{n}_D{d}"


@pytest.fixture(params=GPU_SHAPES, ids=shape_id)
def gpu_shape(request: pytest.FixtureRequest) -> tuple[int, int, int, int]:
    return request.param


@pytest.fixture
def make_qkv():
    from fused_attn.workloads import make_qkv as _make

    return _make
