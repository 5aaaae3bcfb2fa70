"""Shared test configuration: the ``gpu`` marker and fixture paths."""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The PyTorch references in the GPU tests must be true fp32 (cuDNN convolutions
# default to TF32 on this hardware).
torch.backends.cudnn.allow_tf32 = False
torch.backends.cuda.matmul.allow_tf32 = False


def reference_path() -> str | None:
    """Checkout of the reference ``unblend`` project for the tests that import it.

    ``UNBLEND_REFERENCE`` names it; without the variable, a ``reference``
    directory beside this repository is used when present. ``None`` when
    neither exists (those tests skip).
    """
    path = os.environ.get("UNBLEND_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    return path if os.path.isdir(os.path.join(path, "unblend")) else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name: str) -> dict:
    """Load a committed golden fixture."""
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / rms(b)."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / (b.pow(2).mean().sqrt() + 1e-30))
