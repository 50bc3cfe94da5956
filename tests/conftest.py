"""Shared pytest setup: the ``gpu`` marker, import paths and fixture loading."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for entry in (str(ROOT), str(ROOT / "oracle")):
    if entry not in sys.path:
        sys.path.insert(0, entry)
os.environ.setdefault("DABSN_SILENCE_ROUTING", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def reference_available() -> bool:
    """True when the installed reference package (``baseline/_ref``) imports."""
    ref = ROOT / "baseline" / "_ref"
    if ref.is_dir() and str(ref) not in sys.path:
        sys.path.append(str(ref))
    try:
        import dabsn  # noqa: F401
    except Exception:
        return False
    return True


def max_rel_err(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """max |a-e| / max(|e|_inf, tiny): the relative error the tolerances use."""
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    denom = max(float(e.abs().max()), 1e-12) if e.numel() else 1.0
    return float((a - e).abs().max()) / denom if e.numel() else 0.0
