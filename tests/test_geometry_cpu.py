"""Host check of the kernels' index arithmetic (``dabsn_b200/csrc/geometry.cuh``):
the persistent GEMM's tile order covers every tile once, the grid-wide
scan's cluster split delivers every partial sum once, in bounds, with the byte
count each receiving mbarrier expects, and the read's GEMMs never read a
region of the row kernels' [B, T, Np] planes that the row kernels skipped
(with a deliberately wrong store rule caught) (``tests/geometry_check.cpp``)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_kernel_index_arithmetic(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path / "geometry_check"
    subprocess.run([cxx, "-std=c++17", "-O1", f"-I{ROOT / 'dabsn_b200' / 'csrc'}",
                    str(ROOT / "tests" / "geometry_check.cpp"), "-o", str(exe)], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.startswith("ok"), res.stdout
