"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol the public header declares, and the backend refuses loudly when the
CUDA path cannot run."""

from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import ROOT, reference_available

HEADER = ROOT / "include" / "dabsn_b200.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(dabsn_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = _declared_functions()
    for required in ("dabsn_core_scan_fwd", "dabsn_core_scan_bwd", "dabsn_read_fwd",
                     "dabsn_read_bwd", "dabsn_long_fwd", "dabsn_long_bwd"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from dabsn_b200 import _native

    lib = ctypes.CDLL(str(_native.LIB_PATH))
    for name in _declared_functions():
        assert hasattr(lib, name), name
    # the ctypes binding covers exactly the declared surface
    assert set(_native.EXPORTED) >= set(_declared_functions())


def test_version_string_without_gpu():
    from dabsn_b200 import _native

    assert "sm_100a" in _native.version()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU refusal path")
def test_required_backend_fails_loudly_without_gpu():
    if not reference_available():
        pytest.skip("reference package not installed")
    import dabsn_b200

    ok, why = dabsn_b200.native_available()
    assert not ok and why
    with pytest.raises(RuntimeError, match="required"):
        dabsn_b200.enable_b200(required=True)
    assert dabsn_b200.enable_b200(required=False) == {
        "core_scan": False, "admitted_three_way_read": False, "long_memory": False}


def test_ops_reject_cpu_tensors():
    from dabsn_b200 import ops

    x = torch.zeros(1, 2, 4)
    with pytest.raises(TypeError):
        ops.core_scan_forward(x, x, torch.zeros(4, 4), torch.zeros(4, 4), [torch.zeros(4)] * 19,
                              torch.zeros(1, 4), torch.ones(1, 4), torch.zeros(1, 4))


def test_status_reports_b200_section():
    if not reference_available():
        pytest.skip("reference package not installed")
    import dabsn_b200

    st = dabsn_b200.status()
    assert "b200" in st and st["b200"]["arch"] == "sm_100a"
    assert "active_backend" in st
