"""The drop-in tests need the reference package itself (``baseline/_ref``,
installed by ``__graft_entry__.build()``).  Their fixtures skip when it is
missing so a CPU-only checkout still runs; on a GPU box that would hide the
whole drop-in, so this test fails there instead.  It sorts after the other
GPU test files so a run that stops at the first failure has run them first."""

from __future__ import annotations

import pytest

from conftest import ROOT, reference_available


@pytest.mark.gpu
def test_reference_package_importable():
    assert reference_available(), (
        f"the reference package is not importable from {ROOT / 'baseline' / '_ref'}: run "
        "__graft_entry__.build() (pip-installs the reference there) before the GPU tests")
    import dabsn
    import dabsn.kernels  # noqa: F401

    assert hasattr(dabsn, "DABSNSequenceLM")
