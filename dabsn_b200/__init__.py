"""dabsn_b200 — B200 (sm_100a) CUDA backend for the DABSN scan + read hot path.

Plugs in behind the reference library's ``dabsn.kernels`` surface:

    import dabsn, dabsn_b200
    dabsn_b200.install()                      # optional: hook dabsn.kernels.enable/status
    dabsn.kernels.enable("cuda", required=True)   # or dabsn_b200.enable(required=True)

after which ``DABSNModel``, ``DABSNSequenceLM``, ``train_step`` and the
checkpoint code run unchanged on the B200 kernels.  The kernels themselves
are a C-ABI shared library (``include/dabsn_b200.h``) loaded with ctypes;
``dabsn_b200.ops`` exposes them on torch tensors directly.
"""

from __future__ import annotations

from .backend import b200_status, enable, enable_b200, install, native_available, status

__all__ = ["b200_status", "enable", "enable_b200", "install", "native_available", "status"]
__version__ = "0.1.0"
