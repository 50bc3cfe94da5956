"""ctypes binding of ``libdabsn_b200.so`` (the C ABI declared in
``include/dabsn_b200.h``).

The library is loaded lazily and only from this package's directory.  If it
is missing or a call fails, a ``RuntimeError`` is raised: there is no silent
fallback to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libdabsn_b200.so"

F32 = 0
BF16 = 1

STATUS = {
    0: "ok",
    1: "bad shape",
    2: "unsupported dtype",
    3: "launch failure",
    4: "unsupported configuration",
    5: "device wait timed out",
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int


class CoreParams(ctypes.Structure):
    """Mirror of ``dabsn_core_params``."""

    _fields_ = [
        (name, _vp)
        for name in (
            "beta",
            "log_kappa",
            "logit_recover",
            "k_s",
            "k_y",
            "k_b",
            "k_n",
            "k_bias",
            "r_s",
            "r_y",
            "r_b",
            "r_n",
            "r_bias",
            "logit_c_decay",
            "k_c",
            "r_c",
            "logit_alpha",
            "log_lambda",
            "logit_c_suppress",
        )
    ]


# name -> argtypes (restype is always int except where noted)
_SIGNATURES = {
    "dabsn_version": ([], ctypes.c_char_p),
    "dabsn_last_error": ([], ctypes.c_char_p),
    "dabsn_device_status": ([_i32], _i32),
    "dabsn_core_scan_fwd": (
        [_i32, _i64, _i64, _i64, _vp, _vp, _vp, ctypes.POINTER(CoreParams)] + [_vp] * 15,
        _i32,
    ),
    "dabsn_core_scan_bwd": (
        [_i32, _i64, _i64, _i64] + [_vp] * 7 + [ctypes.POINTER(CoreParams)] + [_vp] * 20,
        _i32,
    ),
    "dabsn_core_scan_wide_scratch_bytes": ([_i64], ctypes.c_size_t),
    "dabsn_core_scan_wide_fwd": (
        [_i64, _i64, _i64, _vp, _vp, _vp, ctypes.POINTER(CoreParams)] + [_vp] * 15
        + [ctypes.c_size_t, _vp],
        _i32,
    ),
    "dabsn_delta_ckpt_floats": ([_i64, _i64, _i64], ctypes.c_size_t),
    "dabsn_permanent_delta_fwd": ([_i32, _i64, _i64, _i64] + [_vp] * 6, _i32),
    "dabsn_permanent_delta_bwd": ([_i32, _i64, _i64, _i64] + [_vp] * 10, _i32),
    "dabsn_local_field_gather": ([_i32] + [_i64] * 5 + [_vp] * 4, _i32),
    "dabsn_local_field_scatter": ([_i32] + [_i64] * 5 + [_vp] * 5, _i32),
    "dabsn_linear_ce_ld": ([_i64], _i64),
    "dabsn_linear_ce_workspace_floats": ([_i64, _i64], ctypes.c_size_t),
    "dabsn_linear_ce_fwd": ([_i64, _i64, _i64] + [_vp] * 4 + [_i32, _i32] + [_vp] * 4, _i32),
    "dabsn_linear_ce_bwd": ([_i64, _i64, _i64] + [_vp] * 4 + [_i32, _i32] + [_vp] * 5 + [_i32, _vp], _i32),
    "dabsn_tp_buffer_bytes": ([_i64], ctypes.c_size_t),
    "dabsn_tp_alloc": ([ctypes.c_size_t, ctypes.POINTER(_vp)], _i32),
    "dabsn_tp_free": ([_vp], _i32),
    "dabsn_tp_ipc_handle": ([_vp, _vp], _i32),
    "dabsn_tp_ipc_open": ([_vp, ctypes.POINTER(_vp)], _i32),
    "dabsn_tp_ipc_close": ([_vp], _i32),
    "dabsn_core_scan_tp_fwd": (
        [_i64] * 5 + [_i32, _i32, ctypes.POINTER(_vp), ctypes.c_uint32,
                      ctypes.POINTER(ctypes.c_uint32), _vp, _vp, _vp, ctypes.POINTER(CoreParams)]
        + [_vp] * 14 + [_vp],
        _i32,
    ),
    "dabsn_core_scan_tp_bwd": (
        [_i64] * 5 + [_i32, _i32, ctypes.POINTER(_vp), ctypes.c_uint32,
                      ctypes.POINTER(ctypes.c_uint32)] + [_vp] * 7 + [ctypes.POINTER(CoreParams)]
        + [_vp] * 2 + [_i32] + [_vp] * 17 + [_vp],
        _i32,
    ),
    "dabsn_core_scan_wide_fwd_noalloc": (
        [_i64, _i64, _i64, _vp, _vp, _vp, ctypes.POINTER(CoreParams)] + [_vp] * 14 + [_vp],
        _i32,
    ),
    "dabsn_core_scan_wide_bwd": (
        [_i64, _i64, _i64] + [_vp] * 7 + [ctypes.POINTER(CoreParams)] + [_vp] * 2
        + [_i32, ctypes.c_uint32] + [_vp] * 18 + [ctypes.c_size_t, _vp],
        _i32,
    ),
    "dabsn_ce_logits_fwd": ([_i32, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp], _i32),
    "dabsn_ce_logits_bwd": ([_i32, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp], _i32),
    "dabsn_input_proj_fwd": ([_i64, _i64, _i64, _vp, _i64] + [_vp] * 6, _i32),
    "dabsn_input_proj_bwd": ([_i64, _i64, _i64, _vp, _i64] + [_vp] * 8, _i32),
    "dabsn_rec_grad": ([_i64, _i64, _vp, _i64] + [_vp] * 5, _i32),
    "dabsn_read_out_fwd": ([_i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64] + [_vp] * 6, _i32),
    "dabsn_read_out_bwd": ([_i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64] + [_vp] * 7, _i32),
    "dabsn_glue_blocks": ([_i64], _i64),
    "dabsn_read_out_grad_prep": ([_i64, _i64] + [_vp] * 8, _i32),
    "dabsn_colsum_bf16": ([_i64, _i64, _vp, _vp, _vp], _i32),
    "dabsn_long_chunk": ([], _i32),
    "dabsn_long_fwd": ([_i32, _i64, _i64, _i64] + [_vp] * 8, _i32),
    "dabsn_long_bwd": ([_i32, _i64, _i64, _i64] + [_vp] * 11, _i32),
    "dabsn_read_fwd": ([_i32, _i64, _i64, _i64, _i64, _i32, _i64] + [_vp] * 16, _i32),
    "dabsn_read_bwd": ([_i32, _i64, _i64, _i64, _i64, _i32, _i64] + [_vp] * 24, _i32),
    "dabsn_admission_fwd": ([_i32, _i64, _i64, _i64, _i32] + [_vp] * 7 + [_i32] + [_vp] * 9, _i32),
    "dabsn_bank_gather": ([_i32, _i64, _i64, _i64, _i64] + [_vp] * 7 + [_i32] + [_vp] * 9, _i32),
    "dabsn_admission_bwd": ([_i32, _i64, _i64, _i64, _i64] + [_vp] * 7 + [_i32] + [_vp] * 13, _i32),
    "dabsn_read_wide_ld": ([_i64], _i64),
    "dabsn_read_wide_fwd_workspace": ([_i64, _i64, _i64], ctypes.c_size_t),
    "dabsn_read_wide_bwd_workspace": ([_i64, _i64, _i64], ctypes.c_size_t),
    "dabsn_read_wide_fwd": ([_i64, _i64, _i64, _i64, _i32, _i64] + [_vp] * 16
                            + [ctypes.c_size_t, _vp], _i32),
    "dabsn_read_wide_bwd": ([_i64, _i64, _i64, _i64, _i32, _i64] + [_vp] * 25
                            + [ctypes.c_size_t, _vp], _i32),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the shared library (once) and bind every C-ABI signature.

    ``DABSN_B200_LIB`` names another build of the library to load instead
    (e.g. a diagnostic build compiled with ``-DDABSN_SCAN_TRACE``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("DABSN_B200_LIB", str(LIB_PATH)))
        if not path.exists():
            raise RuntimeError(
                f"dabsn_b200 native library not found at {LIB_PATH}; "
                "build it with `python -m dabsn_b200.build` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
    return _lib


def is_loaded() -> bool:
    return _lib is not None


def version() -> str:
    return load().dabsn_version().decode()


def device_status(reset: bool = False) -> int:
    """Bounded-wait status of the current device (0 = no timeout); syncs."""
    return int(load().dabsn_device_status(1 if reset else 0))


DEVICE_CODES = {
    3: "a bounded wait of the forward scan timed out",
    4: "a bounded wait of the reverse scan timed out",
    6: "a bounded wait of the tensor-core GEMM timed out",
    7: "a cross-entropy target lies outside [0, V) and is not ignore_index",
}


def raise_on_device_status() -> None:
    """Raise when an earlier launch recorded an error in the device's status
    word.

    Every device-side wait of this library is bounded; one that gives up
    records a code there and ends its launch early, so that launch's outputs
    are invalid.  The cross-entropy kernels record a target outside the
    vocabulary the same way (the reference raises on it).  The word is read
    (and cleared) here, at host points where the step synchronises anyway
    (the admitted bank's width read), so the error reaches the caller instead
    of passing silently.  Reading it synchronises the device."""
    code = device_status(reset=True)
    if code != 0:
        what = DEVICE_CODES.get(code, f"device status code {code}")
        raise RuntimeError(f"dabsn_b200: {what} in an earlier launch; its outputs are invalid")


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().dabsn_last_error().decode(errors="replace")
        raise RuntimeError(f"dabsn_b200 {what} failed ({STATUS.get(status, status)}): {msg}")
