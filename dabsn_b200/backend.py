"""Binding of the B200 kernels behind the reference's ``dabsn.kernels`` surface.

``enable(backend, required=...)`` mirrors ``dabsn.kernels.enable``
(src/dabsn/kernels/__init__.py:91-139): one explicit backend family per
process, ``required=True`` refuses missing support with ``RuntimeError``.
Enabling the ``"b200"`` family (also reached as ``"cuda"`` once
:func:`install` has hooked the reference module) does what
``enable_triton_kernels`` does for the Triton family (triton.py:486-510):

* ``dabsn::core_scan_batched`` gets the B200 CUDA kernel
  (``register_kernel("cuda")``) and the B200 reverse scan as its autograd
  formula (``torch.library.register_autograd``; CPU tensors keep the
  reference's own reverse);
* the CUDA admitted read that ``DABSNRead._admitted_read`` imports at call
  time (read.py:465) becomes the B200 flash read;
* the long-memory channel that ``DABSNRead._long_scan_from_state`` imports at
  call time (read.py:587) becomes the fused B200 long scan;
* the class flags that route the model onto these paths are set
  (``_cuda_native_enabled``, ``_long_native_enabled`` and the ``_required``
  twins).

Models, ``train_step`` and checkpoints run unchanged; nothing here edits the
reference's files.
"""

from __future__ import annotations

import os
import threading

import torch

from . import _native
from . import autograd as AG
from . import ops

_STATE: dict[str, object] = {"enabled": False, "required": False, "error": None}
_LOCK = threading.Lock()


def _reference():
    import dabsn  # noqa: F401  (the reference package)
    import dabsn.kernels as kernels
    import dabsn.kernels.batched_runtime as batched
    import dabsn.kernels.long as long_mod
    import dabsn.kernels.triton as triton_mod
    from dabsn.core import DABSNCore
    from dabsn.read import DABSNRead

    return kernels, batched, long_mod, triton_mod, DABSNCore, DABSNRead


def native_available() -> tuple[bool, str | None]:
    """Whether the CUDA library loads and a CUDA device is visible."""
    if not torch.cuda.is_available():
        return False, "CUDA is not available"
    try:
        _native.load()
    except Exception as exc:  # noqa: BLE001
        return False, f"{type(exc).__name__}: {exc}"
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        return False, f"sm_{major}{minor} device; the library is built for sm_100a only"
    return True, None


def _log(component: str, decision: str, **fields) -> None:
    try:
        from dabsn.runtime.dispatch import log_routing_once

        log_routing_once(component, decision, **fields)
    except Exception:  # noqa: BLE001 - observability must never break a step
        pass


def warn_fallback(component: str, reason: str, **fields) -> None:
    """A CUDA call this backend hands back to the reference's own code: made
    visible as the reference makes its own fast-path exits visible
    (``warn_routing_once`` emits ``PERFORMANCE_FALLBACK``, which
    ``strict_events`` turns into an error; runtime/dispatch.py:61-101)."""
    try:
        from dabsn.runtime.dispatch import warn_routing_once
    except Exception:  # noqa: BLE001 - the reference package is what we report into
        return
    warn_routing_once(component, reason, requested_path="b200", selected_path="reference",
                      **fields)


def _core_kernel(*inputs):
    wx = inputs[0]
    route = "b200_cluster_scan" if int(wx.shape[-1]) <= ops.NARROW_MAX_H else "b200_grid_scan"
    _log("core_scan", route, batch=int(wx.shape[0]), hidden=int(wx.shape[-1]),
         dtype=str(wx.dtype).replace("torch.", ""))
    return AG.core_forward_kernel(*inputs)


def enable_b200(*, required: bool = False) -> dict[str, bool]:
    """Install the B200 kernels into the reference package (idempotent)."""
    ok, why = native_available()
    if not ok:
        _STATE["error"] = why
        if required:
            raise RuntimeError(f"B200 (sm_100a) DABSN kernels were required but unavailable: {why}")
        return {"core_scan": False, "admitted_three_way_read": False, "long_memory": False}
    kernels, batched, long_mod, triton_mod, DABSNCore, DABSNRead = _reference()
    with _LOCK:
        op = batched._core_scan_batched_op
        op.register_kernel("cuda")(_core_kernel)
        torch.library.register_autograd(
            op,
            AG.make_core_backward(batched._core_scan_batched_backward),
            setup_context=batched._core_scan_batched_setup,
        )
        triton_mod.cuda_compact_three_way_read = AG.three_way_read
        import dabsn.runtime as runtime_mod
        import dabsn.runtime.loss as loss_mod

        ce = loss_mod.chunked_linear_cross_entropy
        fused_ce = AG.make_linear_cross_entropy(getattr(ce, "__wrapped_reference__", ce))
        loss_mod.chunked_linear_cross_entropy = fused_ce
        runtime_mod.chunked_linear_cross_entropy = fused_ce
        cel = loss_mod.chunked_cross_entropy_from_logits
        fused_cel = AG.make_ce_from_logits(getattr(cel, "__wrapped_reference__", cel))
        loss_mod.chunked_cross_entropy_from_logits = fused_cel
        runtime_mod.chunked_cross_entropy_from_logits = fused_cel
        import sys as _sys

        pretrain_mod = _sys.modules.get("dabsn.pretrain")
        if pretrain_mod is not None and hasattr(pretrain_mod, "chunked_cross_entropy_from_logits"):
            pretrain_mod.chunked_cross_entropy_from_logits = fused_cel
        import dabsn.kernels.local_field as lf_mod
        import dabsn.kernels.permanent as perm_mod

        perm_op = perm_mod._permanent_delta_scan_op
        perm_op.register_kernel("cuda")(AG.permanent_forward_kernel)
        torch.library.register_autograd(
            perm_op, AG.make_permanent_backward(perm_mod._permanent_delta_scan_registered_backward),
            setup_context=perm_mod._permanent_delta_scan_setup)
        lf_op = lf_mod._local_field_gather_op
        lf_op.register_kernel("cuda")(AG.local_field_kernel)
        torch.library.register_autograd(
            lf_op, AG.make_local_field_backward(lf_mod._local_field_gather_registered_backward),
            setup_context=lf_mod._local_field_gather_setup)
        if AG._REFERENCE_LONG is None:
            AG._REFERENCE_LONG = long_mod.fused_long_scan_from_state
        long_mod.fused_long_scan_from_state = AG.long_scan_from_state
        from dabsn.core import TensorParallelDABSNCore

        from . import tensor_parallel as TP

        current_tp = TensorParallelDABSNCore.forward_from_state
        TensorParallelDABSNCore.forward_from_state = TP.make_tp_forward(
            getattr(current_tp, "__wrapped_reference__", current_tp))
        if os.environ.get("DABSN_B200_PROJ", "1") != "0":
            current_core = DABSNCore.forward_from_state
            DABSNCore.forward_from_state = AG.make_core_forward(
                getattr(current_core, "__wrapped_reference__", current_core))
        if os.environ.get("DABSN_B200_FUSED_ADMISSION", "1") != "0":
            current = DABSNRead._unified_forward
            original = getattr(current, "__wrapped_reference__", current)
            DABSNRead._unified_forward = AG.make_unified_forward(original)
        for cls in (DABSNCore, DABSNRead):
            setattr(cls, "_cuda_native_enabled", True)
            setattr(cls, "_cuda_native_required", bool(required))
        setattr(DABSNRead, "_long_native_enabled", True)
        # The B200 hook itself refuses nothing on CUDA and hands CPU tensors to
        # the reference's implementation, so the reference's "CPU tensor while
        # CUDA was required" guard stays off (CPU models keep working).
        setattr(DABSNRead, "_long_native_required", False)
        _STATE.update(enabled=True, required=bool(required), error=None)
    return {"core_scan": True, "admitted_three_way_read": True, "long_memory": True}


def b200_status() -> dict[str, object]:
    ok, why = native_available()
    info: dict[str, object] = {
        "enabled": bool(_STATE["enabled"]),
        "required": bool(_STATE["required"]),
        "available": ok,
        "unavailable_reason": why,
        "library": str(_native.LIB_PATH),
        "library_loaded": _native.is_loaded(),
        "version": _native.version() if ok else None,
        "arch": "sm_100a",
        "kernels": {
            "core_scan": "persistent cluster scan, DSMEM exchange (fwd + reverse)",
            "admitted_three_way_read": "flash-tiled exact three-way read (fwd + reverse)",
            "long_memory": "fused three-recurrence long channel (fwd + chunk-recompute reverse)",
            "read_admission": "fused token statistics, membership, bank order and gathers",
            "tensor_parallel_core": "cross-GPU grid-wide scan, peer stores + bounded barrier (BF16)",
            "permanent_delta_scan": "one CTA per sequence, state in shared memory, checkpointed reverse",
            "local_field_gather": "gather + inverse-index reverse (no atomics)",
            "linear_cross_entropy": "tcgen05 readout GEMM with softmax epilogues (BF16)",
            "cross_entropy_from_logits": "one-pass log-sum-exp and softmax-gradient sweeps",
            "core_input_projections": "tcgen05 GEMM, W(x) and Wg(x) in one launch (BF16)",
            "recurrent_matrix_gradient": "tcgen05 GEMM, grad Ug and grad A in one launch (BF16)",
        },
        "ignored_reference_flags": {
            k: os.environ[k]
            for k in (
                "DABSN_CORE_BACKEND",
                "DABSN_FUSED_CORE_MAX_H",
                "DABSN_BATCHED_STEP_COMPILE",
                "DABSN_SCAN_GRAPH",
                "DABSN_TRAIN_READ_BACKEND",
                "DABSN_FLASH_PREC",
                "DABSN_LONG_SCAN_CHUNK",
            )
            if k in os.environ
        },
    }
    if ok:
        info["device"] = torch.cuda.get_device_name()
    return info


def enable(backend: str = "auto", *, required: bool = False) -> dict[str, object]:
    """Mirror of ``dabsn.kernels.enable`` with the ``"b200"`` family added.

    ``"auto"`` and ``"cuda"`` select the B200 family when a CUDA device is
    visible; ``"reference"`` and ``"cpu"`` go to the reference's own
    implementation.  Returns :func:`status`.
    """
    kernels = _reference()[0]
    normalized = backend.lower()
    if normalized == "auto":
        normalized = "b200" if torch.cuda.is_available() else "cpu"
    if normalized == "cuda":
        normalized = "b200"
    if normalized not in {"reference", "cpu", "b200"}:
        raise ValueError("backend must be one of: auto, reference, cpu, cuda, b200")
    active = getattr(kernels, "_ACTIVE_BACKEND", "reference")
    if normalized == "b200":
        if active not in {"reference", "b200"}:
            raise RuntimeError(
                f"DABSN backend already selected as {active}; "
                "select a different backend in a fresh process"
            )
        results = enable_b200(required=required)
        if required and not all(results.values()):
            raise RuntimeError(f"required B200 primitives unavailable: {results}")
        if all(results.values()):
            kernels._ACTIVE_BACKEND = "b200"
        return status()
    original = _ORIGINAL.get("enable", kernels.enable)
    original(normalized, required=required)
    return status()


_ORIGINAL: dict[str, object] = {}


def status() -> dict[str, object]:
    """``dabsn.kernels.status()`` plus a ``"b200"`` sub-report."""
    kernels = _reference()[0]
    original = _ORIGINAL.get("status", kernels.status)
    report = dict(original())
    report["b200"] = b200_status()
    return report


def install() -> None:
    """Hook ``dabsn.kernels.enable`` / ``status`` so existing callers reach the
    B200 family through the reference's own entry points (``enable("cuda")``
    selects it).  Idempotent."""
    kernels = _reference()[0]
    with _LOCK:
        if "enable" not in _ORIGINAL:
            _ORIGINAL["enable"] = kernels.enable
            _ORIGINAL["status"] = kernels.status
        kernels.enable = enable
        kernels.status = status
