"""The forward wide scan that allocates nothing, against the one that takes
caller scratch.

``dabsn_core_scan_wide_fwd_noalloc`` serves callers that cannot allocate
device memory while they run the scan (allocator or memory-pool callbacks,
host frameworks that own every allocation).  It keeps its scratch in a static
device array shared by all calls, so two calls in a row on different inputs
must each give what ``dabsn_core_scan_wide_fwd`` gives with fresh scratch:
nothing left in the array by the first call may leak into the second.  Both
run the same kernel, but its partial sums are combined with shared-memory
atomics whose order varies between runs, so a BF16 output can move by an ulp;
the bar is the one of the other wide-scan tests (max |a - e| / max |e| <=
1e-2, about two BF16 ulps).

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import max_rel_err
from test_gpu_parity import _core_inputs

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-2


def _args(B, T, H, seed):
    from dabsn_b200 import ops

    dev = torch.device("cuda")
    inputs = [x.to(dev, torch.float32) for x in _core_inputs(B, T, H, seed)]
    Wx, Wgx = (x.to(torch.bfloat16).contiguous() for x in inputs[:2])
    rec = torch.cat((inputs[2], inputs[3]), dim=0).to(torch.bfloat16).contiguous()
    pack = ops._ParamPack(list(inputs[4:20]), list(inputs[20:23]), H)
    inits = [x.contiguous() for x in inputs[23:26]]
    return Wx, Wgx, rec, pack, inits


def _outputs(B, T, H):
    dev = torch.device("cuda")
    U = torch.full((B, T, 2 * H), float("nan"), device=dev, dtype=torch.bfloat16)
    tapes = [torch.full((B, T, H), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(7)]
    fins = [torch.full((B, H), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(3)]
    return [U, *tapes, *fins]


def _call(lib, name, B, T, H, args, outs, scratch=None):
    from dabsn_b200 import _native, ops

    Wx, Wgx, rec, pack, inits = args
    ptrs = [ops._ptr(Wx), ops._ptr(Wgx), ops._ptr(rec), ctypes.byref(pack.struct),
            *[ops._ptr(t) for t in inits], *[ops._ptr(o) for o in outs]]
    stream = ops._stream(torch.device("cuda"))
    if scratch is None:
        st = getattr(lib, name)(B, T, H, *ptrs, stream)
    else:
        st = getattr(lib, name)(B, T, H, *ptrs, ops._ptr(scratch), scratch.numel(), stream)
    _native.check(st, name)


def test_noalloc_forward_matches_scratch_forward_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dabsn_b200 import _native

    lib = _native.load()
    for B, T, H, seed in ((20, 9, 512, 11), (32, 6, 2048, 12)):
        args = _args(B, T, H, seed)
        scratch = torch.empty(int(lib.dabsn_core_scan_wide_scratch_bytes(H)), dtype=torch.uint8,
                              device="cuda")
        expected = _outputs(B, T, H)
        _call(lib, "dabsn_core_scan_wide_fwd", B, T, H, args, expected, scratch)
        got = _outputs(B, T, H)
        _call(lib, "dabsn_core_scan_wide_fwd_noalloc", B, T, H, args, got)
        torch.cuda.synchronize()
        assert _native.device_status() == 0
        for i, (a, e) in enumerate(zip(got, expected)):
            assert torch.isfinite(a.float()).all(), f"H={H} output {i} not written"
            assert max_rel_err(a, e) <= FWD_TOL, f"H={H} output {i}: {max_rel_err(a, e)}"


def test_noalloc_forward_rejects_oversize():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dabsn_b200 import _native

    lib = _native.load()
    B, T, H = 2, 3, 4096
    null = ctypes.c_void_p(0)
    st = lib.dabsn_core_scan_wide_fwd_noalloc(B, T, H, *([null] * 3), None, *([null] * 14), null)
    assert st != 0
    assert "static scratch" in lib.dabsn_last_error().decode()
