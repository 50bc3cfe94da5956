"""The two primitives of the dabsn.kernels surface on the B200 family.

``dabsn::permanent_delta_scan`` and ``dabsn::local_field_gather`` run their
CUDA kernels (registered on the reference's ops) against the reference's
own results (golden fixtures) and the float64 oracle: forward <= 1e-4 and
gradients <= 1e-3 relative in FP32 (the gather and its reverse are exact).
The delta scan's reverse rebuilds states from checkpoints every 64 steps;
T = 700 crosses several of them.
"""

from __future__ import annotations

import pytest
import torch

import dabsn_oracle as O
from conftest import load_golden, max_rel_err, reference_available

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def b200():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels

    dabsn.kernels.enable("cuda", required=True)
    return dabsn_b200


def _delta(k, v, beta, w):
    from dabsn.kernels.permanent import permanent_delta_scan

    leaves = [t.cuda().float().requires_grad_() for t in (k, v, beta)]
    out = permanent_delta_scan(*leaves)
    grads = torch.autograd.grad((out * w.cuda().float()).sum(), leaves)
    return out, grads


@pytest.mark.parametrize("name", ["permanent_f64", "permanent_f32"])
def test_permanent_delta_matches_reference_fixture(b200, name):
    fx = load_golden(name)
    out, grads = _delta(*fx["inputs"], fx["out_weight"])
    assert max_rel_err(out, fx["output"]) <= FWD_TOL
    for a, e in zip(grads, fx["grads"]):
        assert max_rel_err(a, e) <= GRAD_TOL, max_rel_err(a, e)


@pytest.mark.parametrize("B,T,h", [(2, 700, 64), (1, 33, 128), (3, 5, 7)])
def test_permanent_delta_matches_oracle(b200, B, T, h):
    g = torch.Generator().manual_seed(T + h)
    k = torch.nn.functional.normalize(torch.randn(B, T, h, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(B, T, h, generator=g, dtype=torch.float64)
    beta = torch.rand(B, T, generator=g, dtype=torch.float64) * 0.5
    w = torch.randn(B, T, h, generator=g, dtype=torch.float64)
    leaves = [t.clone().requires_grad_() for t in (k, v, beta)]
    ref = O.permanent_delta_scan(*leaves)
    ref_grads = torch.autograd.grad((ref * w).sum(), leaves)
    out, grads = _delta(k, v, beta, w)
    assert max_rel_err(out, ref) <= FWD_TOL
    for a, e in zip(grads, ref_grads):
        assert max_rel_err(a, e) <= GRAD_TOL, max_rel_err(a, e)


def test_local_field_gather_matches_reference_fixture(b200):
    from dabsn.kernels.local_field import _local_field_gather_op

    fx = load_golden("local_field_f64")
    x = fx["inputs"][0].cuda().float().requires_grad_()
    out = _local_field_gather_op(x, fx["patch"].cuda())
    assert torch.equal(out.cpu(), fx["output"].float())  # a gather is exact
    (gx,) = torch.autograd.grad((out * fx["out_weight"].cuda().float()).sum(), [x])
    assert max_rel_err(gx, fx["grads"][0]) <= 1e-6
    # larger case against the oracle, repeated cells and unread cells included
    g = torch.Generator().manual_seed(3)
    xb = torch.randn(3, 200, 48, generator=g)
    patch = torch.randint(0, 150, (120, 9), generator=g)
    xg = xb.cuda().requires_grad_()
    out = _local_field_gather_op(xg, patch.cuda())
    w = torch.randn(out.shape, generator=g)
    (gx,) = torch.autograd.grad((out * w.cuda()).sum(), [xg])
    xr = xb.double().requires_grad_()
    ref = O.local_field_gather(xr, patch)
    (gr,) = torch.autograd.grad((ref * w.double()).sum(), [xr])
    assert torch.equal(out.cpu(), ref.float())
    assert max_rel_err(gx, gr) <= 1e-6
