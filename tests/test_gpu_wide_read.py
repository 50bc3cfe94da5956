"""Tensor-core three-way read (states wider than 256 units, BF16).

* Against the float64 oracle on BF16-rounded inputs: forward max |a - e| /
  max |e| <= 3e-2, gradients ||a - e|| / ||e|| <= 5e-2.  The read rounds the
  score products, the softmax weights and the value products to BF16 as the
  reference's BF16 path does (compact_admitted.py:40-80), so it differs from
  exact arithmetic by a few BF16 ulps.  The scale and the four gains are
  scalars whose gradients sum B*T*N cancelling terms: rounding only the
  upstream gradient to BF16 moves the oracle's own values by up to 6%.  Their
  bar is twice that measured spread, at least 1e-1.
* Against the SIMT read at H = 256, where both exist, under the same BF16
  inputs: the same bars.
"""

from __future__ import annotations

import pytest
import torch

import dabsn_oracle as O
from conftest import max_rel_err
from test_gpu_parity import _bank

pytestmark = pytest.mark.gpu

FWD_TOL = 3e-2
GRAD_NORM_TOL = 5e-2
SCALAR_GRAD_TOL = 1e-1
NAMES = ["q", "k", "w", "nw", "cq", "ck", "kb", "adm", "scale", "sg", "pg", "ig", "cg"]


def _norm_rel(a, e):
    a = a.detach().double().cpu()
    e = e.detach().double().cpu()
    den = float(e.norm())
    return float((a - e).norm()) / den if den > 0 else float(a.norm())


def _inputs(B, T, H, drop, seed):
    diff, idx, valid = _bank(B, T, H, seed, drop)
    # the BF16 read sees BF16 activations: round them once for every party
    for i in range(6):
        diff[i] = diff[i].to(torch.bfloat16).double()
    return diff, idx, valid


def _device_read(diff, idx, valid, mode, wout):
    from dabsn_b200 import _native
    from dabsn_b200 import autograd as AG

    dev = torch.device("cuda")
    cl = [x.to(dev, torch.float32).requires_grad_() for x in diff]
    T = cl[0].shape[1]
    out = AG.ThreeWayRead.apply(*cl, idx.to(dev), valid.to(dev), 0 if mode == "seq" else 1, T,
                                torch.bfloat16)
    grads = torch.autograd.grad((out * wout.to(dev, out.dtype)).sum(), cl)
    torch.cuda.synchronize()
    assert _native.device_status() == 0
    return out, grads


@pytest.mark.parametrize("B,T,H,drop,mode", [
    (2, 70, 512, 0.3, "seq"), (2, 130, 1024, 0.0, "seq"), (1, 300, 512, 0.5, "field"),
    (3, 40, 2048, 0.2, "seq"), (2, 257, 768, 0.6, "seq"),
])
def test_wide_read_matches_oracle(B, T, H, drop, mode):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    diff, idx, valid = _inputs(B, T, H, drop, T * 7 + H)
    leaves = [x.clone().requires_grad_() for x in diff]
    q, k, w, nw, cq, ck, kb, adm, scale, sg, pg, ig, cg = leaves
    ref = O.three_way_read(q, k, w, nw, cq, ck, kb, adm, scale, idx, valid, mode=mode,
                           short_gain=sg, pad_gain=pg, induct_gain=ig, cocktail_gain=cg)
    g = torch.Generator().manual_seed(3)
    wout = torch.randn(ref.shape, generator=g, dtype=torch.float64)
    ref_grads = torch.autograd.grad((ref * wout).sum(), leaves, retain_graph=True)
    wout_bf = wout.to(torch.bfloat16).double()
    spread = torch.autograd.grad((ref * wout_bf).sum(), leaves)
    out, grads = _device_read(diff, idx, valid, mode, wout)
    assert max_rel_err(out, ref) <= FWD_TOL, max_rel_err(out, ref)
    for n, a, e, e2 in zip(NAMES, grads, ref_grads, spread):
        tol = GRAD_NORM_TOL
        if e.numel() == 1:
            tol = max(SCALAR_GRAD_TOL, 2.0 * _norm_rel(e2, e))
        assert _norm_rel(a, e) <= tol, f"{n}: {_norm_rel(a, e)}"


@pytest.mark.parametrize("mode", ["seq", "field"])
def test_wide_read_matches_simt_read(mode, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dabsn_b200 import ops

    diff, idx, valid = _inputs(2, 150, 256, 0.3, 11)
    wout = torch.randn(2, 150, 256, generator=torch.Generator().manual_seed(5),
                       dtype=torch.float64)
    out_n, grads_n = _device_read(diff, idx, valid, mode, wout)
    monkeypatch.setattr(ops, "NARROW_READ_MAX_H", 0)
    out_w, grads_w = _device_read(diff, idx, valid, mode, wout)
    assert max_rel_err(out_w, out_n) <= FWD_TOL, max_rel_err(out_w, out_n)
    for n, a, e in zip(NAMES, grads_w, grads_n):
        assert _norm_rel(a, e) <= GRAD_NORM_TOL, f"{n}: {_norm_rel(a, e)}"


def test_wide_read_empty_rows_and_padding():
    """Rows with no admitted entry read zero; padded bank entries get zero
    gradients."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    diff, idx, valid = _inputs(2, 33, 512, 0.0, 5)
    # sequence 1 admits only positions >= 20: its rows 0..19 see nothing
    valid[1] = False
    valid[1, 20:] = True
    idx[1, 20:] = torch.arange(20, 33)
    wout = torch.randn(2, 33, 512, generator=torch.Generator().manual_seed(2),
                       dtype=torch.float64)
    out, grads = _device_read(diff, idx, valid, "seq", wout)
    assert float(out[1, :20].abs().max()) == 0.0
    for g in grads[1:4]:
        assert float(g[1, :20].abs().max()) == 0.0
