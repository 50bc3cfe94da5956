"""Readout + cross-entropy on the tcgen05 GEMM against the reference's own
``chunked_linear_cross_entropy`` (runtime/loss.py:138-184) under BF16
autocast, on ragged shapes (rows and vocabulary not multiples of 128), with a
bias and ignored targets, at both output tile widths of the GEMM (256, the
default, and 128 through DABSN_B200_CE_BN).  The loss must agree within 2e-3 relative; the
gradients, whose logits' softmax gradient is rounded to BF16 once here where
the reference keeps FP32, within 2e-2 normwise.
"""

from __future__ import annotations

import pytest
import torch

from conftest import reference_available

pytestmark = pytest.mark.gpu


def _norm_rel(a, e):
    a, e = a.detach().double().cpu(), e.detach().double().cpu()
    return float((a - e).norm()) / max(float(e.norm()), 1e-12)


@pytest.mark.parametrize("bn", ["256", "128"])
@pytest.mark.parametrize("rows,V,D", [(600, 1000, 256), (4096, 32000, 512), (129, 64, 64)])
def test_linear_ce_matches_reference(rows, V, D, bn, monkeypatch):
    monkeypatch.setenv("DABSN_B200_CE_BN", bn)
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels
    import dabsn.runtime as runtime

    dabsn.kernels.enable("cuda", required=True)
    fused = runtime.chunked_linear_cross_entropy
    reference = fused.__wrapped_reference__
    g = torch.Generator().manual_seed(rows + V)
    hidden = torch.randn(rows, D, generator=g).cuda()
    weight = (torch.randn(V, D, generator=g) / D**0.5).cuda()
    bias = (0.1 * torch.randn(V, generator=g)).cuda()
    targets = torch.randint(0, V, (rows,), generator=g).cuda()
    targets[::7] = -100
    results = []
    for fn in (fused, reference):
        h, w, b = (t.clone().requires_grad_() for t in (hidden, weight, bias))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = fn(h, w, b, targets)
        loss.backward()
        results.append((loss.detach().float(), h.grad, w.grad, b.grad))
    (lf, *gf), (lr, *gr) = results
    assert abs(float(lf) - float(lr)) <= 2e-3 * abs(float(lr)), (float(lf), float(lr))
    for name, a, e in zip(("hidden", "weight", "bias"), gf, gr):
        assert _norm_rel(a, e) <= 2e-2, (name, _norm_rel(a, e))


@pytest.mark.parametrize("budget", [None, 64])
def test_linear_ce_all_targets_ignored(budget):
    """Every target ignored: the reference's single-shot branch (the default
    at these sizes) returns NaN, its chunked branch (a 64-logit budget) 0;
    both with zero gradients.  The fused loss follows the same branch."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels
    import dabsn.runtime as runtime

    dabsn.kernels.enable("cuda", required=True)
    fused = runtime.chunked_linear_cross_entropy
    reference = fused.__wrapped_reference__
    g = torch.Generator().manual_seed(5)
    hidden = torch.randn(33, 64, generator=g).cuda()
    weight = (torch.randn(40, 64, generator=g) / 8).cuda()
    bias = (0.1 * torch.randn(40, generator=g)).cuda()
    targets = torch.full((33,), -100, dtype=torch.int64).cuda()
    losses = []
    for fn in (fused, reference):
        h, w, b = (t.clone().requires_grad_() for t in (hidden, weight, bias))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = fn(h, w, b, targets, chunk_budget=budget)
        loss.backward()
        losses.append(float(loss))
        for grad in (h.grad, w.grad, b.grad):
            assert grad is None or float(grad.abs().max()) == 0.0
    lf, lr = losses
    if budget is None:
        assert lf != lf and lr != lr, (lf, lr)  # NaN
    else:
        assert lf == 0.0 and lr == 0.0, (lf, lr)


def test_linear_ce_chunked_reverse_matches_single_shot_and_reference():
    """A chunk budget bounds the reverse's dlogits workspace: 1000 rows run in
    three chunks (400, 400, 200) with dweight accumulated in FP32, and match
    the same loss run in one chunk and the reference's chunked loss."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200
    from dabsn_b200 import _native
    from dabsn_b200.autograd import _linear_ce_row_chunk

    dabsn_b200.install()
    import dabsn.kernels
    import dabsn.runtime as runtime

    dabsn.kernels.enable("cuda", required=True)
    rows, V, D = 1000, 3000, 256
    ld = int(_native.load().dabsn_linear_ce_ld(V))
    budget = 200 * ld
    assert _linear_ce_row_chunk(rows, V, budget) == 400
    assert _linear_ce_row_chunk(rows, V, None) == rows
    fused = runtime.chunked_linear_cross_entropy
    reference = fused.__wrapped_reference__
    g = torch.Generator().manual_seed(11)
    hidden = torch.randn(rows, D, generator=g).cuda()
    weight = (torch.randn(V, D, generator=g) / D**0.5).cuda()
    bias = (0.1 * torch.randn(V, generator=g)).cuda()
    targets = torch.randint(0, V, (rows,), generator=g).cuda()
    targets[::5] = -100
    results = []
    for fn, kw in ((fused, {"chunk_budget": budget}), (fused, {}),
                   (reference, {"chunk_budget": budget})):
        h, w, b = (t.clone().requires_grad_() for t in (hidden, weight, bias))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = fn(h, w, b, targets, **kw)
        loss.backward()
        results.append((loss.detach().float(), h.grad, w.grad, b.grad))
    (lc, *gc), (ls, *gs), (lr, *gr) = results
    assert abs(float(lc) - float(ls)) <= 1e-6 * abs(float(ls))
    for name, a, e in zip(("hidden", "weight", "bias"), gc, gs):
        # the chunks and the single shot differ only in where FP32 sums split
        assert _norm_rel(a, e) <= 1e-3, (name, _norm_rel(a, e))
    assert abs(float(lc) - float(lr)) <= 2e-3 * abs(float(lr))
    for name, a, e in zip(("hidden", "weight", "bias"), gc, gr):
        assert _norm_rel(a, e) <= 2e-2, (name, _norm_rel(a, e))


def test_linear_ce_rejects_bad_target():
    """A target outside [0, V) that is not ignore_index: NaN loss and device
    status 7, raised at the next synchronisation (the reference's gather
    raises on such a target)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200
    from dabsn_b200 import _native

    dabsn_b200.install()
    import dabsn.kernels
    import dabsn.runtime as runtime

    dabsn.kernels.enable("cuda", required=True)
    g = torch.Generator().manual_seed(7)
    hidden = torch.randn(64, 64, generator=g).cuda()
    weight = (torch.randn(100, 64, generator=g) / 8).cuda()
    targets = torch.randint(0, 100, (64,), generator=g).cuda()
    targets[5] = 100
    _native.device_status(reset=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = runtime.chunked_linear_cross_entropy(hidden, weight, None, targets)
    torch.cuda.synchronize()
    assert torch.isnan(loss)
    with pytest.raises(RuntimeError, match="outside"):
        _native.raise_on_device_status()
    assert _native.device_status() == 0
