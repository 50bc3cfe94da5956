"""Cross-entropy over materialised logits: the one-pass kernels behind
``dabsn.runtime.loss.chunked_cross_entropy_from_logits`` (the default loss of
the reference's ``train_step``) against the reference's own function on the
same GPU tensors.

Bars: loss relative error <= 1e-5 (FP32 sums of log-sum-exps; the kernels
use the hardware exponential, ~2 ulp); gradients max |a - e| / max |e| <=
1e-5 for FP32 logits and <= 1e-2 for BF16 logits (both write the FP32 value
rounded once to BF16; a last-bit difference of the exponential can move a
value across a BF16 rounding boundary: one BF16 ulp is 2^-8 relative).
Both of the reference's branches are covered: single shot (rows * V within
the element budget, NaN when every target is ignored) and chunked (0 then).
"""

from __future__ import annotations

import pytest
import torch

from conftest import max_rel_err, reference_available

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-5
GRAD_TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2}


@pytest.fixture(scope="module")
def fns():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels
    import dabsn.runtime.loss as loss_mod

    dabsn.kernels.enable("cuda", required=True)
    fused = loss_mod.chunked_cross_entropy_from_logits
    return fused, fused.__wrapped_reference__


def _case(shape, V, dtype, ignore_frac, seed):
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(*shape, V, generator=g) * 3.0).to(dtype).cuda()
    tgt = torch.randint(0, V, shape, generator=g)
    tgt[torch.rand(shape, generator=g) < ignore_frac] = -100
    return logits, tgt.cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,V,budget", [((4, 64), 1000, None), ((4, 64), 1000, 1 << 12),
                                            ((3, 17), 1001, None), ((2, 33), 32000, None),
                                            ((256,), 64, 1 << 10)])
def test_ce_from_logits_matches_reference(fns, dtype, shape, V, budget):
    fused, ref = fns
    logits, tgt = _case(shape, V, dtype, 0.1, 7 + V)
    a = logits.clone().requires_grad_(True)
    e = logits.clone().requires_grad_(True)
    la = fused(a, tgt, chunk_budget=budget)
    le = ref(e, tgt, chunk_budget=budget)
    assert abs(float(la) - float(le)) <= LOSS_TOL * abs(float(le)), (float(la), float(le))
    la.backward()
    le.backward()
    assert a.grad.dtype == dtype and a.grad.shape == logits.shape
    assert max_rel_err(a.grad, e.grad) <= GRAD_TOL[dtype], max_rel_err(a.grad, e.grad)


@pytest.mark.parametrize("budget,expect_nan", [(None, True), (1 << 8, False)])
def test_ce_from_logits_all_ignored(fns, budget, expect_nan):
    fused, ref = fns
    logits, tgt = _case((2, 40), 512, torch.bfloat16, 1.0, 3)
    a = logits.clone().requires_grad_(True)
    la = fused(a, tgt, chunk_budget=budget)
    le = ref(logits.clone(), tgt, chunk_budget=budget)
    assert bool(torch.isnan(la)) == expect_nan == bool(torch.isnan(le))
    if not expect_nan:
        assert float(la) == float(le) == 0.0
    la.backward()
    assert float(a.grad.abs().max()) == 0.0


def test_ce_from_logits_rejects_bad_target(fns):
    from dabsn_b200 import _native

    fused, _ = fns
    logits, tgt = _case((2, 8), 100, torch.float32, 0.0, 5)
    tgt[0, 3] = 100  # outside [0, V)
    _native.device_status(reset=True)
    loss = fused(logits, tgt)
    torch.cuda.synchronize()
    assert torch.isnan(loss)
    with pytest.raises(RuntimeError, match="outside"):
        _native.raise_on_device_status()
    assert _native.device_status() == 0
