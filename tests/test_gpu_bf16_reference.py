"""BF16 autocast drop-in parity against the reference's own CUDA path.

Configs 4 and 5 train under BF16 autocast at widths 1024 and 2048.  Here one
forward + backward of a one-block ``DABSNSequenceLM`` at those widths (T = 512,
Zipf(1.1) tokens over a 32000-token vocabulary) runs on this library's
backend and, in a child process on the same GPU, on the reference's own CUDA
family (``enable("cuda")``) under the same autocast; the reference also runs
in FP32 there, which measures how far BF16 itself moves each quantity.

Bars (the reference's BF16 policy: rtol 2e-2 for forward drift and 5 % for
gradients, kernels/batched_runtime.py:88-90, 168-186):

* logits: max |a - e| / max |e| <= 3e-2 against the reference's BF16 logits;
  loss: relative difference <= 1e-2;
* every parameter gradient whose norm in the reference's FP32 run is at
  least 1e-4 of the largest parameter gradient's: ||a - e|| / ||e|| <=
  max(5e-2, 1.5 x the reference's own BF16-vs-FP32 distance for that tensor)
  against the reference's BF16 gradient, and this backend no further from the
  reference's FP32 gradient than 1.5 x the reference's BF16 one, plus 1e-2;
* smaller gradients (rounding noise: e.g. the read's null_bias, whose exact
  gradient is zero because softmax ignores a shift, measures 2e-16 in FP32
  and differs by 27x between the reference's own BF16 and FP32 runs):
  ||a - e|| <= 5e-2 x 1e-4 x the largest gradient norm.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import max_rel_err, reference_available

pytestmark = pytest.mark.gpu

CASES = ["1024:512:2", "2048:512:2"]
LOGIT_TOL = 3e-2
LOSS_TOL = 1e-2
GRAD_NORM_TOL = 5e-2
SIGNIFICANT = 1e-4  # gradients below this fraction of the largest are noise-level


def _norm_rel(a, e):
    a = a.detach().double().cpu()
    e = e.detach().double().cpu()
    den = float(e.norm())
    return float((a - e).norm()) / den if den > 0 else float(a.norm())


@pytest.fixture(scope="module")
def reference_runs(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    out = tmp_path_factory.mktemp("bf16ref") / "ref.pt"
    here = Path(__file__).resolve().parent
    res = subprocess.run([sys.executable, str(here / "_reference_bf16_run.py"), str(out),
                          ",".join(CASES)], capture_output=True, text=True, timeout=1800)
    assert res.returncode == 0, res.stderr[-3000:]
    return torch.load(out, weights_only=False)


@pytest.fixture(scope="module")
def b200():
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels

    st = dabsn.kernels.enable("cuda", required=True)
    assert st["active_backend"] == "b200"
    return dabsn_b200


@pytest.mark.parametrize("case", CASES)
def test_bf16_autocast_matches_reference_cuda(reference_runs, b200, case):
    from _reference_bf16_run import batch, model, run

    H, T, B = (int(v) for v in case.split(":"))
    ids, tgt = (t.cuda() for t in batch(T, B))
    m = model(H).cuda()
    mine = run(m, ids, tgt, True)
    blk = m.backbone.blocks[0]
    assert blk.read._last_three_way_backend == "b200_tensor_core"
    ref, ref32 = reference_runs[(case, "bf16")], reference_runs[(case, "fp32")]

    err = max_rel_err(mine["logits"], ref["logits"])
    assert err <= LOGIT_TOL, f"logits vs reference BF16: {err}"
    ref_spread = max_rel_err(ref["logits"], ref32["logits"])
    mine_32 = max_rel_err(mine["logits"], ref32["logits"])
    assert mine_32 <= 1.5 * ref_spread + 1e-2, (mine_32, ref_spread)
    assert abs(mine["loss"] - ref["loss"]) <= LOSS_TOL * abs(ref["loss"]), (mine["loss"],
                                                                          ref["loss"])
    assert set(mine["grads"]) == set(ref["grads"])
    scale = max(float(g.norm()) for g in ref32["grads"].values())
    floor = SIGNIFICANT * scale
    worst = []
    for name, g in mine["grads"].items():
        e, e32 = ref["grads"][name], ref32["grads"][name]
        if float(e32.norm()) < floor:
            diff = float((g.double() - e.double()).norm())
            assert diff <= GRAD_NORM_TOL * floor, f"{name}: |a - e| {diff} (noise-level gradient)"
            continue
        spread = _norm_rel(e, e32)
        tol = max(GRAD_NORM_TOL, 1.5 * spread)
        d = _norm_rel(g, e)
        worst.append((d / tol, name, d, spread))
        assert d <= tol, f"{name}: {d} vs reference BF16 (bar {tol}, BF16 spread {spread})"
        d32 = _norm_rel(g, e32)
        assert d32 <= 1.5 * spread + 1e-2, f"{name}: {d32} vs reference FP32 (spread {spread})"
    worst.sort(reverse=True)
    print(f"H={H}: logits {err:.3g} (BF16 spread {ref_spread:.3g}); worst grads {worst[:3]}")
