"""State drift over long sequences: the B200 path (FP32) against the
reference's own implementation in FP32 and FP64, forward only, at config 2's
length-extrapolation run (T = 3200) and config 3 at T = 1024, 4096, 16384
(batch 2, random-init weights, seeded uniform tokens).  The logits must stay
within the forward bar (max |a - e| / max |e| <= 1e-4) at every length; the
measured drift against FP64 is ~5e-6 at T = 16384.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import max_rel_err, reference_available

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
CASES = ("c2:3200", "c3:1024", "c3:4096", "c3:16384")


def test_long_sequence_state_drift(tmp_path, capsys):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    here = Path(__file__).resolve().parent
    out = tmp_path / "reference_logits.pt"
    res = subprocess.run([sys.executable, str(here / "_reference_logits.py"), str(out),
                          ",".join(CASES)], capture_output=True, text=True, timeout=1500)
    assert res.returncode == 0, res.stderr[-2000:]
    refs = torch.load(out)

    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels

    dabsn.kernels.enable("cuda", required=True)
    sys.path.insert(0, str(here))
    from _reference_logits import model, tokens

    lines = []
    for case in CASES:
        cfg, T = case.split(":")
        m, V = model(cfg)
        m = m.cuda().eval()
        with torch.no_grad():
            logits = m.forward_sequence(tokens(V, int(T)).cuda())
        e32 = max_rel_err(logits, refs[(case, str(torch.float32))])
        e64 = max_rel_err(logits, refs[(case, str(torch.float64))])
        r64 = max_rel_err(refs[(case, str(torch.float32))], refs[(case, str(torch.float64))])
        lines.append(f"{case}: vs reference FP32 {e32:.2e}, vs FP64 {e64:.2e} "
                     f"(reference FP32 vs FP64 {r64:.2e}), bank width {m.backbone.blocks[0].read.last_n_max}")
        assert e32 <= FWD_TOL and e64 <= FWD_TOL, lines[-1]
    with capsys.disabled():
        print("\n" + "\n".join(lines))
