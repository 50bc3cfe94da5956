"""tcgen05 / TMA GEMM of the wide read against the mma.sync GEMM.

The score product and the value-gradient products of the tensor-core read run
on the 5th-generation tensor cores (TMEM accumulator, TMA-staged operands) by
default; DABSN_B200_TCGEN05=0 selects the mma.sync kernel.  Both accumulate in
FP32 and round to BF16, in different orders, so read outputs and gradients
agree within a few BF16 ulps (max |a - e| / max |e| <= 1e-2).  Shapes cover
ragged tiles (T, N not multiples of 128) and a contraction with a tail
(H = 520: 8 elements past the last 64-wide slice), at both output tile widths
(256, the default, and 128 through DABSN_B200_READ_BN).
"""

from __future__ import annotations

import pytest
import torch

from conftest import max_rel_err
from test_gpu_wide_read import _device_read, _inputs

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.mark.parametrize("B,T,H,drop,mode", [
    (2, 300, 520, 0.3, "seq"), (1, 200, 1024, 0.0, "field"), (3, 129, 512, 0.5, "seq"),
])
@pytest.mark.parametrize("bn", ["256", "128"])
def test_tcgen05_read_matches_mma_sync(B, T, H, drop, mode, bn, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    monkeypatch.setenv("DABSN_B200_READ_BN", bn)
    diff, idx, valid = _inputs(B, T, H, drop, 17 + T + H)
    wout = torch.randn(B, T, H, generator=torch.Generator().manual_seed(4), dtype=torch.float64)
    monkeypatch.setenv("DABSN_B200_TCGEN05", "1")
    out_t, grads_t = _device_read(diff, idx, valid, mode, wout)
    monkeypatch.setenv("DABSN_B200_TCGEN05", "0")
    out_m, grads_m = _device_read(diff, idx, valid, mode, wout)
    assert max_rel_err(out_t, out_m) <= TOL, max_rel_err(out_t, out_m)
    for i, (a, e) in enumerate(zip(grads_t, grads_m)):
        assert max_rel_err(a, e) <= TOL or float(e.abs().max()) < 1e-6, (i, max_rel_err(a, e))
