"""Host logic of the fused readout + cross-entropy drop-in: the fused loss
follows the branch the reference's ``chunked_linear_cross_entropy`` would take
(runtime/loss.py:138-184) -- single shot through ``F.cross_entropy``, which
gives NaN when every target is ignored, or chunked, which gives 0 -- so its
predicate must agree with the reference's own choice for every budget and
``DABSN_LOSS_CHUNK_SCORES`` setting.  Runs on the CPU: the reference's
chunked branch is intercepted, nothing is launched."""

from __future__ import annotations

import pytest
import torch

from conftest import reference_available


@pytest.mark.parametrize("env", [None, "off", "OFF", "19", "20", "abc", "0"])
@pytest.mark.parametrize("budget", [None, 0, 19, 20, 21, 1 << 30])
def test_single_shot_predicate_matches_reference(env, budget, monkeypatch):
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    import dabsn.runtime.loss as loss_mod

    from dabsn_b200.autograd import _reference_single_shot

    if env is None:
        monkeypatch.delenv("DABSN_LOSS_CHUNK_SCORES", raising=False)
    else:
        monkeypatch.setenv("DABSN_LOSS_CHUNK_SCORES", env)
    taken = []

    def chunked(*args):
        taken.append("chunked")
        return torch.zeros(())

    monkeypatch.setattr(loss_mod.ChunkedLinearCrossEntropy, "apply", staticmethod(chunked))
    original = loss_mod.chunked_linear_cross_entropy
    rows, vocab = 4, 5  # 20 logits
    h = torch.randn(rows, 3)
    w = torch.randn(vocab, 3)
    t = torch.randint(0, vocab, (rows,))
    original(h, w, None, t, chunk_budget=budget)
    reference_single = not taken
    assert _reference_single_shot(original, rows, vocab, budget) == reference_single
