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


@pytest.mark.parametrize("env", [None, "off", "5000000", "abc"])
@pytest.mark.parametrize("budget", [None, 0, 64, 10_000_000])
def test_reverse_row_chunk(env, budget, monkeypatch):
    """Rows per reverse chunk of the fused loss: with a budget (argument
    first, then DABSN_LOSS_CHUNK_SCORES) the BF16 dlogits chunk holds at most
    2 x budget elements but at least one 128-row tile; without one (or
    "off", or an unparsable value) at most 1 GiB; never more than the rows."""
    from dabsn_b200 import _native
    from dabsn_b200.autograd import _linear_ce_row_chunk

    if env is None:
        monkeypatch.delenv("DABSN_LOSS_CHUNK_SCORES", raising=False)
    else:
        monkeypatch.setenv("DABSN_LOSS_CHUNK_SCORES", env)
    rows, V = 131072, 32000
    ld = int(_native.load().dabsn_linear_ce_ld(V))
    eff = budget if budget is not None else (int(env) if env and env.isdigit() else None)
    if eff is not None and eff > 0:
        want = max(128, (2 * eff) // ld)
    else:
        want = (1 << 30) // (2 * ld)
    assert _linear_ce_row_chunk(rows, V, budget) == min(rows, want)
    assert _linear_ce_row_chunk(100, V, budget) == min(100, want)
