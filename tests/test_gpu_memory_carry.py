"""Carried memory and the query-bank read on the B200 family.

The same exactness gates the reference holds for ``dabsn.memory`` (chunked
ingest, split ingest + query, incremental decode, a selective bank), run with
the B200 kernels: the query-bank read hands the read bank positions relative
to the query window (negative for entries before it) and the long channel an
initial state.  Logits must match the dense pass within the north-star
forward bar (rel 1e-4, atol 1e-5 as the reference's CPU gate).  A gradient
check through ``forward_query_bank`` with a query window starting at 40 (bank
positions down to -40) compares with the reference's CPU path at the gradient
bar.
"""

from __future__ import annotations

import copy

import pytest
import torch

from conftest import max_rel_err, reference_available

pytestmark = pytest.mark.gpu

VOCAB, BATCH, TOKENS = 61, 2, 48
ATOL, RTOL = 1e-5, 1e-4
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


def _model(seed=0):
    from dabsn.model import DABSNLayerSpec, DABSNSequenceLM

    torch.manual_seed(seed)
    return DABSNSequenceLM(
        vocab=VOCAB, hidden_dim=16, depth=2,
        layers=[DABSNLayerSpec(hidden_dim=16, state_dim=16, read_geometry="seq"),
                DABSNLayerSpec(hidden_dim=16, state_dim=16, read_geometry="seq")],
    ).eval().cuda()


def _ids(seed=3, tokens=TOKENS):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, VOCAB, (BATCH, tokens), generator=g).cuda()


def _selective(model):
    with torch.no_grad():
        for block in model.backbone.blocks:
            block.read.admit_window.fill_(-3.0)


@pytest.mark.parametrize("chunk_size", [None, 1, 7, 16, 48])
def test_chunked_ingest_matches_dense_forward(b200, chunk_size):
    from dabsn.memory import forward_with_memory

    model, ids = _model(), _ids()
    with torch.no_grad():
        reference = model.forward_sequence(ids)
    logits, memory = forward_with_memory(model, ids, chunk_size=chunk_size, extend=True)
    assert torch.allclose(logits, reference, atol=ATOL, rtol=RTOL), \
        float((logits - reference).abs().max())
    assert memory.position == TOKENS and memory.entries == TOKENS
    assert model.backbone.blocks[0].read._last_three_way_backend == "b200_flash_exact"


def test_selective_bank_matches_dense_forward(b200):
    from dabsn.memory import forward_with_memory

    model, ids = _model(), _ids()
    _selective(model)
    with torch.no_grad():
        reference = model.forward_sequence(ids)
    assert model.backbone.blocks[0].read.last_n_max < TOKENS, "bank was not sparse"
    logits, _ = forward_with_memory(model, ids, chunk_size=8, extend=True)
    assert torch.allclose(logits, reference, atol=ATOL, rtol=RTOL)


def test_split_ingest_then_query_and_decode(b200):
    from dabsn.memory import forward_with_memory, ingest

    model, ids = _model(), _ids()
    with torch.no_grad():
        reference = model.forward_sequence(ids)[:, 32:]
    memory = ingest(model, ids[:, :32], chunk_size=8)
    logits, unchanged = forward_with_memory(model, ids[:, 32:], memory)
    assert torch.allclose(logits, reference, atol=ATOL, rtol=RTOL)
    assert unchanged is memory and memory.entries == 32
    steps = []
    for i in range(ids.shape[1] - 32):
        step, memory = forward_with_memory(model, ids[:, 32 + i:33 + i], memory, extend=True)
        steps.append(step)
    assert torch.allclose(torch.cat(steps, dim=1), reference, atol=ATOL, rtol=RTOL)
    assert memory.entries == TOKENS


def test_query_bank_read_gradients_match_cpu_reference(b200):
    """forward_query_bank with bank positions before the window (negative
    relative positions) through the B200 read, forward and backward."""
    from dabsn.read import DABSNRead

    torch.manual_seed(5)
    H, L, start = 32, 96, 40
    read_cpu = DABSNRead(H, "seq")
    read_gpu = copy.deepcopy(read_cpu).cuda()
    g = torch.Generator().manual_seed(7)
    bank = {
        "write": torch.randn(BATCH, L, H, generator=g),
        "novelty": torch.rand(BATCH, L, H, generator=g),
        "p": torch.rand(BATCH, L, H, generator=g) * 0.3,
        "energy": torch.rand(BATCH, L, H, generator=g),
        "saturation": torch.rand(BATCH, L, H, generator=g),
    }
    q_len = L - start
    y = torch.randn(BATCH, q_len, H, generator=g)
    budget = torch.randn(BATCH, q_len, H, generator=g)
    expr = torch.randn(BATCH, q_len, H, generator=g)

    def run(read, dev):
        leaves = [t.to(dev).requires_grad_() for t in (y, budget, expr, bank["write"])]
        bw = leaves[3]
        out = read.forward_query_bank(
            leaves[0], leaves[1], leaves[2], bw[:, start:], bank["novelty"].to(dev)[:, start:],
            bank["p"].to(dev)[:, start:], bank["energy"].to(dev)[:, start:],
            bank["saturation"].to(dev)[:, start:], bank_y=None, bank_b=None, bank_ay=None,
            bank_write=bw, bank_novelty=bank["novelty"].to(dev), bank_p=bank["p"].to(dev),
            bank_energy=bank["energy"].to(dev), bank_saturation=bank["saturation"].to(dev),
            query_start=start)
        w = torch.randn(out.shape, generator=torch.Generator().manual_seed(1)).to(dev)
        grads = torch.autograd.grad((out * w).sum(), leaves + list(read.parameters()),
                                    allow_unused=True)
        return out, grads

    out_c, g_c = run(read_cpu, "cpu")
    out_g, g_g = run(read_gpu, "cuda")
    assert read_gpu._last_three_way_backend == "b200_flash_exact"
    assert max_rel_err(out_g, out_c) <= RTOL
    scale = max(float(x.abs().max()) for x in g_c if x is not None)
    for a, e in zip(g_g, g_c):
        if e is None:
            assert a is None or float(a.abs().max()) == 0.0
            continue
        err = float((a.double().cpu() - e.double()).abs().max())
        assert err <= GRAD_TOL * max(float(e.abs().max()), 1e-3 * scale), err
