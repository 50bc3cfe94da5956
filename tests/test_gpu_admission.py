"""Fused read admission and admitted bank against the oracle and against the
reference's own glue (read.py:152-303).

Bank membership, order, width and validity are integer results and must be
identical; values match the float64 oracle within the FP32 bars (forward
1e-4, gradients 1e-3, max |a - e| / max |e|).  Under BF16 autocast a block
through the fused path matches the same block through the reference's glue
(same kernels everywhere else) within the BF16 bar, with the same bank.
"""

from __future__ import annotations

import pytest
import torch

import dabsn_oracle as O
from conftest import max_rel_err, reference_available

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
BF16_TOL = 3e-2
PARAMS = ("p_gain", "novelty_gain", "null_bias", "adm_p_gain", "adm_novelty_gain",
          "adm_saturation_gain", "adm_energy_gain", "adm_bias")
OUT_NAMES = ("query", "cocktail", "bank_keys", "bank_writes", "next_writes", "bank_cocktail",
             "bank_key_bias", "bank_admission")


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def _tapes(B, T, H, seed):
    g = torch.Generator().manual_seed(seed)
    expr = torch.randn(B, T, H, generator=g, dtype=torch.float64)
    write = torch.randn(B, T, H, generator=g, dtype=torch.float64)
    nov = torch.rand(B, T, H, generator=g, dtype=torch.float64)
    plast = torch.rand(B, T, H, generator=g, dtype=torch.float64) * 0.3
    energy = torch.rand(B, T, H, generator=g, dtype=torch.float64)
    sat = torch.rand(B, T, H, generator=g, dtype=torch.float64)
    init = dict(p_gain=1.0, novelty_gain=0.5, null_bias=-2.0, adm_p_gain=1.0,
                adm_novelty_gain=0.5, adm_saturation_gain=0.5, adm_energy_gain=0.25,
                adm_bias=-2.0)
    params = {k: torch.tensor([v + 0.1 * float(torch.randn(1, generator=g))],
                              dtype=torch.float64) for k, v in init.items()}
    params["log_temp"] = torch.tensor([0.0], dtype=torch.float64)
    params["admit_window"] = torch.tensor([0.3], dtype=torch.float64)
    return [expr, write, nov, plast, energy, sat], params


def _device_bank(tapes, params, mode, n_cap=None):
    from dabsn_b200 import autograd as AG

    dev = _dev()
    leaves = [t.to(dev, torch.float32).requires_grad_() for t in tapes]
    pl = [params[k].to(dev, torch.float32).requires_grad_() for k in PARAMS]
    window = torch.nn.functional.softplus(params["admit_window"].to(dev, torch.float32))
    outs = AG.AdmittedBank.apply(*leaves, *pl, window, mode, n_cap)
    return leaves, pl, outs


@pytest.mark.parametrize("B,T,H,geometry", [
    (2, 37, 24, "seq"), (3, 64, 128, "seq"), (2, 50, 96, "field"), (2, 1500, 64, "seq"),
])
def test_admission_matches_oracle(B, T, H, geometry):
    tapes, params = _tapes(B, T, H, B * 100 + T + H)
    ref_leaves = [t.clone().requires_grad_() for t in tapes]
    ref_params = {k: v.clone().requires_grad_() for k, v in params.items()}
    ref = O.admitted_bank(*ref_leaves, ref_params, geometry=geometry)
    mode = 0 if geometry == "seq" else 1
    leaves, pl, outs = _device_bank(tapes, params, mode)
    query, cocktail, bk, bw, nw, bc, bb, ba, bi, bv = outs
    assert int(bi.shape[1]) == ref["n_max"]
    assert torch.equal(bi.cpu(), ref["bank_idx"])
    assert torch.equal(bv.cpu(), ref["bank_valid"])
    got = dict(query=query, cocktail=cocktail, bank_keys=bk, bank_writes=bw, next_writes=nw,
               bank_cocktail=bc, bank_key_bias=bb, bank_admission=ba)
    for name in OUT_NAMES:
        assert max_rel_err(got[name], ref[name]) <= FWD_TOL, (name, max_rel_err(got[name], ref[name]))
    g = torch.Generator().manual_seed(9)
    ws = {n: torch.randn(ref[n].shape, generator=g, dtype=torch.float64) for n in OUT_NAMES}
    # padded (invalid) bank entries receive no gradient from the read
    for n in ("bank_keys", "bank_writes", "next_writes", "bank_cocktail", "bank_key_bias",
              "bank_admission"):
        mask = ref["bank_valid"].reshape(ref["bank_valid"].shape + (1,) * (ws[n].dim() - 2))
        ws[n] = ws[n] * mask
    loss_ref = sum((ref[n] * ws[n]).sum() for n in OUT_NAMES)
    ref_grads = torch.autograd.grad(loss_ref, ref_leaves + [ref_params[k] for k in PARAMS])
    loss = sum((got[n] * ws[n].to(got[n].device, got[n].dtype)).sum() for n in OUT_NAMES)
    grads = torch.autograd.grad(loss, leaves + pl)
    names = ["expression", "write", "novelty", "plasticity", "energy", "saturation", *PARAMS]
    scale = max(float(e.abs().max()) for e in ref_grads)
    for n, a, e in zip(names, grads, ref_grads):
        err = float((a.double().cpu() - e).abs().max())
        assert err <= GRAD_TOL * max(float(e.abs().max()), 1e-3 * scale), (n, err)


@pytest.mark.parametrize("H", [1032, 2048, 4104, 4100])
def test_admission_bf16_matches_oracle(H):
    """BF16 activations under autocast: query and keys come out in BF16 and
    the backward reads BF16 gradients (one, two or four 8-element words per
    thread; 4100 takes the element-wise kernel).  Everyone is admitted (a wide
    window), so the bank cannot differ through BF16 rounding of the scores;
    values and gradients match the float64 oracle on the BF16-rounded inputs
    within the BF16 bar."""
    from dabsn_b200 import autograd as AG

    dev = _dev()
    B, T = 2, 48
    tapes, params = _tapes(B, T, H, H)
    params["admit_window"] = torch.tensor([50.0], dtype=torch.float64)
    tapes = [t.to(torch.bfloat16).double() for t in tapes]
    ref_leaves = [t.clone().requires_grad_() for t in tapes]
    ref_params = {k: v.clone().requires_grad_() for k, v in params.items()}
    ref = O.admitted_bank(*ref_leaves, ref_params, geometry="seq")
    leaves = [t.to(dev, torch.bfloat16).requires_grad_() for t in tapes]
    pl = [params[k].to(dev, torch.float32).requires_grad_() for k in PARAMS]
    window = torch.nn.functional.softplus(params["admit_window"].to(dev, torch.float32))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        outs = AG.AdmittedBank.apply(*leaves, *pl, window, 0, None)
    query, cocktail, bk, bw, nw, bc, bb, ba, bi, bv = outs
    assert query.dtype == torch.bfloat16 and bk.dtype == torch.bfloat16
    assert torch.equal(bi.cpu(), ref["bank_idx"]) and torch.equal(bv.cpu(), ref["bank_valid"])
    got = dict(query=query, cocktail=cocktail, bank_keys=bk, bank_writes=bw, next_writes=nw,
               bank_cocktail=bc, bank_key_bias=bb, bank_admission=ba)
    for name in OUT_NAMES:
        assert max_rel_err(got[name], ref[name]) <= BF16_TOL, (name, max_rel_err(got[name], ref[name]))
    g = torch.Generator().manual_seed(5)
    ws = {n: torch.randn(ref[n].shape, generator=g, dtype=torch.float64) for n in OUT_NAMES}
    loss_ref = sum((ref[n] * ws[n]).sum() for n in OUT_NAMES)
    ref_grads = torch.autograd.grad(loss_ref, ref_leaves + [ref_params[k] for k in PARAMS])
    loss = sum((got[n].float() * ws[n].to(dev, torch.float32)).sum() for n in OUT_NAMES)
    grads = torch.autograd.grad(loss, leaves + pl)
    names = ["expression", "write", "novelty", "plasticity", "energy", "saturation"]
    for n, a, e in zip(names, grads[:6], ref_grads[:6]):
        rel = float((a.double().cpu() - e).norm()) / max(float(e.norm()), 1e-12)
        assert rel <= 5e-2 or float(e.norm()) < 1e-6, (n, rel)
    # The 8 parameter gradients are sums over tokens of (BF16-rounded mean) x
    # (token gradient); a single one can cancel to far below its terms, so
    # they are compared as one vector.
    a = torch.cat([x.double().cpu().reshape(-1) for x in grads[6:]])
    e = torch.cat([x.reshape(-1) for x in ref_grads[6:]])
    assert float((a - e).norm()) <= 5e-2 * float(e.norm()), (a, e)


def test_admission_capped_width():
    """A fixed bank width below the member count (the capture-width policy):
    members beyond it are not gathered and receive no bank gradient."""
    tapes, params = _tapes(2, 40, 32, 3)
    params["admit_window"] = torch.tensor([50.0], dtype=torch.float64)  # everyone admitted
    leaves, pl, outs = _device_bank(tapes, params, 0, n_cap=10)
    bi, bv = outs[8], outs[9]
    assert bi.shape[1] == 10 and bool(bv.all())
    assert torch.equal(bi.cpu(), torch.arange(10).expand(2, 10))
    bw = outs[3]
    dwrite = torch.autograd.grad(bw.sum(), leaves[1])[0]
    assert float(dwrite[:, 10:].abs().max()) == 0.0
    assert float((dwrite[:, :10] - 1).abs().max()) == 0.0


@pytest.mark.parametrize("H,B,T", [(256, 4, 80), (1056, 2, 64), (2048, 2, 96)])
def test_block_bf16_fused_admission_matches_reference_glue(H, B, T):
    """A thread slice per token (256) and a full CTA per token (1056, 2048) in
    the backward; BF16 query, keys and gradients cross between the admission
    and the read, and the read hands its BF16 result to the fused output
    projection."""
    if not reference_available():
        pytest.skip("reference package (baseline/_ref) not installed")
    _dev()
    import dabsn_b200

    dabsn_b200.install()
    import dabsn.kernels
    from dabsn.model import DABSNBlock
    from dabsn.read import DABSNRead

    dabsn.kernels.enable("cuda", required=True)
    fused = DABSNRead._unified_forward
    original = fused.__wrapped_reference__
    torch.manual_seed(0)
    block = DABSNBlock(H, H, H, "seq").cuda()
    x = torch.randn(B, T, H, device="cuda")
    results = []
    for impl in (fused, original):
        DABSNRead._unified_forward = impl
        try:
            block.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = block.forward_world(x)
            out.float().square().mean().backward()
            results.append((out.detach().float(), block.read.last_n_max,
                            {n: p.grad.detach().float().clone() for n, p in block.named_parameters()
                             if p.grad is not None}))
        finally:
            DABSNRead._unified_forward = fused
    (o1, n1, g1), (o2, n2, g2) = results
    assert n1 == n2
    assert max_rel_err(o1, o2) <= BF16_TOL
    assert set(g1) == set(g2)
    for name in g1:
        e = g2[name]
        rel = float((g1[name] - e).norm()) / max(float(e.norm()), 1e-12)
        assert rel <= 5e-2 or float(e.norm()) < 1e-6, (name, rel)
