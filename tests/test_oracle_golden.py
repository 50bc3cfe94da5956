"""Pin the CPU oracle against fixtures recorded from the reference itself."""

from __future__ import annotations

import pytest
import torch

import dabsn_oracle as O
from conftest import load_golden, max_rel_err

CORE = ["core_f64_small", "core_f64", "core_f32"]
READ = ["read_seq_f64_full", "read_seq_f64_sparse", "read_field_f64_sparse", "read_seq_f32"]
LONG = ["long_f64", "long_f64_state", "long_f32"]


def _tol(dtype):
    return 1e-10 if dtype == torch.float64 else 2e-5


@pytest.mark.parametrize("name", CORE)
def test_core_scan_oracle_matches_reference(name):
    fx = load_golden(name)
    inputs = [x.clone().requires_grad_(True) for x in fx["inputs"]]
    # the reference runs its state chain in FP32 for every activation dtype
    outs = O.core_scan(*inputs, state_dtype=torch.float32)
    tol = 1e-6
    for got, ref in zip(outs, fx["outputs"]):
        assert max_rel_err(got, ref) < tol
    # The reference's registered autograd ignores the gradient of the gate
    # tape (output 7; batched_runtime.py:1613-1620), which no caller consumes.
    weights = list(fx["out_weights"])
    weights[7] = torch.zeros_like(weights[7])
    loss = sum((o * w).sum() for o, w in zip(outs, weights))
    grads = torch.autograd.grad(loss, inputs)
    for i, (got, ref) in enumerate(zip(grads, fx["grads"])):
        assert max_rel_err(got, ref) < 50 * tol, i


@pytest.mark.parametrize("name", READ)
def test_read_oracle_matches_reference(name):
    fx = load_golden(name)
    diff = [x.clone().requires_grad_(True) for x in fx["inputs"]]
    q, k, w, nw, cc, bcc, kb, adm, scale, sg, pg, ig, cg = diff
    out = O.three_way_read(
        q, k, w, nw, cc, bcc, kb, adm, scale, fx["bank_idx"], fx["bank_valid"],
        mode=fx["mode"], short_gain=sg, pad_gain=pg, induct_gain=ig, cocktail_gain=cg,
        score_dtype=torch.float32,  # the reference forms scores in FP32
    )
    tol = 1e-6
    assert max_rel_err(out, fx["output"]) < tol
    grads = torch.autograd.grad((out * fx["out_weight"]).sum(), diff)
    for i, (got, ref) in enumerate(zip(grads, fx["grads"])):
        assert max_rel_err(got, ref) < 10 * tol, i


@pytest.mark.parametrize("name", LONG)
def test_long_oracle_matches_reference(name):
    fx = load_golden(name)
    write = fx["write"].clone().requires_grad_(True)
    plast = fx["plasticity"].clone().requires_grad_(True)
    params = [p.clone().requires_grad_(True) for p in fx["params"]]
    state = None
    if fx["initial_state"] is not None:
        state = [s.clone().requires_grad_(True) for s in fx["initial_state"]]
    out, final = O.long_scan(write, plast, *params, initial_state=state, return_final_state=True)
    tol = _tol(write.dtype)
    assert max_rel_err(out, fx["output"]) < tol
    for got, ref in zip(final, fx["final"]):
        assert max_rel_err(got, ref) < tol
    loss = (out * fx["out_weight"]).sum() + sum((f * w).sum() for f, w in zip(final, fx["final_weights"]))
    wrt = [write, plast, *params] + (state or [])
    grads = torch.autograd.grad(loss, wrt)
    for i, (got, ref) in enumerate(zip(grads, fx["grads"])):
        assert max_rel_err(got, ref) < 10 * tol, i


@pytest.mark.parametrize("name", ["block_f64", "block_f32"])
def test_block_oracle_matches_reference(name):
    fx = load_golden(name)
    params = {k: v.clone().requires_grad_(True) for k, v in fx["state_dict"].items()}
    x = fx["x"].clone().requires_grad_(True)
    # reference CPU path: FP32 core state chain, dense read in the input dtype
    out = O.block_forward(params, x, core_state_dtype=torch.float32)
    tol = 1e-6
    assert max_rel_err(out, fx["output"]) < 10 * tol
    names = fx["param_names"]
    grads = torch.autograd.grad((out * fx["out_weight"]).sum(), [x, *[params[n] for n in names]], allow_unused=True)
    assert max_rel_err(grads[0], fx["grad_x"]) < 100 * tol
    for n, g in zip(names, grads[1:]):
        ref = fx["grad_params"][n]
        if g is None:
            assert float(ref.abs().max()) == 0.0, n
        else:
            # scalar gains sum many cancelling terms: FP32 noise is absolute
            err = float((g.double() - ref.double()).abs().max())
            assert err <= 100 * tol * float(ref.abs().max()) + 1e-8, n


@pytest.mark.parametrize("name", ["permanent_f64", "permanent_f32"])
def test_permanent_delta_oracle_matches_reference(name):
    fx = load_golden(name)
    leaves = [t.clone().double().requires_grad_() for t in fx["inputs"]]
    out = O.permanent_delta_scan(*leaves)
    tol = 1e-10 if name.endswith("f64") else 1e-4
    assert max_rel_err(out, fx["output"]) <= tol
    grads = torch.autograd.grad((out * fx["out_weight"].double()).sum(), leaves)
    for a, e in zip(grads, fx["grads"]):
        assert max_rel_err(a, e) <= (1e-9 if name.endswith("f64") else 1e-3)


def test_local_field_oracle_matches_reference():
    fx = load_golden("local_field_f64")
    x = fx["inputs"][0].clone().requires_grad_()
    out = O.local_field_gather(x, fx["patch"])
    assert torch.equal(out, fx["output"])
    (gx,) = torch.autograd.grad((out * fx["out_weight"]).sum(), [x])
    assert max_rel_err(gx, fx["grads"][0]) <= 1e-12


LINEAR_CE = ["linear_ce_f64_single", "linear_ce_f64_chunked", "linear_ce_f64_empty_single",
             "linear_ce_f64_empty_chunked"]


@pytest.mark.parametrize("name", LINEAR_CE)
def test_linear_cross_entropy_oracle_matches_reference(name):
    fx = load_golden(name)
    h, w, b = (x.clone().requires_grad_(True) for x in fx["inputs"])
    loss = O.linear_cross_entropy(h, w, b, fx["targets"],
                                  empty="nan" if fx["single_shot"] else "zero")
    ref = fx["loss"]
    if torch.isnan(ref):
        assert torch.isnan(loss)
        # every target ignored: the reference's gradients are zero
        for g in fx["grads"]:
            assert float(g.abs().max()) == 0.0
        return
    assert abs(float(loss) - float(ref)) <= 1e-12 * max(1.0, abs(float(ref)))
    grads = torch.autograd.grad(loss, [h, w, b])
    for i, (got, want) in enumerate(zip(grads, fx["grads"])):
        if float(want.abs().max()) == 0.0:
            assert float(got.abs().max()) == 0.0, i
        else:
            assert max_rel_err(got, want) < 1e-10, (i, max_rel_err(got, want))
