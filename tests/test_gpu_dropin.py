"""Drop-in parity: the reference's own modules run unchanged on the B200
backend and match the reference's recorded results.

Needs the installed reference package (``baseline/_ref``); skipped otherwise.
"""

from __future__ import annotations

import copy

import pytest
import torch

from conftest import load_golden, max_rel_err, reference_available

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
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

    st = dabsn.kernels.enable("cuda", required=True)
    assert st["b200"]["enabled"] and st["active_backend"] == "b200"
    return dabsn_b200


def test_block_matches_reference_fixture(b200):
    from dabsn.model import DABSNBlock

    fx = load_golden("block_f32")
    D = fx["x"].shape[-1]
    H = fx["state_dict"]["core.Ug.weight"].shape[0]
    block = DABSNBlock(D, H, H, "seq")
    block.load_state_dict(fx["state_dict"])
    block = block.cuda()
    x = fx["x"].cuda().requires_grad_(True)
    out = block.forward_world(x)
    assert block.read._last_three_way_backend == "b200_flash_exact"
    assert block.read._last_long_backend == "b200_cuda"
    assert block.core._last_core_backend == "cuda_registered"
    assert max_rel_err(out, fx["output"]) <= FWD_TOL
    names = fx["param_names"]
    params = dict(block.named_parameters())
    grads = torch.autograd.grad((out * fx["out_weight"].cuda()).sum(), [x] + [params[n] for n in names],
                                allow_unused=True)
    assert max_rel_err(grads[0], fx["grad_x"]) <= GRAD_TOL
    scale = max(float(g.abs().max()) for g in fx["grad_params"].values())
    for n, g in zip(names, grads[1:]):
        ref = fx["grad_params"][n]
        if g is None:
            assert float(ref.abs().max()) == 0.0, n
            continue
        err = float((g.double().cpu() - ref.double()).abs().max())
        # tensor-relative, with a floor for near-zero scalar gains
        assert err <= GRAD_TOL * max(float(ref.abs().max()), 1e-3 * scale), (n, err)


def _c2_model(seed=0):
    from dabsn import DABSNSequenceLM

    torch.manual_seed(seed)
    return DABSNSequenceLM(64, 128, 1, layers="seq:128:128")


def test_sequence_lm_train_step_matches_cpu_reference(b200):
    """Config-2 model: one AdamW step on the B200 backend vs the reference CPU
    path (whose core scan runs the reference's own reverse)."""
    from dabsn.runtime.api import train_step

    model_cpu = _c2_model()
    model_gpu = copy.deepcopy(model_cpu).cuda()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 64, (8, 32), generator=g)
    tgt = torch.randint(0, 64, (8, 32), generator=g)

    def loss_fn(logits, targets):
        return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))

    class Seq(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.m = m

        def forward(self, x):
            return self.m.forward_sequence(x)

    # gradients of the same loss, before any optimizer step
    for m, dev in ((model_cpu, "cpu"), (model_gpu, "cuda")):
        m.zero_grad(set_to_none=True)
        loss_fn(m.forward_sequence(ids.to(dev)), tgt.to(dev)).backward()
    # Tensor-relative error, with a floor at 1e-3 of the largest gradient in the
    # model: scalar gains (cocktail_gain ...) sum many cancelling terms, so
    # their own magnitude is not a meaningful scale for FP32 rounding.
    scale = max(float(p.grad.abs().max()) for p in model_cpu.parameters() if p.grad is not None)
    for (n, pc), pg in zip(model_cpu.named_parameters(), model_gpu.parameters()):
        if pc.grad is None:
            assert pg.grad is None or float(pg.grad.abs().max()) == 0.0, n
            continue
        err = float((pg.grad.double().cpu() - pc.grad.double()).abs().max())
        assert err <= GRAD_TOL * max(float(pc.grad.abs().max()), 1e-3 * scale), (n, err)

    opt_c = torch.optim.AdamW(model_cpu.parameters(), lr=1e-3, weight_decay=0.1)
    opt_g = torch.optim.AdamW(model_gpu.parameters(), lr=1e-3, weight_decay=0.1)
    lc = train_step(Seq(model_cpu), ids, tgt, opt_c, loss_fn=loss_fn, clip_grad_norm=1.0)
    lg = train_step(Seq(model_gpu), ids.cuda(), tgt.cuda(), opt_g, loss_fn=loss_fn, clip_grad_norm=1.0)
    assert abs(lc - lg) <= 1e-4 * max(1.0, abs(lc))
    # Adam's first step is ~lr*sign(g): parameters agree to the gradient bar
    for (n, pc), pg in zip(model_cpu.named_parameters(), model_gpu.parameters()):
        assert max_rel_err(pg, pc) <= GRAD_TOL, n


def test_status_and_routes(b200):
    import dabsn.kernels

    st = dabsn.kernels.status()
    assert st["b200"]["available"] and st["b200"]["library_loaded"]
    assert "sm_100a" in st["b200"]["version"]


def test_wide_lm_bf16_autocast_trains(b200):
    """A width-512 LM under BF16 autocast runs the grid-wide scan and the
    tensor-core read end to end; one AdamW step gives finite gradients and a
    lower loss on the same batch."""
    from dabsn import DABSNSequenceLM

    torch.manual_seed(0)
    model = DABSNSequenceLM(128, 512, 1, layers="seq:512:512").cuda()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 128, (4, 96), generator=g).cuda()
    tgt = torch.randint(0, 128, (4, 96), generator=g).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    losses = []
    for _ in range(3):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model.forward_sequence(ids)
        loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, 128), tgt.reshape(-1))
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in model.parameters() if p.grad is not None)
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    blocks = [m for m in model.modules() if hasattr(m, "_last_three_way_backend")]
    assert blocks and all(b._last_three_way_backend == "b200_tensor_core" for b in blocks)


@pytest.mark.parametrize("geometry", ["field", "hybrid"])
def test_field_and_hybrid_geometry_grads_match_cpu_reference(b200, geometry):
    """Whole-sequence (field) and mixed (hybrid) read geometries: the fused
    admission takes the whole-sequence floor, the read the field masks (and,
    for hybrid, both reads with the learned gate); gradients of one loss match
    the reference CPU path."""
    from dabsn import DABSNSequenceLM

    torch.manual_seed(3)
    model_cpu = DABSNSequenceLM(48, 64, 2, layers=f"{geometry}:64:64,seq:64:64")
    model_gpu = copy.deepcopy(model_cpu).cuda()
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 48, (4, 40), generator=g)
    tgt = torch.randint(0, 48, (4, 40), generator=g)
    for m, dev in ((model_cpu, "cpu"), (model_gpu, "cuda")):
        m.zero_grad(set_to_none=True)
        logits = m.forward_sequence(ids.to(dev))
        torch.nn.functional.cross_entropy(logits.reshape(-1, 48), tgt.to(dev).reshape(-1)).backward()
    assert model_gpu.backbone.blocks[0].read.last_read_contract.get("admission_backend") == "b200_fused"
    scale = max(float(p.grad.abs().max()) for p in model_cpu.parameters() if p.grad is not None)
    for (n, pc), pg in zip(model_cpu.named_parameters(), model_gpu.parameters()):
        if pc.grad is None:
            assert pg.grad is None or float(pg.grad.abs().max()) == 0.0, n
            continue
        err = float((pg.grad.double().cpu() - pc.grad.double()).abs().max())
        assert err <= GRAD_TOL * max(float(pc.grad.abs().max()), 1e-3 * scale), (n, err)
