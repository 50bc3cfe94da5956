"""Generate the golden fixtures from the reference implementation itself.

Run in a container that has the reference source tree (not on the GPU box):

    CXX=/usr/bin/g++ python tests/golden/make_golden.py --reference-src <path to dabsn/src>

Each fixture stores seeded inputs, the reference's outputs and the reference's
gradients of a fixed random linear functional of the outputs.  They pin
``oracle/dabsn_oracle.py`` (``tests/test_oracle_golden.py``) and are replayed
through the CUDA path by the GPU tests.  Sizes are small so the files stay a
few hundred KB in total.

Reference entry points exercised (paths inside the reference project):
  * ``dabsn::core_scan_batched``  src/dabsn/kernels/batched_runtime.py:1507-1634
  * ``dense_bmm_three_way_read_exact``  src/dabsn/kernels/compact_admitted.py:16-80
  * ``DABSNRead._long_scan_from_state`` loop  src/dabsn/read.py:577-640
  * ``DABSNBlock.forward_world`` (seq)  src/dabsn/model.py:309-372
  * ``_scan_forward`` / ``_scan_backward`` (delta-rule scan of
    ``dabsn::permanent_delta_scan``)  src/dabsn/kernels/permanent.py:56-110
  * ``dabsn::local_field_gather`` and its registered backward
    src/dabsn/kernels/local_field.py:208-240
  * ``chunked_linear_cross_entropy`` (single-shot and chunked branches, with
    ignored targets and with every target ignored)
    src/dabsn/runtime/loss.py:138-184
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _core_inputs(B, T, H, dtype, seed):
    g = torch.Generator().manual_seed(seed)

    def r(*shape, scale=1.0, shift=0.0):
        return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale + shift).to(dtype)

    inputs = [
        r(B, T, H),  # Wx
        r(B, T, H, scale=2.0),  # Wgx
        r(H, H, scale=1.0 / H**0.5),  # Ug
        r(H, H, scale=0.5 / H**0.5),  # A
        r(H, scale=0.1),  # beta
        r(H, scale=0.3, shift=-2.25),  # log_kappa
        r(H, scale=0.5, shift=-1.0),  # logit_recover
    ]
    inputs += [r(H, scale=0.5) for _ in range(10)]  # k_s..r_bias
    inputs += [r(H, scale=0.3, shift=2.2)]  # logit_c_decay
    inputs += [r(H, scale=0.5), r(H, scale=0.5)]  # k_c, r_c
    inputs += [r((), shift=-2.0, scale=0.2), r((), shift=-1.0, scale=0.2), r((), shift=-3.0, scale=0.2)]
    inputs += [r(B, H, scale=0.3), torch.rand(B, H, generator=g, dtype=torch.float64).to(dtype), r(B, H, scale=0.1).abs()]
    return inputs


def make_core(ref, B, T, H, dtype, seed):
    from dabsn.kernels.batched_runtime import _core_scan_batched_op

    inputs = [x.clone().requires_grad_(True) for x in _core_inputs(B, T, H, dtype, seed)]
    outs = _core_scan_batched_op(*inputs)
    g = torch.Generator().manual_seed(seed + 1)
    weights = [torch.randn(o.shape, generator=g, dtype=torch.float64).to(o.dtype) for o in outs]
    loss = sum((o * w).sum() for o, w in zip(outs, weights))
    grads = torch.autograd.grad(loss, inputs)
    return {
        "inputs": [x.detach() for x in inputs],
        "outputs": [o.detach() for o in outs],
        "out_weights": weights,
        "grads": [gr.detach() for gr in grads],
    }


def _read_inputs(B, T, H, dtype, seed, drop):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, generator=g, dtype=torch.float64), dim=-1)
    writes = torch.randn(B, T, H, generator=g, dtype=torch.float64)
    member = torch.rand(B, T, generator=g, dtype=torch.float64) > drop
    member[:, 0] = True
    counts = member.sum(1)
    order = torch.argsort(member.double(), dim=1, descending=True, stable=True)
    N = int(counts.max())
    idx = order[:, :N]
    valid = torch.arange(N).unsqueeze(0) < counts.unsqueeze(1)
    bank_writes = torch.gather(writes, 1, idx.unsqueeze(-1).expand(-1, -1, H))
    bank_keys = torch.nn.functional.normalize(bank_writes, dim=-1)
    nidx = (idx + 1).clamp(max=T - 1)
    next_writes = torch.gather(writes, 1, nidx.unsqueeze(-1).expand(-1, -1, H))
    cocktail = torch.nn.functional.normalize(torch.rand(B, T, 4, generator=g, dtype=torch.float64), dim=-1)
    bank_cocktail = torch.gather(cocktail, 1, idx.unsqueeze(-1).expand(-1, -1, 4))
    kb = torch.randn(B, T, generator=g, dtype=torch.float64)
    adm = torch.randn(B, T, generator=g, dtype=torch.float64)
    bank_kb = torch.gather(kb, 1, idx)
    bank_adm = torch.gather(adm, 1, idx)
    scale = torch.tensor([2.0 * H**0.5], dtype=torch.float64)
    gains = [torch.tensor([v], dtype=torch.float64) for v in (1.0, 0.8, 0.3, 1.2)]
    diff = [q, bank_keys, bank_writes, next_writes, cocktail, bank_cocktail, bank_kb, bank_adm, scale, *gains]
    diff = [x.to(dtype) for x in diff]
    return diff, idx, valid


def make_read(ref, B, T, H, dtype, seed, mode, drop):
    from dabsn.kernels.compact_admitted import dense_bmm_three_way_read_exact

    diff, idx, valid = _read_inputs(B, T, H, dtype, seed, drop)
    diff = [x.clone().requires_grad_(True) for x in diff]
    q, k, w, nw, cc, bcc, kb, adm, scale, sg, pg, ig, cg = diff
    out = dense_bmm_three_way_read_exact(
        q, k, w, nw, cc, bcc, kb, adm, scale, idx, valid,
        mode=mode, short_gain=sg, pad_gain=pg, induct_gain=ig, cocktail_gain=cg,
    )
    g = torch.Generator().manual_seed(seed + 1)
    weight = torch.randn(out.shape, generator=g, dtype=torch.float64).to(out.dtype)
    grads = torch.autograd.grad((out * weight).sum(), diff)
    return {
        "inputs": [x.detach() for x in diff],
        "bank_idx": idx,
        "bank_valid": valid,
        "mode": mode,
        "output": out.detach(),
        "out_weight": weight,
        "grads": [gr.detach() for gr in grads],
    }


def make_long(ref, B, T, H, dtype, seed, with_state):
    from dabsn.read import DABSNRead

    torch.manual_seed(seed)
    read = DABSNRead(H, "seq").to(dtype)
    with torch.no_grad():
        for name in ("logit_retain", "logit_expect_retain", "logit_retention_decay", "logit_retention_strength"):
            getattr(read, name).add_(torch.randn(1, dtype=dtype) * 0.5)
    g = torch.Generator().manual_seed(seed)
    write = (torch.randn(B, T, H, generator=g, dtype=torch.float64)).to(dtype).requires_grad_(True)
    plast = torch.rand(B, T, H, generator=g, dtype=torch.float64).to(dtype).requires_grad_(True)
    state = None
    if with_state:
        state = tuple(
            (torch.randn(B, H, generator=g, dtype=torch.float64) * s + o).to(dtype).requires_grad_(True)
            for s, o in ((0.3, 0.0), (0.3, 0.0), (0.2, 0.8))
        )
    assert not getattr(DABSNRead, "_long_native_enabled", False)
    out, final = read._long_scan_from_state(
        write, plast, write, initial_state=state, return_final_state=True
    )
    params = [read.logit_retain, read.logit_expect_retain, read.logit_retention_decay, read.logit_retention_strength]
    wg = torch.Generator().manual_seed(seed + 1)
    weight = torch.randn(out.shape, generator=wg, dtype=torch.float64).to(out.dtype)
    fweights = [torch.randn(f.shape, generator=wg, dtype=torch.float64).to(f.dtype) for f in final]
    loss = (out * weight).sum() + sum((f * fw).sum() for f, fw in zip(final, fweights))
    wrt = [write, plast, *params] + (list(state) if state is not None else [])
    grads = torch.autograd.grad(loss, wrt)
    return {
        "write": write.detach(),
        "plasticity": plast.detach(),
        "params": [p.detach().clone() for p in params],
        "initial_state": None if state is None else [s.detach() for s in state],
        "output": out.detach(),
        "final": [f.detach() for f in final],
        "out_weight": weight,
        "final_weights": fweights,
        "grads": [gr.detach() for gr in grads],
    }


def make_block(ref, B, T, D, H, dtype, seed):
    from dabsn.model import DABSNBlock

    torch.manual_seed(seed)
    block = DABSNBlock(D, H, H, "seq").to(dtype)
    with torch.no_grad():
        for name, p in block.named_parameters():
            if p.dim() == 1 and p.numel() > 0:
                p.add_(torch.randn_like(p) * 0.1)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g, dtype=torch.float64).to(dtype).requires_grad_(True)
    out = block.forward_world(x)
    weight = torch.randn(out.shape, generator=g, dtype=torch.float64).to(out.dtype)
    names = [n for n, _ in block.named_parameters()]
    params = [p for _, p in block.named_parameters()]
    grads = torch.autograd.grad((out * weight).sum(), [x, *params], allow_unused=True)
    grads = [torch.zeros_like(p) if gr is None else gr for p, gr in zip([x, *params], grads)]
    return {
        "x": x.detach(),
        "state_dict": {k: v.detach().clone() for k, v in block.state_dict().items()},
        "param_names": names,
        "output": out.detach(),
        "out_weight": weight,
        "grad_x": grads[0].detach(),
        "grad_params": {n: gr.detach() for n, gr in zip(names, grads[1:])},
        "n_max": block.read.last_n_max,
    }


def make_permanent(B, T, h, dtype, seed):
    from dabsn.kernels.permanent import _scan_backward, _scan_forward

    g = torch.Generator().manual_seed(seed)
    k = torch.nn.functional.normalize(torch.randn(B, T, h, generator=g, dtype=dtype), dim=-1)
    v = torch.randn(B, T, h, generator=g, dtype=dtype)
    beta = torch.rand(B, T, generator=g, dtype=dtype)
    out_weight = torch.randn(B, T, h, generator=g, dtype=dtype)
    out = _scan_forward(k, v, beta)
    dk, dv, dbeta = _scan_backward(k, v, beta, out_weight)
    return {"inputs": [k, v, beta], "output": out, "out_weight": out_weight,
            "grads": [dk, dv, dbeta]}


def make_local_field(B, C, N, K, D, dtype, seed):
    from dabsn.kernels.local_field import _local_field_gather_op

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, C, D, generator=g, dtype=dtype, requires_grad=True)
    patch = torch.randint(0, C, (N, K), generator=g)
    out = _local_field_gather_op(x, patch)
    out_weight = torch.randn(out.shape, generator=g, dtype=dtype)
    (gx,) = torch.autograd.grad((out * out_weight).sum(), [x])
    return {"inputs": [x.detach()], "patch": patch, "output": out.detach(),
            "out_weight": out_weight, "grads": [gx]}


def make_linear_ce(rows, V, D, dtype, seed, chunk_budget, all_ignored=False):
    from dabsn.runtime.loss import chunked_linear_cross_entropy

    g = torch.Generator().manual_seed(seed)
    h = torch.randn(rows, D, generator=g, dtype=dtype, requires_grad=True)
    w = (torch.randn(V, D, generator=g, dtype=dtype) / D**0.5).requires_grad_()
    b = (0.1 * torch.randn(V, generator=g, dtype=dtype)).requires_grad_()
    t = torch.randint(0, V, (rows,), generator=g)
    t[::5] = -100
    if all_ignored:
        t[:] = -100
    loss = chunked_linear_cross_entropy(h, w, b, t, chunk_budget=chunk_budget)
    grads = torch.autograd.grad(loss, [h, w, b])
    return {"inputs": [h.detach(), w.detach(), b.detach()], "targets": t,
            "chunk_budget": chunk_budget, "single_shot": chunk_budget is None,
            "loss": loss.detach(), "grads": [gr.detach() for gr in grads]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", default=None, help="comma-separated fixture names to (re)write")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    os.environ.setdefault("DABSN_SILENCE_ROUTING", "1")
    import dabsn  # noqa: F401  (the reference package)

    torch.manual_seed(0)
    out = Path(args.out)
    fixtures = {
        "core_f64_small": make_core(None, 2, 5, 3, torch.float64, 11),
        "core_f64": make_core(None, 3, 17, 8, torch.float64, 12),
        "core_f32": make_core(None, 4, 33, 16, torch.float32, 13),
        "read_seq_f64_full": make_read(None, 2, 9, 5, torch.float64, 21, "seq", 0.0),
        "read_seq_f64_sparse": make_read(None, 3, 20, 8, torch.float64, 22, "seq", 0.5),
        "read_field_f64_sparse": make_read(None, 2, 13, 6, torch.float64, 23, "field", 0.4),
        "read_seq_f32": make_read(None, 2, 40, 16, torch.float32, 24, "seq", 0.3),
        "long_f64": make_long(None, 2, 11, 5, torch.float64, 31, False),
        "long_f64_state": make_long(None, 3, 7, 4, torch.float64, 32, True),
        "long_f32": make_long(None, 2, 40, 16, torch.float32, 33, False),
        "block_f64": make_block(None, 2, 12, 6, 8, torch.float64, 41),
        "block_f32": make_block(None, 3, 24, 16, 16, torch.float32, 42),
        "permanent_f64": make_permanent(2, 70, 16, torch.float64, 51),
        "permanent_f32": make_permanent(3, 150, 32, torch.float32, 52),
        "local_field_f64": make_local_field(2, 11, 9, 5, 3, torch.float64, 61),
        # 37 x 50 logits: one shot by default, chunked (4 rows) under a 200 budget
        "linear_ce_f64_single": make_linear_ce(37, 50, 16, torch.float64, 71, None),
        "linear_ce_f64_chunked": make_linear_ce(37, 50, 16, torch.float64, 72, 200),
        "linear_ce_f64_empty_single": make_linear_ce(9, 7, 8, torch.float64, 73, None, True),
        "linear_ce_f64_empty_chunked": make_linear_ce(9, 7, 8, torch.float64, 74, 20, True),
    }
    only = None if args.only is None else set(args.only.split(","))
    for name, data in fixtures.items():
        if only is not None and name not in only:
            continue
        torch.save(data, out / f"{name}.pt")
        print("wrote", name)


if __name__ == "__main__":
    main()
