"""Tensor parallelism over state units on two GPUs.

Each rank wraps its slice of one core in the reference's
``TensorParallelDABSNCore`` (core.py:609-874) and runs the B200 cross-GPU scan
(BF16, autocast); the same core unsplit runs the single-GPU grid-wide scan on
the same inputs.  Public tapes, final states and every gradient (local
parameter slices, the summed scalar and input gradients) must agree within
two BF16 ulps of the outputs (max |a - e| / max |e| <= 1e-2) and 2e-2 normwise
for gradients (the two launch the same kernels but split the step's product
over different CTA sets, so summation orders differ).  Skipped with fewer
than two GPUs.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2
GRAD_TOL = 2e-2


def _rel(a, e):
    a, e = a.detach().double().cpu(), e.detach().double().cpu()
    return float((a - e).abs().max()) / max(float(e.abs().max()), 1e-12)


def _norm_rel(a, e):
    a, e = a.detach().double().cpu(), e.detach().double().cpu()
    return float((a - e).norm()) / max(float(e.norm()), 1e-12)


def _worker(rank, world, port, root, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        sys.path[:0] = [root, str(Path(root) / "baseline" / "_ref")]
        import dabsn_b200

        dabsn_b200.install()
        import dabsn.kernels
        from dabsn.core import DABSNCore, TensorParallelDABSNCore

        dabsn.kernels.enable("cuda", required=True)
        torch.manual_seed(0)
        D, H, B, T = 64, 512, 4, 24
        src = DABSNCore(D, H).cuda()
        tp = TensorParallelDABSNCore(src, group=dist.group.WORLD, rank=rank,
                                     world_size=world).cuda()
        g = torch.Generator().manual_seed(1)
        x = torch.randn(B, T, D, generator=g).cuda()
        weights = None
        res = {}
        for name, core in (("tp", tp), ("full", src)):
            xi = x.clone().requires_grad_()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                fields, final = core.forward_from_state(xi, return_cocktail=True,
                                                        return_final_state=True)
            outs = [t.float() for t in (*fields, *final)]
            if weights is None:
                gw = torch.Generator().manual_seed(2)
                weights = [torch.randn(o.shape, generator=gw).cuda() for o in outs]
            sum((o * w).sum() for o, w in zip(outs, weights)).backward()
            res[name] = (outs, xi.grad, core)
        errs = {}
        for i, (a, e) in enumerate(zip(res["tp"][0], res["full"][0])):
            errs[f"out{i}"] = (_rel(a, e), OUT_TOL)
        errs["input_grad"] = (_norm_rel(res["tp"][1], res["full"][1]), GRAD_TOL)
        cut = tp.tensor_slice
        for name, p in tp.named_parameters():
            q = dict(src.named_parameters())[name]
            if p.grad is None:
                continue
            ref = q.grad
            if p.shape != q.shape:  # this rank's rows / units
                ref = ref[cut]
            errs[name] = (_norm_rel(p.grad, ref), GRAD_TOL)
        out[rank] = {"errs": errs, "backend": tp._last_core_backend,
                     "status": int(__import__("dabsn_b200")._native.device_status())}
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_scan_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    root = str(Path(__file__).resolve().parents[1])
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, root, out), nprocs=2, join=True)
    for rank in (0, 1):
        r = out[rank]
        assert r["backend"] == "tensor_parallel_b200"
        assert r["status"] == 0
        bad = {k: v for k, (v, tol) in r["errs"].items() if not v <= tol}
        assert not bad, (rank, bad)
