"""Child process of the BF16 drop-in test: the reference package's own CUDA
family (``dabsn.kernels.enable("cuda")``: its Triton/ATen path, no hooks of
this library) runs one forward + backward of a one-block ``DABSNSequenceLM``
at the wide-state widths of configs 4 and 5, under BF16 autocast and in FP32,
and saves logits, loss and every parameter gradient.  A separate process,
because the backend family is chosen once per process.

usage: python _reference_bf16_run.py OUT.pt H:T:B[,H:T:B...]
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.append(str(Path(__file__).resolve().parents[1] / "baseline" / "_ref"))

VOCAB = 32000


def model(H: int):
    from dabsn import DABSNSequenceLM

    torch.manual_seed(11)
    return DABSNSequenceLM(VOCAB, H, 1, layers=f"seq:{H}:{H}")


def batch(T: int, B: int):
    """Seeded Zipf(1.1) token ids and targets, as configs 4 and 5 use."""
    g = torch.Generator().manual_seed(21)
    p = torch.arange(1, VOCAB + 1, dtype=torch.float64).pow(-1.1)
    flat = torch.multinomial(p / p.sum(), 2 * B * T, replacement=True, generator=g)
    return flat[: B * T].reshape(B, T), flat[B * T:].reshape(B, T)


def run(m, ids, tgt, autocast: bool):
    """One forward + backward; returns logits, loss and gradients (CPU, FP32)."""
    m.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        logits = m.forward_sequence(ids)
    loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, VOCAB), tgt.reshape(-1))
    loss.backward()
    grads = {n: p.grad.float().cpu() for n, p in m.named_parameters() if p.grad is not None}
    return {"logits": logits.float().cpu(), "loss": float(loss), "grads": grads}


def main() -> None:
    import dabsn.kernels

    dabsn.kernels.enable("cuda", required=True)
    out, cases = sys.argv[1], sys.argv[2].split(",")
    result = {}
    for case in cases:
        H, T, B = (int(v) for v in case.split(":"))
        ids, tgt = (t.cuda() for t in batch(T, B))
        m = model(H).cuda()
        result[(case, "bf16")] = run(m, ids, tgt, True)
        result[(case, "fp32")] = run(m, ids, tgt, False)
        core = m.backbone.blocks[0].core
        result[(case, "route")] = str(getattr(core, "_last_core_backend", ""))
        del m
        torch.cuda.empty_cache()
    torch.save(result, out)


if __name__ == "__main__":
    main()
