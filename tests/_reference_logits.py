"""Child process of the state-drift test: the reference package's own eager
implementation (``dabsn.kernels.enable("reference")``, no hooks) computes
logits of the config-2 / config-3 models on the GPU in FP32 and FP64 and
saves them.  A separate process, because the backend family is chosen once
per process.

usage: python _reference_logits.py OUT.pt CFG:T[,CFG:T...]
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.append(str(Path(__file__).resolve().parents[1] / "baseline" / "_ref"))


def model(cfg: str):
    from dabsn import DABSNSequenceLM

    torch.manual_seed(0)
    if cfg == "c3":
        return DABSNSequenceLM(60, 256, 2, layers="seq:256:256,seq:256:256"), 60
    return DABSNSequenceLM(64, 128, 1, layers="seq:128:128"), 64


def tokens(V: int, T: int, batch: int = 2):
    g = torch.Generator().manual_seed(5)
    return torch.randint(0, V, (batch, T), generator=g)


def main() -> None:
    import dabsn.kernels

    dabsn.kernels.enable("reference")
    out, cases = sys.argv[1], sys.argv[2].split(",")
    result = {}
    for case in cases:
        cfg, T = case.split(":")
        for dtype in (torch.float32, torch.float64):
            m, V = model(cfg)
            m = m.to("cuda", dtype).eval()
            with torch.no_grad():
                logits = m.forward_sequence(tokens(V, int(T)).cuda())
            result[(case, str(dtype))] = logits.double().cpu()
    torch.save(result, out)


if __name__ == "__main__":
    main()
