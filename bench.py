#!/usr/bin/env python
"""Benchmark of the DABSN scan + read path, forward + backward, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c4|c5]
                    [--impl b200|reference|reference-cuda]

One step = one training step of the configured ``DABSNSequenceLM`` (forward,
cross-entropy, backward through the scan + read path, AdamW update) on one
seeded synthetic batch per GPU.  The default workload is config 5 (width 2048,
T = 4096, global batch 32 sharded over the GPUs, BF16 autocast): the
"scan+read throughput sweep at 1/2/4/8 GPUs" the metric is quoted on.

``--impl b200`` (default) runs the reference library's own model code with the
B200 backend enabled; ``--impl reference`` runs the reference's own CPU
implementation (its C++/OpenMP backend, ``enable("cpu")``) on the host cores,
on rank 0 only; ``--impl reference-cuda`` runs the reference's own CUDA
family (``enable("cuda")``: its Triton/ATen path) on the same GPU with the same
timing, and the b200 arm reports it as ``reference_cuda`` at N = 1.

Rank 0 prints ONE JSON line.  Multi-GPU runs are launched with torchrun (one
process per GPU, NCCL, data parallel with per-GPU batch fixed: weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REF = ROOT / "baseline" / "_ref"
for p in (str(ROOT),):
    if p not in sys.path:
        sys.path.insert(0, p)
if REF.is_dir() and str(REF) not in sys.path:
    sys.path.append(str(REF))


def _reference_import_error() -> str | None:
    """None when the reference package imports, else a one-line reason."""
    try:
        import dabsn  # noqa: F401
        import dabsn.kernels  # noqa: F401
    except Exception as exc:  # noqa: BLE001
        return (f"reference package not importable from {REF} ({type(exc).__name__}: {exc}); "
                "__graft_entry__.build() installs it there")
    return None
os.environ.setdefault("DABSN_SILENCE_ROUTING", "1")

# BASELINE configs run as bench workloads.  c5 is the default.
CONFIGS = {
    "c2": dict(
        workload="config2: DABSNSequenceLM vocab 64, width 128, 1 seq block, fp32, batch 32/GPU, "
        "T=64, fwd+bwd+AdamW",
        vocab=64, hidden=128, depth=1, layers="seq:128:128", batch=32, T=64, autocast=False,
    ),
    "c3": dict(
        workload="config3: DABSNSequenceLM vocab 60, width 256, 2 seq blocks, fp32, batch 64/GPU, "
        "T=256, fwd+bwd+AdamW",
        vocab=60, hidden=256, depth=2, layers="seq:256:256,seq:256:256", batch=64, T=256,
        autocast=False,
    ),
    "c4": dict(
        workload="config4: DABSNSequenceLM vocab 32000, width 1024, 2 seq blocks, residual, "
        "mlp_ratio 4, mlp_middle_depth 20, bf16 autocast, batch 16/GPU, T=2048, Zipf(1.1) "
        "tokens, fwd+bwd+AdamW",
        vocab=32000, hidden=1024, depth=2, layers="seq:1024:1024,seq:1024:1024", batch=16,
        T=2048, autocast=True, zipf=1.1,
        model_kw=dict(residual=True, mlp_ratio=4.0, mlp_middle_depth=20, mlp_depth_index=0),
    ),
    "c5": dict(
        workload="config5: DABSNSequenceLM vocab 32000, width 2048, 1 seq block, bf16 autocast, "
        "global batch 32 (batch-sharded), T=4096, Zipf(1.1) tokens, fwd+bwd+AdamW",
        vocab=32000, hidden=2048, depth=1, layers="seq:2048:2048", batch=32, T=4096,
        autocast=True, zipf=1.1, global_batch=True,
    ),
}


def _tokens(cfg, shape, g):
    """Seeded synthetic token ids: uniform, or Zipf(s) over the vocabulary
    (p(k) ~ k^-s for k = 1..V, id = k - 1)."""
    import torch

    V = cfg["vocab"]
    if cfg.get("zipf"):
        p = torch.arange(1, V + 1, dtype=torch.float64).pow(-cfg["zipf"])
        flat = torch.multinomial(p / p.sum(), shape[0] * shape[1], replacement=True, generator=g)
        return flat.reshape(shape)
    return torch.randint(0, V, shape, generator=g)


def _token_kind(cfg):
    return f"Zipf({cfg['zipf']})" if cfg.get("zipf") else "uniform"


def _batch(cfg, world):
    """Per-GPU batch: fixed per GPU, or the global batch split over ranks."""
    if cfg.get("global_batch"):
        return max(1, cfg["batch"] // world)
    return cfg["batch"]
METRIC = "DABSN scan+read tokens/sec fwd+bwd"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def _env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(
        os.environ.get("LOCAL_RANK", "0"))


def _peaks():
    """(HBM GB/s, BF16 TFLOP/s sustained, which): the driver-measured peaks of
    this pool's B200s, else the earlier measurement the profiling recipe
    gives."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return (float(data["hbm_gbs"]), float(data.get("bf16_tflops_sustained",
                                                       data["bf16_tflops"])), "measured")
    return 6650.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------
# algorithmic work per launch, by kernel; B,T,H,N of one block, D its input
# width, V the vocabulary, s activation bytes
# ---------------------------------------------------------------------------
def algorithmic_bytes(kernel: str, B: int, T: int, H: int, N: int, s: int, V: int = 0) -> float:
    """Bytes a launch must move at minimum (each input read once, each output
    written once)."""
    BT = B * T
    if kernel == "core_scan_fwd":
        return BT * H * (2 * s + 9 * s) + 2 * H * H * s
    if kernel == "core_scan_bwd":
        return BT * H * (7 * s + 8 * 4 + 3 * s) + 2 * H * H * s
    if kernel == "read_fwd":
        return BT * H * (s + s + 3 * 4) + 3 * B * N * H * s + BT * 3 * 4
    if kernel == "read_bwd":
        return BT * H * (2 * s + 4 + 3 * 4) + B * N * H * (3 * s + 3 * s) + BT * 8 * 4
    if kernel == "long_fwd":
        return BT * H * (2 * s + 4)
    if kernel == "long_bwd":
        return BT * H * (2 * s + 4 + 2 * s)
    if kernel == "admission_fwd":  # five tapes in; query (read dtype) and token stats out
        return BT * H * (5 * s + s) + BT * 14 * 4
    if kernel == "bank_gather":  # write rows (entry + next) in; writes, next writes, keys out
        return B * N * H * (2 * s + 3 * s)
    if kernel == "admission_bwd":  # expression, write, d query in; bank grads in; 2 grads out
        return BT * H * (2 * s + s + 2 * s) + B * N * H * 3 * s
    if kernel == "read_out_glue":  # FP32 gradient and long channel in; BF16 copy, FP32 dlong out
        return BT * H * (4 + 4 + 2 + 4)
    if kernel == "ce_logits_fwd":  # logits read once
        return BT * V * s
    if kernel == "ce_logits_bwd":  # logits read, gradient written
        return 2 * BT * V * s
    return 0.0


def algorithmic_flops(kernel: str, B: int, T: int, H: int, N: int, D: int) -> float:
    """Multiply-add work (2 FLOPs each) of the tensor-core kernels.  The read
    counts the causal half of its score and value products (bank width N ~ T
    at these configs): forward 3 B T N H (one score product, two value
    products), reverse twice that."""
    BT = B * T
    if kernel == "input_proj_fwd":
        return 4.0 * BT * D * H
    if kernel == "input_proj_bwd":
        return 8.0 * BT * D * H
    if kernel == "rec_grad":
        return 4.0 * BT * H * H
    if kernel == "read_out_fwd":
        return 6.0 * BT * H * H
    if kernel == "read_out_bwd":
        return 12.0 * BT * H * H
    if kernel == "read_fwd" and H > 256:
        return 3.0 * BT * N * H
    if kernel == "read_bwd" and H > 256:
        return 6.0 * BT * N * H
    return 0.0


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 6]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" == r[3 + i].strip()})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": float(rows[0][2]) if rows[0][2].strip().replace(".", "").isdigit() else None,
            "reasons": reasons,
            "samples": len(rows),
        }


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------
def run_b200(args, cfg, family: str = "b200"):
    """Time the training step on the GPU(s).  ``family`` "b200" enables this
    library's backend; "reference_cuda" enables the reference's own CUDA
    family instead (same model, step, inputs and timing; N = 1)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    rank, world, local = _env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    from dabsn import DABSNSequenceLM
    from dabsn_b200 import ops

    if family == "b200":
        import dabsn_b200

        dabsn_b200.install()
    import dabsn.kernels

    dabsn.kernels.enable("cuda", required=True)

    torch.manual_seed(0)
    model = DABSNSequenceLM(cfg["vocab"], cfg["hidden"], cfg["depth"], layers=cfg["layers"],
                            **cfg.get("model_kw", {})).to(dev)
    V, B, T = cfg["vocab"], (cfg["batch"] if args.tp else _batch(cfg, world)), cfg["T"]

    class LM(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.m = m

        def forward(self, ids):
            return self.m.forward_sequence(ids)

    # make_graphed_callables replaces the forward of the module it records, so
    # the eager reference for counting/timing kernels calls the model directly.
    def eager_net(x):
        return model.forward_sequence(x)

    graph_net = LM(model)
    g = torch.Generator().manual_seed(1000 + (0 if args.tp else rank))  # TP: one replicated batch
    ids_host = _tokens(cfg, (B, T), g).pin_memory()
    tgt_host = _tokens(cfg, (B, T), g).pin_memory()
    ids = ids_host.to(dev)
    tgt = tgt_host.to(dev)
    net = graph_net
    if args.graph:
        # The reference's own CUDA-graph training API (runtime/graph.py:292):
        # forward and backward of the module are recorded once and replayed.
        from dabsn.runtime.graph import make_graphed_train_callable

        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=cfg["autocast"]):
            net = make_graphed_train_callable(graph_net, (ids,), warmup_iters=3, verify=False)
    if args.tp and world > 1:
        # Tensor parallel over the state units (the reference's provider does
        # the same swap, providers.py:208): every block's core becomes this
        # rank's TensorParallelDABSNCore; the batch is replicated.
        from dabsn.core import TensorParallelDABSNCore

        for block in model.backbone.blocks:
            block.core = TensorParallelDABSNCore(block.core, group=dist.group.WORLD, rank=rank,
                                                 world_size=world).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.1, fused=True)
    # Data parallel: gradients in one flat FP32 buffer, averaged by NCCL
    # all-reduces of 64 MiB buckets launched from the backward as each bucket's
    # gradients become final, so the exchange overlaps the rest of the
    # backward (dabsn_b200.data_parallel); the sub-millisecond small-width
    # configs keep one all-reduce after the backward.
    dp = None
    if world > 1 and not args.tp:
        from dabsn_b200.data_parallel import FlatGradAllReduce

        mib = int(os.environ.get("DABSN_B200_DP_BUCKET_MB", "64"))  # 0: one all-reduce
        dp = FlatGradAllReduce(model.parameters(), dev,
                               bucket_bytes=(mib << 20) if (mib > 0 and cfg["hidden"] >= 1024)
                               else None)
    current = {"net": net}
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    import dabsn.runtime as dabsn_runtime

    def loss_of(net, x, y):
        """Mean next-token cross-entropy through the reference's own loss API:
        ``chunked_cross_entropy_from_logits`` on the model's logits (the
        default loss of ``runtime.api.train_step``, runtime/api.py:22-31), or, with
        ``chunked_loss`` in the config, the reference's readout + chunked
        cross-entropy API on the hidden states (runtime/loss.py:138; the B200
        family binds its fused kernels there)."""
        if cfg.get("chunked_loss"):
            hidden = model.forward_hidden(x)
            return dabsn_runtime.chunked_linear_cross_entropy(
                hidden, model.readout.weight, model.readout.bias, y)
        logits = net(x)
        return dabsn_runtime.chunked_cross_entropy_from_logits(logits, y)

    def zero_grads():
        if dp is None:
            opt.zero_grad(set_to_none=True)
        else:
            dp.zero()

    def step(x, y):
        zero_grads()
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=cfg["autocast"]):
            loss = loss_of(current["net"], x, y)
        loss.backward()
        if dp is not None:
            dp.all_reduce()
        opt.step()
        return loss

    for _ in range(args.warmup):
        step(ids, tgt)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def timed_loop(e2e: bool, kernel_events: bool):
        evs = []
        ops.KERNEL_EVENTS = {} if kernel_events else None
        launches0 = ops.LAUNCH_COUNT["n"]
        barrier()
        torch.cuda.synchronize()
        t_wall = time.perf_counter()
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            if e2e:
                ids.copy_(ids_host, non_blocking=True)
                tgt.copy_(tgt_host, non_blocking=True)
                loss = step(ids, tgt)
                loss_host.copy_(loss.detach(), non_blocking=True)
                e1.record()
                e1.synchronize()
                float(loss_host)
            else:
                step(ids, tgt)
                e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        barrier()
        wall = time.perf_counter() - t_wall
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        kev = ops.KERNEL_EVENTS
        ops.KERNEL_EVENTS = None
        launches = ops.LAUNCH_COUNT["n"] - launches0
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
        return ms, kev, launches, wall

    if args.profile_steps:
        # Launch-list mode for a profiler: N steps, each preceded by the L2
        # flush (whose fill kernel marks the step boundary), then exit.
        for _ in range(args.profile_steps):
            flush.zero_()
            step(ids, tgt)
        torch.cuda.synchronize()
        return None

    # Launches of this library's kernels per step, counted on one eager step
    # (graph replays launch the same kernels without passing through Python).
    n0 = ops.LAUNCH_COUNT["n"]
    zero_grads()
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=cfg["autocast"]):
        loss_of(eager_net, ids, tgt).backward()
    launches_per_step = ops.LAUNCH_COUNT["n"] - n0
    zero_grads()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    ms, _, _, wall = timed_loop(e2e=False, kernel_events=False)
    clocks = sampler.stop()
    ms_e2e, _, _, _ = timed_loop(e2e=True, kernel_events=False)
    launches = launches_per_step * args.steps
    # Per-kernel durations: the same step run eagerly (identical kernels and
    # shapes), each launch bracketed by CUDA events on its stream.
    kev = None
    if family == "b200":
        current["net"] = eager_net
        _, kev, _, _ = timed_loop(e2e=False, kernel_events=True)
        current["net"] = net

    tokens = B * T * (1 if args.tp else world)
    value = tokens / (ms / 1e3)
    e2e_value = tokens / (ms_e2e / 1e3)

    # dominant kernel and its roofline
    per_kernel = {}
    for name, pairs in (kev or {}).items():
        times = [a.elapsed_time(b) for a, b in pairs]
        per_kernel[name] = {"launches": len(times), "total_ms": sum(times),
                            "mean_us": 1e3 * sum(times) / len(times)}
    roofline = None
    rooflines = {}
    if per_kernel:
        H = cfg["hidden"]
        N = model.backbone.blocks[0].read.last_n_max or T
        D = H
        s = 2 if cfg["autocast"] else 4
        hbm, tflops, peak_kind = _peaks()
        for name, k in per_kernel.items():
            mean_s = k["mean_us"] * 1e-6
            fl = algorithmic_flops(name, B, T, H, N, D)
            if fl > 0:
                ach = fl / mean_s / 1e12
                rooflines[name] = {"bound": "tensor", "achieved": round(ach, 1), "peak": tflops,
                                   "unit": "TFLOP/s", "frac": round(ach / tflops, 4),
                                   "flops_per_launch": fl}
                continue
            by = algorithmic_bytes(name, B, T, H, N, s, cfg["vocab"])
            if by > 0:
                ach = by / mean_s / 1e9
                rooflines[name] = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm,
                                   "unit": "GB/s", "frac": round(ach / hbm, 4),
                                   "bytes_per_launch": by}
                if name.startswith("core_scan") or name.startswith("long"):
                    # T sequential steps: at small per-GPU batch neither roofline
                    # binds and the per-step latency does (the latency floor)
                    rooflines[name]["latency"] = {
                        "sequential_steps": T, "us_per_step": round(k["mean_us"] / T, 3),
                        "hbm_time_us_per_step": round(by / (hbm * 1e3) / T, 4)}
        top = max(per_kernel, key=lambda k: per_kernel[k]["total_ms"])
        if top in rooflines:
            r = rooflines[top]
            traffic = None
            tf = ROOT / "profiles" / f"traffic_{args.config}.json"
            if tf.exists():
                traffic = json.loads(tf.read_text()).get(top)
            roofline = {"kernel": top, "bound": r["bound"], "achieved": r["achieved"],
                        "peak": r["peak"], "peak_kind": peak_kind + " " + (
                            "hbm_gbs" if r["bound"] == "hbm" else "bf16_tflops_sustained"),
                        "unit": r["unit"], "frac": r["frac"], "traffic": traffic}
            for key in ("bytes_per_launch", "flops_per_launch", "latency"):
                if key in r:
                    roofline[key] = r[key]
            roofline["step_share"] = round(per_kernel[top]["mean_us"] / 1e3 / ms, 4)

    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong" if (args.tp or cfg.get("global_batch")) else "weak",
        "vs_baseline": None,
        "dtype": "bf16" if cfg["autocast"] else "f32",
        "data": f"synthetic: seeded {_token_kind(cfg)} tokens (per-rank seed 1000+rank), "
                "random-init weights",
        "config": {"workload": cfg["workload"], "global_batch": B * (1 if args.tp else world),
                   "seq_len": T, "parallelism": f"tp{world}" if args.tp else f"dp{world}",
                   "sequences_per_gpu": B,
                   "grad_all_reduce": ("tensor parallel: the module's own reductions"
                                       if args.tp else "none (one GPU)" if dp is None else
                                       f"{len(dp.buckets)} buckets overlapping the backward"
                                       if dp.overlap else "one after the backward"),
                   "l2": "flushed (256 MiB write) before every timed step",
                   "n_max": model.backbone.blocks[0].read.last_n_max},
        "impl": "b200" if family == "b200" else "reference-cuda",
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": ids_host.numel() * 8 * 2, "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "graph": bool(args.graph),
        "kernels": {k: {kk: round(vv, 3) if isinstance(vv, float) else vv for kk, vv in v.items()}
                    for k, v in per_kernel.items()},
        "library_ms_per_step": round(sum(v["total_ms"] for v in per_kernel.values()) / args.steps, 3),
        "roofline": roofline,
        "rooflines": rooflines,
        "clocks": clocks,
        "wall_s_timed": round(wall, 3),
    }
    if family == "b200" and rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args)
    if family == "b200" and rank == 0 and world == 1 and args.reference_cuda_result is not None:
        result["reference_cuda"] = args.reference_cuda_result
    if world > 1:
        dist.destroy_process_group()
    return result if rank == 0 else None


def _child_bench(args, impl: str, steps: int, warmup: int, timeout: int):
    """Run one ``bench.py --impl <impl>`` arm in a fresh process (the
    reference's backend family is process-wide) and return its JSON line."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", impl, "--config", args.config,
           "--steps", str(steps), "--warmup", str(warmup)]
    if args.batch is not None:
        cmd += ["--batch", str(args.batch)]
    if args.seq_len is not None:
        cmd += ["--seq-len", str(args.seq_len)]
    if not args.graph:
        cmd.append("--no-graph")
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    if not lines:
        raise RuntimeError(f"rc={res.returncode}: {res.stderr.strip().splitlines()[-1:]}")
    return json.loads(lines[-1])


def cpu_baseline(args):
    try:
        return _child_bench(args, "reference", args.cpu_steps, 1, 900)["cpu_baseline"]
    except Exception as exc:  # noqa: BLE001
        return {"value": None, "error": f"{type(exc).__name__}: {exc}"}


def reference_cuda(args):
    """The reference's own CUDA family on this GPU, same config and timing."""
    try:
        data = _child_bench(args, "reference-cuda", args.ref_cuda_steps, 3, 1200)
    except Exception as exc:  # noqa: BLE001
        return {"value": None, "error": f"{type(exc).__name__}: {exc}"}
    if "value" not in data:
        return {"value": None, "error": data.get("error", "no value")}
    return {k: data.get(k) for k in ("value", "unit", "ms_per_step", "steps", "warmup", "e2e",
                                     "clocks", "impl")} | {
        "path": "dabsn.kernels.enable('cuda', required=True): the reference's Triton/ATen family"}


# ---------------------------------------------------------------------------
# the reference arm: the reference's own CPU implementation on host cores
# ---------------------------------------------------------------------------
def run_reference(args, cfg):
    rank, world, _ = _env_rank()
    if rank != 0:
        return None
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", str(ROOT / "oracle" / "_ref" / "torch_extensions"))
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    import torch
    import torch.nn.functional as F

    torch.set_num_threads(cores)
    import dabsn.kernels
    import dabsn.runtime as dabsn_runtime
    from dabsn import DABSNSequenceLM

    dabsn.kernels.enable("cpu", required=True)
    torch.manual_seed(0)
    model = DABSNSequenceLM(cfg["vocab"], cfg["hidden"], cfg["depth"], layers=cfg["layers"],
                            **cfg.get("model_kw", {}))
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.1)
    V, B, T = cfg["vocab"], _batch(cfg, world), cfg["T"]
    # bounded sample: the full per-GPU batch when a step is short, else fewer
    # sequences (same model) so the run stays within minutes.  At widths 1024
    # and 2048 one full-length sequence takes the reference's CPU path many
    # minutes per step (its reverse scan is a Python loop over T steps), so the
    # sample is one sequence of the first args.cpu_seq_len tokens; the read's
    # per-token cost grows with T, so this favours the CPU figure.
    sample_t = T
    if cfg["hidden"] <= 128:
        sample_b = B
    elif cfg["hidden"] < 1024:
        sample_b = max(1, B // 8)
    else:
        sample_b = 1
        sample_t = min(T, args.cpu_seq_len)
    g = torch.Generator().manual_seed(1000)
    ids = _tokens(cfg, (sample_b, sample_t), g)
    tgt = _tokens(cfg, (sample_b, sample_t), g)

    def step():
        opt.zero_grad(set_to_none=True)
        logits = model.forward_sequence(ids)
        loss = dabsn_runtime.chunked_cross_entropy_from_logits(logits, tgt)
        loss.backward()
        opt.step()
        return float(loss)

    # One warm-up step (it also loads the extension), then up to K timed
    # steps, stopping once the sample has used its time budget so a
    # --steps K --warmup W run stays within minutes at every config.
    step()
    times = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > args.cpu_budget_s:
            break
    dt = sum(times) / len(times)
    value = sample_b * sample_t / dt
    model_name = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model_name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    sample = (f"{sample_b} x {sample_t} tokens per step (of the {B} x {T} per-GPU batch), "
              f"{len(times)} timed steps (of {args.steps} asked, {args.cpu_budget_s:.0f} s budget) "
              f"after 1 warm-up; {cores} threads; CPU: {model_name}")
    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": len(times),
        "warmup": 1,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong" if cfg.get("global_batch") else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": f"synthetic: seeded {_token_kind(cfg)} tokens, random-init weights",
        "config": {"workload": cfg["workload"], "global_batch": B * world, "seq_len": T,
                   "parallelism": f"dp{world}"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-cuda"])
    ap.add_argument("--cpu-steps", type=int, default=None,
                    help="timed steps of the CPU-baseline sample (default: ~10-30 s of work)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seq-len", type=int, default=256,
                    help="sequence length of the CPU reference sample at widths >= 1024")
    ap.add_argument("--cpu-budget-s", type=float, default=60.0,
                    help="time budget of the CPU reference sample's timed steps")
    ap.add_argument("--no-reference-cuda", action="store_true",
                    help="skip timing the reference's own CUDA family beside the b200 arm")
    ap.add_argument("--ref-cuda-steps", type=int, default=None,
                    help="timed steps of the reference CUDA leg (default: 3 at c4/c5, 20 else)")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="run N steps after warm-up and exit (for a profiler launch list)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="run the step eagerly instead of through the reference's CUDA-graph API")
    ap.add_argument("--tp", action="store_true",
                    help="tensor parallel over the state units (batch replicated) instead of data "
                         "parallel; BF16 configs")
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch override (small profiler cases); recorded in config")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="sequence length override (small profiler cases); recorded in config")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch is not None or args.seq_len is not None:
        cfg["batch"] = args.batch or cfg["batch"]
        cfg["T"] = args.seq_len or cfg["T"]
        cfg["global_batch"] = False
        cfg["workload"] += f" [override: batch {cfg['batch']}/GPU, T={cfg['T']}]"
    if args.cpu_steps is None:
        args.cpu_steps = {"c2": 100, "c3": 20}.get(args.config, 2)
    if cfg["autocast"]:
        # The reference's graph API (runtime/graph.py) refuses autocast's
        # weight cache, so the BF16 configs run the step eagerly.
        args.graph = False
    if args.ref_cuda_steps is None:
        args.ref_cuda_steps = 3 if args.config in ("c4", "c5") else 20
    err = _reference_import_error()
    if err is not None:
        # The model, the step and both backends' registration points live in
        # the reference package: without it no arm can run.
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": err}), flush=True)
            return
        print(json.dumps({"metric": METRIC, "impl": args.impl, "error": err}), flush=True)
        sys.exit(1)
    args.reference_cuda_result = None
    if (args.impl == "b200" and not args.no_reference_cuda
            and int(os.environ.get("WORLD_SIZE", "1")) == 1):
        # before this process touches the GPU: at config 5 the reference's
        # step needs most of the device's memory
        args.reference_cuda_result = reference_cuda(args)
    if args.impl == "reference":
        result = run_reference(args, cfg)
    else:
        result = run_b200(args, cfg, "b200" if args.impl == "b200" else "reference_cuda")
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
