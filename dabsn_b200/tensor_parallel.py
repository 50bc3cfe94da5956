"""Tensor parallelism over state units for the core scan (BF16).

Drop-in for ``TensorParallelDABSNCore.forward_from_state``
(src/dabsn/core.py:609-874).  The reference runs a Python loop over steps,
each with an NCCL all-gather of the recurrent input and a GEMM
(``_GatherHiddenRecurrent``, core.py:525-600), and backpropagates through the
per-step graph.  Here the whole scan is one cooperative launch per GPU
(``dabsn_core_scan_tp_fwd`` / ``_bwd``): each GPU runs the grid-wide scan on
its units, and every step its CTAs store their slice of the recurrent vector
into every GPU's exchange buffer over NVLink (peer pointers, CUDA IPC) and
meet at a bounded cross-GPU barrier.  The module's contract is kept: local
weights and parameters (the reference's slicing), public tapes gathered once
after the scan with the reference's own ``_gather_fields``, input gradients
summed by ``_SumReplicatedInputGradient``, scalar-parameter gradients summed
by the hooks the reference module registers.
"""

from __future__ import annotations

import ctypes
import threading

import torch
import torch.distributed as dist
from torch import Tensor

from . import _native as N
from . import ops

_LOCK = threading.Lock()


class TPExchange:
    """The exchange buffers of one process group on this GPU: this rank's
    (allocated by the library, shared through a CUDA IPC handle) and every
    peer's (opened from their handles), plus the running barrier count that
    every rank advances identically with each scan launch."""

    _cache: dict[tuple, "TPExchange"] = {}

    @classmethod
    def get(cls, group, H: int, device: torch.device) -> "TPExchange":
        key = (id(group), int(H), device.index)
        with _LOCK:
            ex = cls._cache.get(key)
            if ex is None:
                ex = cls(group, H, device)
                cls._cache[key] = ex
            return ex

    def __init__(self, group, H: int, device: torch.device):
        lib = N.load()
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.P > 8:
            raise RuntimeError("dabsn_b200 tensor parallel scan supports up to 8 GPUs")
        with torch.cuda.device(device):
            nbytes = int(lib.dabsn_tp_buffer_bytes(H))
            own = ctypes.c_void_p()
            N.check(lib.dabsn_tp_alloc(nbytes, ctypes.byref(own)), "tp_alloc")
            handle = (ctypes.c_char * 64)()
            N.check(lib.dabsn_tp_ipc_handle(own, handle), "tp_ipc_handle")
            handles: list = [None] * self.P
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(own.value)
                    continue
                peer = ctypes.c_void_p()
                raw = (ctypes.c_char * 64).from_buffer_copy(h)
                N.check(lib.dabsn_tp_ipc_open(raw, ctypes.byref(peer)), "tp_ipc_open")
                ptrs.append(peer.value)
        self.bufs = (ctypes.c_void_p * self.P)(*ptrs)
        self.base = 0
        dist.barrier(group=group)  # every buffer opened before any scan writes to it

    def advance(self, next_base: ctypes.c_uint32) -> None:
        self.base = int(next_base.value)


def _chunks(B: int):
    for b0 in range(0, B, ops.WIDE_MAX_B):
        yield b0, min(B, b0 + ops.WIDE_MAX_B)


def tp_scan_forward(ex: TPExchange, H: int, ubase: int, Wx: Tensor, Wgx: Tensor, Ug: Tensor,
                    A: Tensor, params: list[Tensor], init_b: Tensor, init_e: Tensor,
                    init_c: Tensor):
    """Local outputs ``(U [B,T,2Hl], novelty, plasticity, expression, write,
    energy, saturation, gate, final_b, final_e, final_c)`` for this rank's
    units; ``Ug``/``A`` are this rank's rows."""
    dev = ops._require_cuda(Wx)
    B, T, Hl = Wx.shape
    bf = torch.bfloat16
    Wx = Wx.detach().to(bf).contiguous()
    Wgx = Wgx.detach().to(bf).contiguous()
    rec = torch.cat((Ug.detach(), A.detach()), dim=0).to(bf).contiguous()
    pack = ops._ParamPack(list(params[:16]), list(params[16:19]), Hl)
    ib, ie, ic = (ops._f32(t, (B, Hl)) for t in (init_b, init_e, init_c))
    U = torch.empty((B, T, 2 * Hl), device=dev, dtype=bf)
    tapes = [torch.empty((B, T, Hl), device=dev, dtype=bf) for _ in range(7)]
    fins = [torch.empty((B, Hl), device=dev, dtype=bf) for _ in range(3)]
    lib = N.load()
    nxt = ctypes.c_uint32()
    with torch.cuda.device(dev), ops._timed("core_scan_tp_fwd", dev):
        for b0, b1 in _chunks(B):
            st = lib.dabsn_core_scan_tp_fwd(
                b1 - b0, T, H, Hl, ubase, ex.P, ex.rank, ex.bufs, ex.base, ctypes.byref(nxt),
                ops._ptr(Wx[b0:b1]), ops._ptr(Wgx[b0:b1]), ops._ptr(rec),
                ctypes.byref(pack.struct), ops._ptr(ib[b0:b1]), ops._ptr(ie[b0:b1]),
                ops._ptr(ic[b0:b1]), ops._ptr(U[b0:b1]), *[ops._ptr(t[b0:b1]) for t in tapes],
                *[ops._ptr(f[b0:b1]) for f in fins], ops._stream(dev),
            )
            N.check(st, "core_scan_tp_fwd")
            ex.advance(nxt)
    return (U, *tapes, *fins)


def _gather_hidden(x: Tensor, group, P: int) -> Tensor:
    """[..., Hl] on every rank -> [..., P*Hl], ranks' slices in rank order."""
    parts = [torch.empty_like(x) for _ in range(P)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=-1)


def _gather_rows(x: Tensor, group, P: int) -> Tensor:
    parts = [torch.empty_like(x) for _ in range(P)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=0)


class TPCoreScan(torch.autograd.Function):
    """Autograd of the tensor-parallel scan.  Inputs: local Wx, Wgx, Ug rows,
    A rows, the 19 parameters (local per-unit slices, replicated scalars),
    local initial b, e, c.  The reverse gathers the full [Ug; A] and the full
    y tape once, runs the cross-GPU reverse scan and forms this rank's rows of
    grad[Ug; A] with one GEMM."""

    @staticmethod
    def forward(ctx, ex, H, ubase, Wx, Wgx, Ug, A, *rest):
        params, (init_b, init_e, init_c) = list(rest[:19]), rest[19:22]
        outs = tp_scan_forward(ex, H, ubase, Wx, Wgx, Ug, A, params, init_b, init_e, init_c)
        U, nov, plast, expr, write, energy, sat, gate, fb, fe, fc = outs
        ctx.ex, ctx.H, ctx.ubase = ex, H, ubase
        ctx.save_for_backward(Wx, Wgx, Ug, A, *params, init_b, init_e, init_c, U, energy, sat,
                              gate, plast, expr)
        ctx.mark_non_differentiable(gate)
        return outs

    @staticmethod
    def backward(ctx, *grads):
        saved = ctx.saved_tensors
        Wx, Wgx, Ug, A = saved[:4]
        params = list(saved[4:23])
        init_b, init_e, init_c = saved[23:26]
        U, e_tape, c_tape, s_tape, plast, expr = saved[26:32]
        ex, H, ubase = ctx.ex, ctx.H, ctx.ubase
        dev = U.device
        B, T, Hl = plast.shape
        bf = torch.bfloat16
        rec_full = torch.cat((_gather_rows(Ug.detach().to(bf), ex.group, ex.P),
                              _gather_rows(A.detach().to(bf), ex.group, ex.P)), dim=0).contiguous()
        pack = ops._ParamPack(params[:16], params[16:19], Hl)
        ib = ops._f32(init_b, (B, Hl))
        ic = ops._f32(init_c, (B, Hl))
        g = [ops._grad_or_none(x) for x in grads]
        gU, gnov, gp, gay, gw, ge, gc = g[:7]
        gfb, gfe, gfc = g[8:11]
        gWx = torch.empty((B, T, Hl), device=dev, dtype=bf)
        gWgx = torch.empty_like(gWx)
        day = torch.empty_like(gWx)
        g_init = torch.empty((3, B, Hl), device=dev, dtype=torch.float32)
        partial = torch.empty((B, 19, Hl), device=dev, dtype=torch.float32)
        lib = N.load()
        nxt = ctypes.c_uint32()
        tapes = [t.detach().contiguous() for t in (U, e_tape, c_tape, s_tape, plast, expr)]

        def sl(t, b0, b1):
            return None if t is None else ops._ptr(t[b0:b1])

        with torch.cuda.device(dev), ops._timed("core_scan_tp_bwd", dev):
            for b0, b1 in _chunks(B):
                st = lib.dabsn_core_scan_tp_bwd(
                    b1 - b0, T, H, Hl, ubase, ex.P, ex.rank, ex.bufs, ex.base, ctypes.byref(nxt),
                    *[sl(t, b0, b1) for t in tapes], ops._ptr(rec_full), ctypes.byref(pack.struct),
                    sl(ib, b0, b1), sl(ic, b0, b1), N.F32,
                    *[sl(x, b0, b1) for x in (gU, gnov, gp, gay, gw, ge, gc, gfb, gfe, gfc)],
                    sl(gWx, b0, b1), sl(gWgx, b0, b1), sl(day, b0, b1), sl(g_init[0], b0, b1),
                    sl(g_init[1], b0, b1), sl(g_init[2], b0, b1), sl(partial, b0, b1),
                    ops._stream(dev),
                )
                N.check(st, "core_scan_tp_bwd")
                ex.advance(nxt)
        # this rank's rows of grad[Ug; A] = [gWgx, day]^T . y over (b, t), y gathered
        y_full = _gather_hidden(U[:, :, :Hl].contiguous(), ex.group, ex.P).reshape(B * T, H)
        grad_rows = torch.cat((gWgx, day), dim=-1).reshape(B * T, 2 * Hl).T @ y_full.to(bf)
        grad_Ug, grad_A = grad_rows.float().split(Hl, dim=0)
        sums = partial.sum(dim=0)
        out = [None, None, None, gWx.to(Wx.dtype), gWgx.to(Wgx.dtype), grad_Ug.to(Ug.dtype),
               grad_A.to(A.dtype)]
        for j in range(16):
            out.append(sums[j].to(params[j].dtype).reshape(params[j].shape))
        for j in range(3):
            p = params[16 + j]
            out.append(sums[16 + j].sum().reshape(p.shape).to(p.dtype))
        for gi, ref in zip(g_init, (init_b, init_e, init_c)):
            out.append(gi.to(ref.dtype).reshape(ref.shape))
        return tuple(out)


def tp_supported(core, inputs: Tensor) -> bool:
    """The B200 tensor-parallel scan covers CUDA, BF16 compute (autocast or
    BF16 inputs), an even split of the state into at most 8 slices of a
    multiple of 8 units, and batch chunks of 32."""
    if not inputs.is_cuda or core.tensor_world_size < 2 or core.tensor_world_size > 8:
        return False
    bf16 = inputs.dtype == torch.bfloat16 or (torch.is_autocast_enabled("cuda")
                                              and torch.get_autocast_dtype("cuda") == torch.bfloat16)
    sizes = core.tensor_sizes
    return (bf16 and len(set(sizes)) == 1 and sizes[0] % 8 == 0
            and core.global_hidden_dim % 16 == 0)


def make_tp_forward(original):
    """``TensorParallelDABSNCore.forward_from_state`` running the B200
    cross-GPU scan; other cases (CPU, FP32, uneven splits) keep the
    reference's method."""

    def forward_from_state(self, inputs, *, initial_state=None, return_writes=False,
                           return_cocktail=False, return_final_state=False):
        if not tp_supported(self, inputs) or torch.compiler.is_compiling():
            if inputs.is_cuda and not torch.compiler.is_compiling():
                from .backend import warn_fallback

                warn_fallback("tensor_parallel_core", "tensor-parallel scan outside the B200 "
                              "kernel's cover (FP32, uneven split or more than 8 slices): the "
                              "reference's per-step loop runs", dtype=str(inputs.dtype),
                              world=int(self.tensor_world_size),
                              corrective_action="run under BF16 autocast with an even split")
            return original(self, inputs, initial_state=initial_state, return_writes=return_writes,
                            return_cocktail=return_cocktail,
                            return_final_state=return_final_state)
        from dabsn.core import _SumReplicatedInputGradient

        if inputs.dim() != 3:
            raise ValueError("DABSNCore inputs must have shape [B,T,input_dim]")
        world_inputs = _SumReplicatedInputGradient.apply(inputs, self.tensor_group)
        batch = world_inputs.shape[0]
        budget, energy, saturation = self._local_state(
            batch, device=world_inputs.device, dtype=torch.float32, initial_state=initial_state)
        projected = self.W(world_inputs)
        gate_projected = self.Wg(world_inputs)
        H = self.global_hidden_dim
        ubase = self.tensor_slice.start
        ex = TPExchange.get(self.tensor_group, H, world_inputs.device)
        params = [self.beta, self.log_kappa, self.logit_recover, self.k_s, self.k_y, self.k_b,
                  self.k_n, self.k_bias, self.r_s, self.r_y, self.r_b, self.r_n, self.r_bias,
                  self.logit_saturation_decay.expand(self.hidden_dim), self.k_saturation,
                  self.r_saturation, self.logit_alpha.reshape(()), self.log_lambda.reshape(()),
                  self.logit_saturation_suppress.reshape(())]
        with torch.autocast("cuda", enabled=False):
            outs = TPCoreScan.apply(ex, H, ubase, projected, gate_projected, self.Ug.weight,
                                    self.A.weight, *params, budget, energy, saturation)
        U, novelty, plasticity, expression, write, energy_tape, saturation_tape = outs[:7]
        fin_b, fin_e, fin_c = outs[8:11]
        Hl = self.hidden_dim
        local_fields = (U[..., :Hl], U[..., Hl:], novelty, plasticity, expression, write,
                        energy_tape, saturation_tape)
        y, budget_tape, novelty, plasticity, expression, write, energy_tape, saturation_tape = (
            self._gather_fields(local_fields))
        trajectory = torch.cat((y, budget_tape), dim=-1)
        if return_cocktail:
            result = (trajectory, novelty, plasticity, expression, write, energy_tape,
                      saturation_tape)
        elif return_writes:
            result = trajectory, novelty, plasticity, expression, write
        else:
            result = trajectory, novelty, plasticity
        self._last_core_backend = "tensor_parallel_b200"
        if return_final_state:
            final_state = self._gather_fields((fin_b, fin_e, fin_c))
            return result, final_state
        return result

    forward_from_state.__wrapped_reference__ = original
    return forward_from_state
