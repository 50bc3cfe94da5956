"""Autograd wiring of the B200 kernels.

* ``core_forward_kernel`` / ``core_backward`` are installed on the reference
  operator ``dabsn::core_scan_batched`` (its CUDA kernel and its autograd
  formula), keeping the reference's saved-context layout so CPU tensors still
  reach the reference's own reverse scan.
* ``ThreeWayRead`` replaces the CUDA admitted read
  (``dabsn.kernels.triton.cuda_compact_three_way_read``).
* ``LongScan`` replaces ``dabsn.kernels.long.fused_long_scan_from_state``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import ops


# ---------------------------------------------------------------------------
# Core scan (reference op schema: batched_runtime.py:1507-1566)
# ---------------------------------------------------------------------------
def core_forward_kernel(*inputs: Tensor) -> tuple[Tensor, ...]:
    """CUDA kernel for ``dabsn::core_scan_batched`` (26 inputs, 11 outputs)."""
    Wx, Wgx, Ug, A = inputs[:4]
    return ops.core_scan_forward(Wx, Wgx, Ug, A, list(inputs[4:23]), *inputs[23:26])


def make_core_backward(reference_backward):
    """Autograd formula: B200 reverse scan for CUDA, the reference's for CPU."""

    def core_backward(ctx, *grad_outputs):
        saved = ctx.saved_tensors
        if not saved[0].is_cuda or saved[0].dtype not in (torch.float32, torch.bfloat16):
            return reference_backward(ctx, *grad_outputs)
        return ops.core_scan_backward(saved, grad_outputs)

    return core_backward


# ---------------------------------------------------------------------------
# Three-way admitted read (compact_admitted.py:16-80 semantics)
# ---------------------------------------------------------------------------
class ThreeWayRead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, keys, writes, next_writes, cocktail, bank_cocktail, key_bias,
                admission, scale, short_gain, pad_gain, induct_gain, cocktail_gain, idx, valid,
                mode, total_steps, compute_dtype):
        cd = compute_dtype
        # key bias and admission keep their precision; the read converts them
        # (to the compute dtype for the narrow read, FP32 for the wide one).
        tensors = [
            t.detach().to(cd).contiguous()
            for t in (query, keys, writes, next_writes, cocktail, bank_cocktail)
        ] + [t.detach().contiguous() for t in (key_bias, admission)]
        scale32 = scale.detach().float().reshape(1).contiguous()
        gains = torch.cat(
            [g.detach().float().reshape(1) for g in (short_gain, pad_gain, induct_gain, cocktail_gain)]
        ).contiguous()
        idx = idx.contiguous()
        valid = valid.to(torch.bool).contiguous()
        out, streams, lse = ops.read_forward(*tensors, scale32, idx, valid, gains, mode, total_steps)
        ctx.save_for_backward(*tensors, scale32, gains, idx, valid, streams, lse)
        ctx.mode = mode
        ctx.total_steps = total_steps
        ctx.in_dtypes = [t.dtype for t in (query, keys, writes, next_writes, cocktail, bank_cocktail,
                                           key_bias, admission)]
        ctx.scale_meta = (scale.dtype, scale.shape)
        ctx.gain_meta = [(g.dtype, g.shape) for g in (short_gain, pad_gain, induct_gain, cocktail_gain)]
        return out.to(query.dtype)

    @staticmethod
    def backward(ctx, gout):
        q, k, w, nw, c, bc, kb, adm, scale32, gains, idx, valid, streams, lse = ctx.saved_tensors
        dq, dcq, dk, dv, dn, db, dck, dscale, dgains = ops.read_backward(
            q, k, w, nw, c, bc, kb, adm, scale32, idx, valid, gains, ctx.mode, ctx.total_steps,
            streams, lse, gout,
        )
        dt = ctx.in_dtypes
        grads = [
            dq.to(dt[0]), dk.to(dt[1]), dv.to(dt[2]), dn.to(dt[3]), dcq.to(dt[4]), dck.to(dt[5]),
            db.to(dt[6]), db.to(dt[7]),
        ]
        s_dt, s_shape = ctx.scale_meta
        grads.append(dscale.reshape(s_shape).to(s_dt))
        for i, (g_dt, g_shape) in enumerate(ctx.gain_meta):
            grads.append(dgains[i].reshape(g_shape).to(g_dt))
        return (*grads, None, None, None, None, None)


def _compute_dtype(query: Tensor) -> torch.dtype:
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return query.dtype


def three_way_read(read, query, bank_keys, bank_writes, next_writes, cocktail, bank_cocktail,
                   bank_key_bias, bank_admission, scale, bank_idx, bank_valid, *, mode: str):
    """Drop-in for ``cuda_compact_three_way_read`` (triton.py:314-483)."""
    if not query.is_cuda:
        raise TypeError("compact CUDA admitted read requires CUDA tensors")
    if mode not in {"seq", "field"}:
        raise ValueError("compact CUDA admitted-read mode must be seq or field")
    cd = _compute_dtype(query)
    with torch.autocast("cuda", enabled=False):
        out = ThreeWayRead.apply(
            query, bank_keys, bank_writes, next_writes, cocktail, bank_cocktail, bank_key_bias,
            bank_admission, scale, read.short_gain, read.pad_gain, read.induct_gain,
            read.cocktail_gain, bank_idx, bank_valid, 0 if mode == "seq" else 1,
            int(query.shape[1]), cd,
        )
    if not torch.compiler.is_compiling():
        read._last_three_way_backend = (
            "b200_flash_exact" if query.shape[-1] <= ops.NARROW_READ_MAX_H else "b200_tensor_core"
        )
    return out


# ---------------------------------------------------------------------------
# Long-memory channel (long.py:492-579 semantics)
# ---------------------------------------------------------------------------
class LongScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, write, plasticity, l_retain, l_expect, l_decay, l_strength, init, want_final):
        logits = torch.cat(
            [x.detach().float().reshape(1) for x in (l_retain, l_expect, l_decay, l_strength)]
        ).contiguous()
        init32 = None if init is None else init.detach().float().contiguous()
        out, ckpt, fin = ops.long_forward(
            write, plasticity, logits, init32, save_checkpoints=True, want_final=bool(want_final)
        )
        ctx.save_for_backward(write, plasticity.to(write.dtype), logits, ckpt)
        ctx.has_init = init is not None
        ctx.init_dtype = None if init is None else init.dtype
        ctx.p_dtype = plasticity.dtype
        ctx.logit_meta = [(x.dtype, x.shape) for x in (l_retain, l_expect, l_decay, l_strength)]
        if fin is None:
            fin = out.new_zeros((3,) + tuple(out.shape[::2]))
        ctx.set_materialize_grads(False)
        return out, fin

    @staticmethod
    def backward(ctx, gout, gfin):
        write, plast, logits, ckpt = ctx.saved_tensors
        dw, dp, dlog, ginit = ops.long_backward(
            write, plast, logits, ckpt, gout, gfin, want_ginit=ctx.has_init
        )
        grads = [dw, dp.to(ctx.p_dtype)]
        for i, (dt, shape) in enumerate(ctx.logit_meta):
            grads.append(dlog[i].reshape(shape).to(dt))
        grads.append(None if ginit is None else ginit.to(ctx.init_dtype))
        grads.append(None)
        return tuple(grads)


_REFERENCE_LONG = None  # the reference's fused_long_scan_from_state, for CPU tensors


def long_scan_from_state(read, write, plasticity, novelty, *, initial_state=None,
                         return_final_state=False):
    """Drop-in for ``fused_long_scan_from_state`` (long.py:492-579).

    CPU tensors keep the reference's own implementation (its C++/OpenMP or
    eager path); CUDA tensors run the fused B200 kernel."""
    if not write.is_cuda:
        if _REFERENCE_LONG is None:
            raise TypeError("dabsn_b200 long-memory channel requires CUDA tensors")
        return _REFERENCE_LONG(read, write, plasticity, novelty, initial_state=initial_state,
                               return_final_state=return_final_state)
    del novelty
    B, T, H = write.shape
    init = None
    if initial_state is not None:
        states = [s.to(device=write.device) for s in initial_state]
        if any(s.shape != (B, H) for s in states):
            raise ValueError(f"initial long-scan state must have shape {(B, H)}")
        init = torch.stack(states, dim=0)
    with torch.autocast("cuda", enabled=False):
        out, fin = LongScan.apply(
            write, plasticity, read.logit_retain, read.logit_expect_retain,
            read.logit_retention_decay, read.logit_retention_strength, init,
            bool(return_final_state),
        )
    if not torch.compiler.is_compiling():
        read._last_long_backend = "b200_cuda"
    if return_final_state:
        return out, (fin[0], fin[1], fin[2])
    return out
