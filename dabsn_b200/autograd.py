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

import os

import torch
from torch import Tensor

from . import _native, ops


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
                mode, total_steps, compute_dtype, out_dtype=None):
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
        return out.to(query.dtype if out_dtype is None else out_dtype)

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
        return (*grads, None, None, None, None, None, None)


def _compute_dtype(query: Tensor) -> torch.dtype:
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return query.dtype


def three_way_read(read, query, bank_keys, bank_writes, next_writes, cocktail, bank_cocktail,
                   bank_key_bias, bank_admission, scale, bank_idx, bank_valid, *, mode: str,
                   keep_compute_dtype: bool = False):
    """Drop-in for ``cuda_compact_three_way_read`` (triton.py:314-483).  The
    result comes back in the dtype the reference's query has (FP32 under
    autocast, where ``F.normalize`` runs in FP32), or, with
    ``keep_compute_dtype``, in the dtype the read computes in (for a consumer
    that rounds it to that dtype anyway)."""
    if not query.is_cuda:
        raise TypeError("compact CUDA admitted read requires CUDA tensors")
    if mode not in {"seq", "field"}:
        raise ValueError("compact CUDA admitted-read mode must be seq or field")
    cd = _compute_dtype(query)
    if keep_compute_dtype:
        out_dtype = cd
    else:
        out_dtype = torch.float32 if torch.is_autocast_enabled("cuda") else query.dtype
    with torch.autocast("cuda", enabled=False):
        out = ThreeWayRead.apply(
            query, bank_keys, bank_writes, next_writes, cocktail, bank_cocktail, bank_key_bias,
            bank_admission, scale, read.short_gain, read.pad_gain, read.induct_gain,
            read.cocktail_gain, bank_idx, bank_valid, 0 if mode == "seq" else 1,
            int(query.shape[1]), cd, out_dtype,
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


# ---------------------------------------------------------------------------
# Read admission + admitted bank (read.py:152-303 semantics)
# ---------------------------------------------------------------------------
_ADM_PARAMS = ("p_gain", "novelty_gain", "null_bias", "adm_p_gain", "adm_novelty_gain",
               "adm_saturation_gain", "adm_energy_gain", "adm_bias")


class AdmittedBank(torch.autograd.Function):
    """Token statistics, membership, stable bank order and the bank gathers in
    three kernels; the backward assembles every input gradient of a token in
    one kernel.  ``n_cap`` fixes the bank width (capture-safe path); ``None``
    sizes it to the largest member count, as the reference does."""

    @staticmethod
    def forward(ctx, expression, write, novelty, plasticity, energy, saturation, p_gain,
                novelty_gain, null_bias, adm_p_gain, adm_novelty_gain, adm_saturation_gain,
                adm_energy_gain, adm_bias, window, mode, n_cap):
        act = expression.dtype
        params = torch.cat([p.detach().float().reshape(1) for p in (
            p_gain, novelty_gain, null_bias, adm_p_gain, adm_novelty_gain, adm_saturation_gain,
            adm_energy_gain, adm_bias)]).contiguous()
        win = window.detach().float().reshape(1).contiguous()
        expr = expression.detach().contiguous()
        wr = write.detach().to(act).contiguous()
        # The query and the bank keys are produced in the dtype the read
        # computes in (what it would round them to); the backward recomputes
        # their FP32 values from the expression / write rows and the norms.
        rd = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else act
        if rd not in (torch.float32, torch.bfloat16):
            rd = torch.float32
        query, kb, adm, cocktail, stats, order, counts, inv = ops.admission_forward(
            expr, novelty, plasticity, energy, saturation, params, win, mode, query_dtype=rd)
        if n_cap is None:
            n = max(int(counts.max().item()), 1)
            # the stream is synchronised by the read above: surface any
            # timed-out device wait of the launches before it
            _native.raise_on_device_status()
        else:
            n = int(n_cap)
        bw, bk, nw, bc, bb, ba, bi, bv, kn = ops.bank_gather(wr, kb, adm, cocktail, order,
                                                             counts, n, key_dtype=rd)
        ctx.save_for_backward(expr, wr, stats, cocktail, params, inv, kn)
        ctx.n = n
        ctx.meta = [(t.dtype, t.shape) for t in (novelty, plasticity, energy, saturation)]
        ctx.param_meta = [(p.dtype, p.shape) for p in (
            p_gain, novelty_gain, null_bias, adm_p_gain, adm_novelty_gain, adm_saturation_gain,
            adm_energy_gain, adm_bias)]
        ctx.write_dtype = write.dtype
        ctx.mark_non_differentiable(bi, bv)
        if not (act == torch.float32 or torch.is_autocast_enabled("cuda")):
            cocktail = cocktail.to(act)
        return query, cocktail, bk, bw, nw, bc, bb, ba, bi, bv

    @staticmethod
    def backward(ctx, d_query, d_cocktail, d_keys, d_writes, d_next, d_bc, d_bb, d_ba, _i, _v):
        expr, wr, stats, cocktail, params, inv, kn = ctx.saved_tensors
        d_expr, d_write, d_means, part = ops.admission_backward(
            expr, wr, stats, cocktail, params, inv, kn, ctx.n,
            (d_query, d_cocktail, d_keys, d_writes, d_next, d_bc, d_bb, d_ba))
        B, T, H = expr.shape
        # d_means columns: plasticity, novelty, energy, saturation
        col = {"novelty": 1, "plasticity": 0, "energy": 2, "saturation": 3}
        tape_grads = []
        for name, (dt, shape) in zip(("novelty", "plasticity", "energy", "saturation"), ctx.meta):
            g = d_means[..., col[name]].unsqueeze(-1).to(dt).expand(B, T, H)
            tape_grads.append(g)
        psum = part.sum(dim=(0, 1))
        pgrads = [psum[i].reshape(shape).to(dt) for i, (dt, shape) in enumerate(ctx.param_meta)]
        return (d_expr, d_write.to(ctx.write_dtype), *tape_grads, *pgrads, None, None, None)


def make_unified_forward(original):
    """Drop-in for ``DABSNRead._unified_forward`` (read.py:152-303) that builds
    the admitted bank with the fused kernels on CUDA.  CPU tensors, tracing
    (fake tensors, torch.compile) and models whose reads do not take the
    compact CUDA path keep the reference's own method."""
    from torch._subclasses.fake_tensor import is_fake
    import torch.nn.functional as F

    def unified_forward(self, y, budget, expression, write, novelty, plasticity, energy,
                        saturation, field_shape=None):
        compact_cuda = expression.is_cuda and bool(getattr(type(self), "_cuda_native_enabled",
                                                           False))
        if (not compact_cuda or torch.compiler.is_compiling() or is_fake(expression)
                or expression.dtype not in (torch.float32, torch.bfloat16)):
            if (compact_cuda and not torch.compiler.is_compiling() and not is_fake(expression)):
                from .backend import warn_fallback

                warn_fallback("read_admission", "admission for a dtype the fused kernels do not "
                              "cover: the reference's admission runs",
                              dtype=str(expression.dtype),
                              corrective_action="run the read in FP32 or under BF16 autocast")
            return original(self, y, budget, expression, write, novelty, plasticity, energy,
                            saturation, field_shape)
        from dabsn.read import _stream_is_capturing

        rp = self.short_read
        batch, seq_len, hidden = expression.shape
        scale = (F.softplus(rp.log_temp) + 1.0) * (hidden**0.5)
        window = F.softplus(self.admit_window)
        seq = self.read_geometry == "seq"
        admission_policy = "causal_write_prefix_max" if seq else "whole_sequence_max"
        self.last_admit_gate_mean = None
        capture_safe = bool(getattr(self, "_capture_safe_bank", False)) or _stream_is_capturing()
        n_cap = None
        if capture_safe:
            cap = getattr(self, "_capture_bank_width", None)
            n_cap = max(1, min(int(cap) if cap else seq_len, seq_len))
        dt = expression.dtype
        tapes = [t.to(dt) for t in (novelty, plasticity, energy, saturation)]
        (query, cocktail, keys, writes, next_writes, bank_cocktail, bank_bias, bank_adm,
         bank_idx, bank_valid) = AdmittedBank.apply(
            expression, write, *tapes, *[getattr(rp, n) for n in _ADM_PARAMS], window,
            0 if seq else 1, n_cap)
        n_max = int(bank_idx.shape[1])
        self.last_n_max = n_max
        read_paths = 2 if self.read_geometry == "hybrid" else 1
        self.last_read_contract = {
            "read_strategy": "eager_admitted_bank",
            "exact": True,
            "approximation_reason": None,
            "bank_growth": "grows_with_T" if n_max >= seq_len else "data_dependent",
            "stored_writes_preserved": True,
            "max_admitted_bank": n_max,
            "estimated_read_work": int(batch) * int(seq_len) * n_max * 3 * read_paths,
            "dense_masks_materialized": True,
            "context_parallel": False,
            "admission_policy": admission_policy,
            "kernel_backend": "eager_reference",
        }
        trace = bool(self.collect_traces)
        if not seq and trace:
            self.last_field_neighbors = float(bank_valid.detach().sum(dim=1).float().mean().cpu())
        elif not seq:
            self.last_field_neighbors = None

        # The long channel does not depend on the read; computing it first
        # decides whether the output projection takes the fused GEMM, whose
        # BF16 operand the read can then hand over without an FP32 round trip.
        long = self._long_scan(write, plasticity, novelty)
        fused_out = (self.read_geometry != "hybrid"
                     and _read_out_eligible(y, budget, long, rp.out))

        def read(mode):
            if fused_out:
                return three_way_read(
                    self, query, keys, writes, next_writes, cocktail, bank_cocktail, bank_bias,
                    bank_adm, scale, bank_idx, bank_valid, mode=mode, keep_compute_dtype=True)
            return self._admitted_read(
                query, keys, writes, next_writes, cocktail, bank_cocktail, bank_bias, bank_adm,
                scale, None, None, None, None, bank_idx=bank_idx, bank_valid=bank_valid,
                mode=mode)

        if self.read_geometry == "seq":
            retrieved = read("seq")
            self.last_hybrid_gate = None
            self.last_seq_norm = float(retrieved.detach().norm().cpu()) if trace else None
            self.last_field_norm = None
            self.last_field_neighbors = None
        elif self.read_geometry == "field":
            retrieved = read("field")
            self.last_hybrid_gate = None
            self.last_seq_norm = None
            self.last_field_norm = float(retrieved.detach().norm().cpu()) if trace else None
        else:
            seq_retrieved = read("seq")
            field_retrieved = read("field")
            if self.hybrid_gate_override is None:
                gate = torch.sigmoid(self.hybrid_gate)
            else:
                gate = torch.as_tensor(float(self.hybrid_gate_override), device=query.device,
                                       dtype=query.dtype)
            self.last_hybrid_gate = float(gate.detach().cpu()) if trace else None
            seq_contribution = (1.0 - gate) * seq_retrieved
            field_contribution = gate * field_retrieved
            self.last_seq_norm = float(seq_contribution.detach().norm().cpu()) if trace else None
            self.last_field_norm = (float(field_contribution.detach().norm().cpu())
                                    if trace else None)
            retrieved = seq_contribution + field_contribution
        self.last_read_contract.update({
            "read_strategy": "compact_flash_admitted_bank",
            "dense_masks_materialized": False,
            "kernel_backend": getattr(self, "_last_three_way_backend", "eager_reference"),
            "admission_backend": "b200_fused",
        })
        self.last_long_scan_norm = float(long.detach().norm().cpu()) if trace else None
        if fused_out:
            with torch.autocast("cuda", enabled=False):
                return ReadOutput.apply(y, budget, retrieved, rp.out.weight, rp.out.bias, long,
                                        self.long_gain)
        output = rp.out(torch.cat([y, budget, retrieved], dim=-1))
        return output + self.long_gain * long

    unified_forward.__wrapped_reference__ = original
    return unified_forward


# ---------------------------------------------------------------------------
# Primitives of the dabsn.kernels surface (permanent.py, local_field.py)
# ---------------------------------------------------------------------------
def permanent_forward_kernel(k: Tensor, v: Tensor, beta: Tensor) -> Tensor:
    """CUDA kernel for ``dabsn::permanent_delta_scan`` (permanent.py:384-388)."""
    return ops.permanent_delta_forward(k, v, beta)


def make_permanent_backward(reference_backward):
    """Autograd formula of ``dabsn::permanent_delta_scan``: the B200 reverse
    scan for CUDA tensors, the reference's for CPU tensors."""

    def backward(ctx, grad_out):
        k, v, beta = ctx.saved_tensors
        if not k.is_cuda:
            return reference_backward(ctx, grad_out)
        return ops.permanent_delta_backward(k, v, beta, grad_out)

    return backward


def local_field_kernel(inputs: Tensor, patch: Tensor) -> Tensor:
    """CUDA kernel for ``dabsn::local_field_gather`` (local_field.py:208-214)."""
    return ops.local_field_gather(inputs, patch)


def make_local_field_backward(reference_backward):
    def backward(ctx, grad_out):
        if not grad_out.is_cuda:
            return reference_backward(ctx, grad_out)
        (patch,) = ctx.saved_tensors
        return ops.local_field_scatter(grad_out, patch, ctx.cells), None

    return backward


# ---------------------------------------------------------------------------
# Readout + cross-entropy (runtime/loss.py:52-231)
# ---------------------------------------------------------------------------
class LinearCrossEntropy(torch.autograd.Function):
    """Mean cross-entropy of ``hidden @ weight^T + bias`` on the tcgen05 GEMM;
    saves the inputs and the per-row log-sum-exp, never the logits."""

    @staticmethod
    def forward(ctx, hidden, weight, bias, targets, ignore_index, round_bf16, empty_nan=False,
                row_chunk=None):
        bf = torch.bfloat16
        h = hidden.detach().to(bf).contiguous()
        w = weight.detach().to(bf).contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        t = targets.detach().to(torch.int64).contiguous()
        lse, tgt = ops.linear_ce_forward(h, w, b, t, ignore_index, round_bf16)
        valid = t != ignore_index
        count = valid.sum().clamp_min(1).to(torch.float32)
        loss = ((lse - tgt) * valid).sum() / count
        if empty_nan:
            # the reference's single-shot branch (F.cross_entropy) averages over
            # no rows when every target is ignored: NaN loss, zero gradients
            loss = torch.where(valid.any(), loss, torch.full_like(loss, float("nan")))
        ctx.save_for_backward(h, w, b if b is not None else torch.empty(0, device=h.device), t,
                              lse, count)
        ctx.has_bias = bias is not None
        ctx.meta = (hidden.dtype, weight.dtype, None if bias is None else bias.dtype)
        ctx.ignore_index = ignore_index
        ctx.round_bf16 = round_bf16
        ctx.row_chunk = row_chunk
        return loss

    @staticmethod
    def backward(ctx, grad):
        h, w, b, t, lse, count = ctx.saved_tensors
        scale = (grad.float() / count).reshape(1).contiguous()  # stays on the device
        dh, dw, db = ops.linear_ce_backward(h, w, b if ctx.has_bias else None, t,
                                            ctx.ignore_index, ctx.round_bf16, lse, scale,
                                            ctx.row_chunk)
        hd, wd, bd = ctx.meta
        return (dh.to(hd), dw.to(wd), (None if db is None else db.to(bd)), None, None, None, None,
                None)


def _reference_single_shot(original, rows: int, vocab: int, chunk_budget) -> bool:
    """Whether the reference's function would compute this call in one shot
    with ``F.cross_entropy`` (runtime/loss.py:162-180: ``DABSN_LOSS_CHUNK_SCORES``
    set to ``off``, or rows * vocab within the element budget) rather than
    chunked.  The two branches differ only when every target is ignored (NaN
    against 0); the fused loss follows the branch the reference would take."""
    import os
    import sys

    env = os.environ.get("DABSN_LOSS_CHUNK_SCORES", "")
    if env.lower() == "off":
        return True
    budget = chunk_budget
    if budget is None and env:
        try:
            budget = int(env)
        except ValueError:
            budget = None
    default = getattr(sys.modules.get(getattr(original, "__module__", ""), None),
                      "_DEFAULT_CHUNK_BUDGET", 1 << 24)
    return rows * vocab <= (budget if budget is not None else default)


# Reverse workspace bound when the caller names no budget: the BF16 dlogits of
# one row chunk stay within 1 GiB.
_CE_DEFAULT_WORKSPACE_BYTES = 1 << 30
# Smallest row chunk: one 128-row tile of the reverse GEMMs.
_CE_MIN_CHUNK_ROWS = 128


def _linear_ce_row_chunk(rows: int, vocab: int, chunk_budget) -> int:
    """Rows per reverse chunk.  With a budget (``chunk_budget`` or
    ``DABSN_LOSS_CHUNK_SCORES``; runtime/loss.py:32-39) the BF16 dlogits chunk
    holds at most 2 x budget elements (the bytes of the reference's FP32
    chunk logits), but no fewer than 128 rows; without one, at most 1 GiB."""
    ld = int(_native.load().dabsn_linear_ce_ld(vocab))
    budget = chunk_budget
    env = os.environ.get("DABSN_LOSS_CHUNK_SCORES", "")
    if budget is None and env and env.lower() != "off":
        try:
            budget = int(env)
        except ValueError:
            budget = None
    if budget is not None and budget > 0:
        per = (2 * budget) // ld
    else:
        per = _CE_DEFAULT_WORKSPACE_BYTES // (2 * ld)
    return max(1, min(rows, max(per, _CE_MIN_CHUNK_ROWS)))


def make_linear_cross_entropy(original):
    """Drop-in for ``dabsn.runtime.chunked_linear_cross_entropy``: BF16 CUDA
    inputs (BF16 tensors or autocast) run the fused kernels; everything else
    keeps the reference's function."""

    def chunked_linear_cross_entropy(hidden, weight, bias, targets, *, ignore_index=-100,
                                     chunk_budget=None):
        autocast = hidden.is_cuda and torch.is_autocast_enabled("cuda") and (
            torch.get_autocast_dtype("cuda") == torch.bfloat16)
        bf16 = autocast or (hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16)
        if not hidden.is_cuda or not bf16 or hidden.shape[-1] % 8:
            if hidden.is_cuda:
                from .backend import warn_fallback

                warn_fallback("linear_cross_entropy", "readout + cross-entropy outside the fused "
                              "kernels' cover (FP32 operands or a width not a multiple of 8): "
                              "the reference's chunked loss runs", dtype=str(hidden.dtype),
                              width=int(hidden.shape[-1]),
                              corrective_action="run the loss under BF16 autocast")
            return original(hidden, weight, bias, targets, ignore_index=ignore_index,
                            chunk_budget=chunk_budget)
        flat = hidden.reshape(-1, hidden.shape[-1])
        single = _reference_single_shot(original, flat.shape[0], weight.shape[0], chunk_budget)
        row_chunk = _linear_ce_row_chunk(flat.shape[0], weight.shape[0], chunk_budget)
        with torch.autocast("cuda", enabled=False):
            return LinearCrossEntropy.apply(flat, weight, bias, targets.reshape(-1),
                                            int(ignore_index), True, single, row_chunk)

    chunked_linear_cross_entropy.__wrapped_reference__ = original
    return chunked_linear_cross_entropy


class CrossEntropyFromLogits(torch.autograd.Function):
    """Mean cross-entropy over materialised logits in one pass each way: the
    logits are read in their own dtype and never widened in memory; the
    gradient is written in that dtype directly."""

    @staticmethod
    def forward(ctx, logits, targets, ignore_index, empty_nan):
        flat = logits.detach().reshape(-1, logits.shape[-1])
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        t = targets.detach().reshape(-1).to(torch.int64).contiguous()
        lse, tgt = ops.ce_logits_forward(flat, t, ignore_index)
        valid = t != ignore_index
        count = valid.sum().clamp_min(1).to(torch.float32)
        loss = ((lse - tgt) * valid).sum() / count
        if empty_nan:
            # the reference's single-shot branch (F.cross_entropy) averages over
            # no rows when every target is ignored: NaN loss, zero gradients
            loss = torch.where(valid.any(), loss, torch.full_like(loss, float("nan")))
        ctx.save_for_backward(flat, t, lse, count)
        ctx.shape = logits.shape
        ctx.ignore_index = ignore_index
        return loss

    @staticmethod
    def backward(ctx, grad):
        flat, t, lse, count = ctx.saved_tensors
        scale = (grad.float() / count).reshape(1).contiguous()  # stays on the device
        dl = ops.ce_logits_backward(flat, t, ctx.ignore_index, lse, scale)
        return dl.reshape(ctx.shape), None, None, None


def make_ce_from_logits(original):
    """Drop-in for ``dabsn.runtime.loss.chunked_cross_entropy_from_logits``
    (runtime/loss.py:187-231; the default loss of ``runtime.api.train_step``):
    CUDA FP32/BF16 logits run the one-pass kernels; other inputs (CPU, FP64,
    FP16) keep the reference's function."""

    def chunked_cross_entropy_from_logits(logits, targets, *, ignore_index=-100,
                                          chunk_budget=None):
        if (not logits.is_cuda or logits.dtype not in (torch.float32, torch.bfloat16)
                or torch.compiler.is_compiling()):
            if logits.is_cuda and logits.dtype == torch.float16:
                from .backend import warn_fallback

                warn_fallback("cross_entropy_from_logits", "FP16 logits: the reference's "
                              "chunked loss runs", dtype=str(logits.dtype))
            return original(logits, targets, ignore_index=ignore_index, chunk_budget=chunk_budget)
        rows = logits.numel() // max(1, logits.shape[-1])
        single = _reference_single_shot(original, rows, logits.shape[-1], chunk_budget)
        with torch.autocast("cuda", enabled=False):
            return CrossEntropyFromLogits.apply(logits, targets, int(ignore_index), single)

    chunked_cross_entropy_from_logits.__wrapped_reference__ = original
    return chunked_cross_entropy_from_logits


class CoreInputProjection(torch.autograd.Function):
    """``W(x)`` and ``Wg(x)`` of the core (core.py:280-283) in one tcgen05
    GEMM launch with the bias in the epilogue, and their reverse in two (dx
    accumulating both pairs; dW and dWg as two problems).  BF16 operands as
    autocast casts them; FP32 parameter gradients from BF16 GEMM outputs, as
    autocast's casts return them."""

    @staticmethod
    def forward(ctx, x, W, Wg, bias_g):
        bf = torch.bfloat16
        shape = x.shape
        xb = x.detach().reshape(-1, shape[-1]).to(bf).contiguous()
        Wb = W.detach().to(bf).contiguous()
        Wgb = Wg.detach().to(bf).contiguous()
        b = None if bias_g is None else bias_g.detach().float().contiguous()
        wx, wgx = ops.input_proj_forward(xb, Wb, Wgb, b)
        ctx.save_for_backward(xb, Wb, Wgb)
        ctx.meta = (x.dtype, shape, W.dtype, Wg.dtype, None if bias_g is None else bias_g.dtype)
        H = W.shape[0]
        return wx.reshape(*shape[:-1], H), wgx.reshape(*shape[:-1], H)

    @staticmethod
    def backward(ctx, g_wx, g_wgx):
        xb, Wb, Wgb = ctx.saved_tensors
        xdt, shape, wdt, wgdt, bdt = ctx.meta
        H = Wb.shape[0]
        bf = torch.bfloat16
        rows = xb.shape[0]
        g1 = (torch.zeros((rows, H), device=xb.device, dtype=bf) if g_wx is None
              else g_wx.reshape(rows, H).to(bf).contiguous())
        g2 = (torch.zeros((rows, H), device=xb.device, dtype=bf) if g_wgx is None
              else g_wgx.reshape(rows, H).to(bf).contiguous())
        dx, dW, dWg = ops.input_proj_backward(xb, Wb, Wgb, g1, g2, ctx.needs_input_grad[0])
        # the bias gradient as autocast's addmm forms it: a BF16 row sum
        db = (ops.colsum_bf16(g2).to(bf).to(bdt)
              if (bdt is not None and ctx.needs_input_grad[3]) else None)
        return (None if dx is None else dx.reshape(shape).to(xdt), dW.to(wdt), dWg.to(wgdt), db)


def _proj_eligible(core, inputs) -> bool:
    """The tcgen05 projections cover CUDA inputs under BF16 autocast (the
    configurations whose reference GEMMs are BF16) with widths that are
    multiples of 8."""
    from torch._subclasses.fake_tensor import is_fake

    if (not inputs.is_cuda or inputs.dim() != 3 or torch.compiler.is_compiling()
            or is_fake(inputs)):
        return False
    if not (torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16):
        return False
    D, H = inputs.shape[-1], core.hidden_dim
    return D % 8 == 0 and H % 8 == 0 and bool(getattr(type(core), "_cuda_native_enabled", False))


def make_core_forward(original):
    """Drop-in for ``DABSNCore.forward_from_state`` (core.py:248-342) that
    forms ``W(x)`` and ``Wg(x)`` with ``CoreInputProjection`` and then runs
    the reference's own registered scan op and result contract; everything
    else (CPU, FP32, tracing, subclasses with their own method) keeps the
    reference's method."""

    def forward_from_state(self, inputs, *, initial_state=None, return_writes=False,
                           return_cocktail=False, return_final_state=False):
        if not _proj_eligible(self, inputs):
            return original(self, inputs, initial_state=initial_state, return_writes=return_writes,
                            return_cocktail=return_cocktail,
                            return_final_state=return_final_state)
        batch = inputs.shape[0]
        if initial_state is None:
            initial_state = self.initial_state(batch, device=inputs.device, dtype=inputs.dtype)
        else:
            state_values = tuple(v.to(device=inputs.device, dtype=inputs.dtype)
                                 for v in initial_state)
            expected = (batch, self.hidden_dim)
            if any(v.shape != expected for v in state_values):
                shapes = tuple(tuple(v.shape) for v in state_values)
                raise ValueError(f"initial_state tensors must have shape {expected}, got {shapes}")
            initial_state = (state_values[0], state_values[1], state_values[2])
        from dabsn.kernels.batched_runtime import dabsn_core_scan_batched

        with torch.autocast("cuda", enabled=False):
            wx, wgx = CoreInputProjection.apply(inputs, self.W.weight, self.Wg.weight,
                                                self.Wg.bias)
        outputs = dabsn_core_scan_batched(
            wx, wgx, self.Ug.weight, self.A.weight, self.beta, self.log_kappa,
            self.logit_recover, self.k_s, self.k_y, self.k_b, self.k_n, self.k_bias, self.r_s,
            self.r_y, self.r_b, self.r_n, self.r_bias,
            self.logit_saturation_decay.expand(self.hidden_dim), self.k_saturation,
            self.r_saturation, self.logit_alpha.reshape(()), self.log_lambda.reshape(()),
            self.logit_saturation_suppress.reshape(()), return_tape=return_cocktail,
            initial_state=initial_state, return_final_state=return_final_state)
        self._last_core_backend = "cuda_registered"
        trajectory, novelty, plasticity, expression, write = outputs[:5]
        if return_cocktail:
            result = (trajectory, novelty, plasticity, expression, write, outputs[5], outputs[6])
            final_offset = 7
        elif return_writes:
            result = trajectory, novelty, plasticity, expression, write
            final_offset = 5
        else:
            result = trajectory, novelty, plasticity
            final_offset = 5
        if return_final_state:
            return result, tuple(outputs[final_offset:final_offset + 3])
        return result

    forward_from_state.__wrapped_reference__ = original
    return forward_from_state


class ReadOutput(torch.autograd.Function):
    """The read's ``out(cat[y, b, retrieved]) + long_gain * long`` (read.py:435-438)
    on the tcgen05 GEMM: three operand pairs accumulated in one launch (y and
    b read in place from the U tape, no concatenated copy), bias and the FP32
    long-channel term in the epilogue; autocast's rounding points (BF16
    operands, BF16 Linear output, FP32 sum)."""

    @staticmethod
    def forward(ctx, y, budget, retrieved, weight, bias, long, long_gain):
        bf = torch.bfloat16
        yb = y.detach() if y.dtype == bf else y.detach().to(bf)
        bb = budget.detach() if budget.dtype == bf else budget.detach().to(bf)
        rb = retrieved.detach().to(bf).contiguous()
        wb = weight.detach().to(bf).contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        lg = long_gain.detach().float().reshape(1).contiguous()
        lf = long.detach().float().contiguous()
        out = ops.read_out_forward(yb, bb, rb, wb, b, lf, lg)
        ctx.save_for_backward(yb, bb, rb, wb, lf, lg)
        ctx.meta = (y.dtype, budget.dtype, retrieved.dtype, weight.dtype,
                    None if bias is None else bias.dtype, long.dtype, long_gain.dtype,
                    long_gain.shape)
        return out.reshape(long.shape)

    @staticmethod
    def backward(ctx, grad):
        yb, bb, rb, wb, lf, lg = ctx.saved_tensors
        ydt, bdt, rdt, wdt, biasdt, ldt, lgdt, lgshape = ctx.meta
        H = wb.shape[0]
        g = grad.reshape(-1, H)
        shape = lf.shape
        if g.dtype == torch.float32:
            # one pass: the BF16 operand, the long channel's gradient, the
            # bias gradient (a BF16 column sum, as autocast's addmm forms it)
            # and the gain's gradient
            gb, dl, colsum, dot = ops.read_out_grad_prep(g.contiguous(), lf.reshape(-1, H), lg)
            dbias = colsum.to(torch.bfloat16).to(biasdt) if biasdt is not None else None
            dlong = dl.reshape(shape).to(ldt)
            dlg = dot.reshape(lgshape).to(lgdt)
        else:
            gb = g.to(torch.bfloat16).contiguous()
            dbias = gb.sum(dim=0).to(biasdt) if biasdt is not None else None
            gf = grad.float()
            dlong = (gf * lg).to(ldt)
            dlg = (gf * lf).sum().reshape(lgshape).to(lgdt)
        dy, db_, dr, dW = ops.read_out_backward(yb, bb, rb, wb, gb)
        return (dy.reshape(shape).to(ydt), db_.reshape(shape).to(bdt), dr.reshape(shape).to(rdt),
                dW.to(wdt), dbias, dlong, dlg)


def _read_out_eligible(y, budget, long, out_linear) -> bool:
    """The fused output projection covers CUDA tensors under BF16 autocast with
    a width that is a multiple of 8 and y / b rows that can be read in place."""
    if not (y.is_cuda and torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16):
        return False
    if torch.compiler.is_compiling() or os.environ.get("DABSN_B200_PROJ", "1") == "0":
        return False
    H = y.shape[-1]
    if H % 8 or out_linear.weight.shape != (H, 3 * H) or long.shape != y.shape:
        return False
    for t in (y, budget):
        if t.stride(-1) != 1 or t.reshape(-1, H).stride(0) % 8 or t.data_ptr() % 16:
            return False
    return True

