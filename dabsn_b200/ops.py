"""Tensor-level wrappers over the C ABI.

Each function takes torch CUDA tensors, allocates its outputs through the
PyTorch caching allocator, and launches on the current CUDA stream of the
tensors' device.  None of them synchronises with the host, so all of them can
be captured in a CUDA graph.
"""

from __future__ import annotations

import ctypes
import os

import torch
from torch import Tensor

from . import _native as N

PARAM_ORDER = N.CoreParams._fields_

# Optional per-kernel timing: when ``KERNEL_EVENTS`` is a dict, every launch
# below records a CUDA event pair on the launching stream under its kernel
# name (used by bench.py for the roofline of the dominant kernel).
KERNEL_EVENTS: dict[str, list] | None = None
LAUNCH_COUNT = {"n": 0}


class _timed:
    def __init__(self, name: str, device: torch.device, launches: int = 1):
        self.name = name
        self.device = device
        self.launches = launches

    def __enter__(self):
        LAUNCH_COUNT["n"] += self.launches
        if KERNEL_EVENTS is not None:
            self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.ev[0].record(torch.cuda.current_stream(self.device))
        return self

    def __exit__(self, *exc):
        if KERNEL_EVENTS is not None:
            self.ev[1].record(torch.cuda.current_stream(self.device))
            KERNEL_EVENTS.setdefault(self.name, []).append(self.ev)
        return False


def _ptr(t: Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def act_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return N.F32
    if dtype == torch.bfloat16:
        return N.BF16
    raise TypeError(f"dabsn_b200 kernels take float32 or bfloat16 activations, got {dtype}")


def _require_cuda(*tensors: Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise TypeError("dabsn_b200 kernels require CUDA tensors")
    for t in tensors:
        if t is not None and t.device != dev:
            raise ValueError("dabsn_b200: all tensors must be on the same device")
    return dev


def _f32(t: Tensor, shape=None) -> Tensor:
    t = t.detach().to(torch.float32)
    if shape is not None:
        t = t.reshape(shape)
    return t.contiguous()


def _grad_or_none(g: Tensor | None) -> Tensor | None:
    if g is None:
        return None
    return g.detach().to(torch.float32).contiguous()


class _ParamPack:
    """Keeps the FP32 parameter tensors alive while the kernel is queued."""

    def __init__(self, per_unit: list[Tensor], scalars: list[Tensor], H: int):
        self.tensors = [_f32(t, (H,)) for t in per_unit] + [_f32(t, (1,)) for t in scalars]
        self.struct = N.CoreParams(*[t.data_ptr() for t in self.tensors])


# ---------------------------------------------------------------------------
# Core scan
# ---------------------------------------------------------------------------
# Widths up to NARROW_MAX_H run the register-resident cluster scan (FP32 or
# BF16); wider states run the grid-wide scan (BF16), 32 sequences per launch.
# DABSN_B200_NARROW_MAX_H lowers the switch-over (tests compare both scans at
# one width).
NARROW_MAX_H = int(os.environ.get("DABSN_B200_NARROW_MAX_H", "256"))
WIDE_MAX_B = 32


def _wide_scratch(lib, H: int, dev: torch.device) -> Tensor:
    """Exchange buffer + barrier counter of the grid-wide scan."""
    return torch.empty(int(lib.dabsn_core_scan_wide_scratch_bytes(H)), dtype=torch.uint8, device=dev)

def core_scan_forward(
    Wx: Tensor, Wgx: Tensor, Ug: Tensor, A: Tensor, params: list[Tensor], init_b: Tensor,
    init_e: Tensor, init_c: Tensor,
) -> tuple[Tensor, ...]:
    """Forward of ``dabsn::core_scan_batched``: 11 outputs in the reference order
    ``(U, novelty, plasticity, expression, write, energy, saturation, gate,
    final_b, final_e, final_c)`` (batched_runtime.py:1098-1205)."""
    dev = _require_cuda(Wx, Wgx, Ug, A)
    B, T, H = Wx.shape
    if Wgx.shape != Wx.shape or Ug.shape != (H, H) or A.shape != (H, H):
        raise ValueError("core_scan_batched received incompatible tensor shapes")
    dt = Wx.dtype
    code = act_code(dt)
    Wx = Wx.detach().contiguous()
    Wgx = Wgx.detach().to(dt).contiguous()
    rec = torch.cat((Ug.detach(), A.detach()), dim=0).to(dt).contiguous()
    pack = _ParamPack(list(params[:16]), list(params[16:19]), H)
    ib, ie, ic = (_f32(t, (B, H)) for t in (init_b, init_e, init_c))
    U = torch.empty((B, T, 2 * H), device=dev, dtype=dt)
    tapes = [torch.empty((B, T, H), device=dev, dtype=dt) for _ in range(7)]
    fins = [torch.empty((B, H), device=dev, dtype=dt) for _ in range(3)]
    if T == 0:
        for f, i in zip(fins, (ib, ie, ic)):
            f.copy_(i)
    else:
        lib = N.load()
        with torch.cuda.device(dev), _timed("core_scan_fwd", dev):
            if H > NARROW_MAX_H:
                if dt != torch.bfloat16:
                    raise TypeError(f"dabsn_b200: states wider than {NARROW_MAX_H} units run in "
                                    "bfloat16 only (use autocast)")
                scratch = _wide_scratch(lib, H, dev)
                for b0 in range(0, B, WIDE_MAX_B):
                    b1 = min(B, b0 + WIDE_MAX_B)
                    st = lib.dabsn_core_scan_wide_fwd(
                        b1 - b0, T, H, _ptr(Wx[b0:b1]), _ptr(Wgx[b0:b1]), _ptr(rec),
                        ctypes.byref(pack.struct), _ptr(ib[b0:b1]), _ptr(ie[b0:b1]),
                        _ptr(ic[b0:b1]), _ptr(U[b0:b1]), *[_ptr(t[b0:b1]) for t in tapes],
                        *[_ptr(f[b0:b1]) for f in fins], _ptr(scratch), scratch.numel(),
                        _stream(dev),
                    )
                    N.check(st, "core_scan_wide_fwd")
            else:
                st = lib.dabsn_core_scan_fwd(
                    code, B, T, H, _ptr(Wx), _ptr(Wgx), _ptr(rec), ctypes.byref(pack.struct),
                    _ptr(ib), _ptr(ie), _ptr(ic), _ptr(U), *[_ptr(t) for t in tapes],
                    *[_ptr(f) for f in fins], _stream(dev),
                )
                N.check(st, "core_scan_fwd")
    return (U, *tapes, *fins)


def core_scan_backward(
    saved: tuple[Tensor, ...], grads: tuple[Tensor | None, ...]
) -> tuple[Tensor | None, ...]:
    """Gradients of the 26 operator inputs.

    ``saved`` is the reference's saved context (the 26 inputs followed by
    ``U, plasticity, expression, energy, saturation, gate, final_b, final_e,
    final_c``; batched_runtime.py:1578-1604).  ``grads`` are the 11 output
    gradients; as in the reference the gate-tape gradient (index 7) is not
    propagated (batched_runtime.py:1613-1620).
    """
    inputs = saved[:26]
    U, plast, expr, e_tape, c_tape, s_tape = saved[26:32]
    Wx, Wgx, Ug, A = inputs[:4]
    params = inputs[4:23]
    init_b, init_e, init_c = inputs[23:26]
    dev = _require_cuda(U)
    B, T, H = plast.shape
    dt = Wx.dtype
    if Wgx.dtype != dt:
        raise RuntimeError("core_scan_batched backward requires Wx and Wgx to share a dtype")
    code = act_code(dt)
    rec = torch.cat((Ug.detach(), A.detach()), dim=0).to(dt).contiguous()
    pack = _ParamPack(list(params[:16]), list(params[16:19]), H)
    ib = _f32(init_b, (B, H))
    ic = _f32(init_c, (B, H))
    wide = H > NARROW_MAX_H
    # The grid-wide reverse reads BF16 tape gradients as they arrive (autograd
    # delivers them in the tapes' dtype); everything else reads FP32.
    tape_grads = [g for g in grads[:7] if g is not None]
    grad_bf16 = wide and bool(tape_grads) and all(g.dtype == torch.bfloat16 for g in tape_grads)
    row_bcast = 0
    if grad_bf16:
        # a gradient that is one value per (sequence, step) expanded over the
        # units (a per-token mean's gradient) is passed as [B, T]
        tg = []
        for i, g in enumerate(grads[:7]):
            if g is not None and i > 0 and g.dim() == 3 and g.stride(-1) == 0:
                row_bcast |= 1 << (i - 1)
                g = g[..., 0]
            tg.append(None if g is None else g.detach().contiguous())
        gU, gnov, gp, gay, gw, ge, gc = tg
    else:
        gU, gnov, gp, gay, gw, ge, gc = (_grad_or_none(g) for g in grads[:7])
    gfb, gfe, gfc = (_grad_or_none(g) for g in grads[8:11])
    gWx = torch.empty((B, T, H), device=dev, dtype=dt)
    gWgx = torch.empty_like(gWx)
    day = torch.empty_like(gWx)
    g_init = torch.empty((3, B, H), device=dev, dtype=torch.float32)
    partial = torch.empty((B, 19, H), device=dev, dtype=torch.float32)
    if T == 0:
        gWx.zero_()
        gWgx.zero_()
        day.zero_()
        partial.zero_()
        for i, g in enumerate((gfb, gfe, gfc)):
            g_init[i].copy_(g if g is not None else torch.zeros(B, H, device=dev))
    else:
        lib = N.load()
        tapes = [t.detach().contiguous() for t in (U, e_tape, c_tape, s_tape, plast, expr)]
        with torch.cuda.device(dev), _timed("core_scan_bwd", dev):
            if H > NARROW_MAX_H:
                if dt != torch.bfloat16:
                    raise TypeError(f"dabsn_b200: states wider than {NARROW_MAX_H} units run in "
                                    "bfloat16 only (use autocast)")
                scratch = _wide_scratch(lib, H, dev)

                def sl(t, b0, b1):
                    return None if t is None else _ptr(t[b0:b1])

                for b0 in range(0, B, WIDE_MAX_B):
                    b1 = min(B, b0 + WIDE_MAX_B)
                    st = lib.dabsn_core_scan_wide_bwd(
                        b1 - b0, T, H, *[sl(t, b0, b1) for t in tapes], _ptr(rec),
                        ctypes.byref(pack.struct), sl(ib, b0, b1), sl(ic, b0, b1),
                        N.BF16 if grad_bf16 else N.F32, row_bcast,
                        *[sl(g, b0, b1) for g in (gU, gnov, gp, gay, gw, ge, gc, gfb, gfe, gfc)],
                        sl(gWx, b0, b1), sl(gWgx, b0, b1), sl(day, b0, b1),
                        sl(g_init[0], b0, b1), sl(g_init[1], b0, b1), sl(g_init[2], b0, b1),
                        sl(partial, b0, b1), _ptr(scratch), scratch.numel(), _stream(dev),
                    )
                    N.check(st, "core_scan_wide_bwd")
            else:
                st = lib.dabsn_core_scan_bwd(
                    code, B, T, H, *[_ptr(t) for t in tapes], _ptr(rec), ctypes.byref(pack.struct),
                    _ptr(ib), _ptr(ic), _ptr(gU), _ptr(gnov), _ptr(gp), _ptr(gay), _ptr(gw),
                    _ptr(ge), _ptr(gc), _ptr(gfb), _ptr(gfe), _ptr(gfc), _ptr(gWx), _ptr(gWgx),
                    _ptr(day), _ptr(g_init[0]), _ptr(g_init[1]), _ptr(g_init[2]), _ptr(partial),
                    _stream(dev),
                )
                N.check(st, "core_scan_bwd")
    # grad[Ug;A] = [gWgx, day]^T . y over all (b, t): a plain library GEMM in
    # the activation dtype, as batched_runtime.py:1474-1481 forms it.
    if dt == torch.bfloat16 and H % 8 == 0 and B * T > 0:
        # the same product on this library's tcgen05 GEMM (one launch, two problems)
        gUg, gA = rec_grad(U.detach().reshape(B * T, 2 * H)[:, :H], gWgx.reshape(B * T, H),
                           day.reshape(B * T, H))
        grad_Ug, grad_A = gUg.float(), gA.float()
    else:
        y_flat = U[:, :, :H].reshape(B * T, H).to(dt)
        grad_rec = (torch.cat((gWgx, day), dim=-1).reshape(B * T, 2 * H).T @ y_flat).float()
        grad_Ug, grad_A = grad_rec.split(H, dim=0)
    sums = partial.sum(dim=0)  # [19, H]
    out: list[Tensor | None] = [gWx.to(Wx.dtype), gWgx.to(Wgx.dtype), grad_Ug.to(Ug.dtype), grad_A.to(A.dtype)]
    for j in range(16):
        out.append(sums[j].to(params[j].dtype).reshape(params[j].shape))
    for j in range(3):
        p = params[16 + j]
        out.append(sums[16 + j].sum().reshape(p.shape).to(p.dtype))
    for g, ref in zip(g_init, (init_b, init_e, init_c)):
        out.append(g.to(ref.dtype).reshape(ref.shape))
    return tuple(out)


# ---------------------------------------------------------------------------
# Long-memory channel
# ---------------------------------------------------------------------------
def long_chunk() -> int:
    return int(N.load().dabsn_long_chunk())


def long_forward(
    write: Tensor, plasticity: Tensor, logits: Tensor, init: Tensor | None, *,
    save_checkpoints: bool, want_final: bool,
) -> tuple[Tensor, Tensor | None, Tensor | None]:
    """Fused long channel forward. ``logits`` is FP32 [4]; ``init`` FP32 [3,B,H]
    (long, expected, retention) or None.  Returns (out [B,T,H] FP32,
    checkpoints or None, final [3,B,H] or None)."""
    dev = _require_cuda(write, plasticity)
    B, T, H = write.shape
    dt = write.dtype
    code = act_code(dt)
    w = write.detach().contiguous()
    p = plasticity.detach().to(dt).contiguous()
    out = torch.empty((B, T, H), device=dev, dtype=torch.float32)
    nch = (T + long_chunk() - 1) // long_chunk()
    ckpt = torch.empty((B, nch, 3, H), device=dev, dtype=torch.float32) if save_checkpoints else None
    fin = torch.empty((3, B, H), device=dev, dtype=torch.float32) if want_final else None
    if T == 0 and fin is not None:
        if init is None:
            fin.zero_()
            fin[2].fill_(1.0)
        else:
            fin.copy_(init)
    if T > 0 and B > 0:
        lib = N.load()
        with torch.cuda.device(dev), _timed("long_fwd", dev):
            st = lib.dabsn_long_fwd(
                code, B, T, H, _ptr(w), _ptr(p), _ptr(logits), _ptr(init), _ptr(out), _ptr(ckpt),
                _ptr(fin), _stream(dev),
            )
        N.check(st, "long_fwd")
    return out, ckpt, fin


def long_backward(
    write: Tensor, plasticity: Tensor, logits: Tensor, ckpt: Tensor, gout: Tensor | None,
    gfin: Tensor | None, want_ginit: bool,
) -> tuple[Tensor, Tensor, Tensor, Tensor | None]:
    """Returns (d write, d plasticity, d logits [4] FP32, d init [3,B,H] or None)."""
    dev = _require_cuda(write)
    B, T, H = write.shape
    dt = write.dtype
    code = act_code(dt)
    w = write.detach().contiguous()
    p = plasticity.detach().to(dt).contiguous()
    go = gout.detach().float().contiguous() if gout is not None else torch.zeros((B, T, H), device=dev)
    gf = gfin.detach().float().contiguous() if gfin is not None else None
    dw = torch.empty((B, T, H), device=dev, dtype=dt)
    dp = torch.empty((B, T, H), device=dev, dtype=dt)
    ginit = torch.empty((3, B, H), device=dev, dtype=torch.float32) if want_ginit else None
    partial = torch.empty((B * H, 4), device=dev, dtype=torch.float32)
    if T == 0 or B == 0:
        dw.zero_()
        dp.zero_()
        partial.zero_()
        if ginit is not None:
            ginit.copy_(gf if gf is not None else torch.zeros_like(ginit))
    else:
        lib = N.load()
        with torch.cuda.device(dev), _timed("long_bwd", dev):
            st = lib.dabsn_long_bwd(
                code, B, T, H, _ptr(w), _ptr(p), _ptr(logits), _ptr(ckpt), _ptr(go), _ptr(gf),
                _ptr(dw), _ptr(dp), _ptr(ginit), _ptr(partial), _stream(dev),
            )
        N.check(st, "long_bwd")
    return dw, dp, partial.sum(dim=0), ginit


# ---------------------------------------------------------------------------
# Three-way admitted read
# ---------------------------------------------------------------------------
# States wider than this run the tensor-core read (BF16).
# DABSN_B200_NARROW_READ_MAX_H lowers the switch-over (tests compare both reads
# at one width).
NARROW_READ_MAX_H = int(os.environ.get("DABSN_B200_NARROW_READ_MAX_H", "256"))


def read_forward(
    query: Tensor, keys: Tensor, writes: Tensor, next_writes: Tensor, cocktail: Tensor,
    bank_cocktail: Tensor, key_bias: Tensor, admission: Tensor, scale: Tensor, idx: Tensor,
    valid: Tensor, gains: Tensor, mode: int, total_steps: int,
) -> tuple[Tensor, Tensor, Tensor]:
    """Query, keys, writes, next writes and cocktails in one activation dtype,
    contiguous; key bias / admission in any float dtype.

    Returns ``(out [B,T,H] activation dtype, saved, lse [B,T,3])``; ``saved``
    is what :func:`read_backward` needs besides the inputs: the per-stream
    reads ``[B,T,3,H]`` FP32 (H <= NARROW_READ_MAX_H) or the BF16 score
    products ``[B,T,ld]`` of the tensor-core read."""
    dev = _require_cuda(query)
    B, T, H = query.shape
    Nb = keys.shape[1]
    if H > NARROW_READ_MAX_H:
        return _read_wide_forward(query, keys, writes, next_writes, cocktail, bank_cocktail,
                                  key_bias, admission, scale, idx, valid, gains, mode,
                                  total_steps)
    code = act_code(query.dtype)
    key_bias = key_bias.to(query.dtype).contiguous()
    admission = admission.to(query.dtype).contiguous()
    out = torch.empty((B, T, H), device=dev, dtype=query.dtype)
    streams = torch.empty((B, T, 3, H), device=dev, dtype=torch.float32)
    lse = torch.empty((B, T, 3), device=dev, dtype=torch.float32)
    if Nb == 0:
        out.zero_()
        streams.zero_()
        lse.fill_(float("inf"))
        return out, streams, lse
    lib = N.load()
    with torch.cuda.device(dev), _timed("read_fwd", dev):
        st = lib.dabsn_read_fwd(
            code, B, T, Nb, H, mode, total_steps, _ptr(query), _ptr(keys), _ptr(writes),
            _ptr(next_writes), _ptr(cocktail), _ptr(bank_cocktail), _ptr(key_bias),
            _ptr(admission), _ptr(scale), _ptr(idx), _ptr(valid), _ptr(gains), _ptr(out),
            _ptr(streams), _ptr(lse), _stream(dev),
        )
    N.check(st, "read_fwd")
    return out, streams, lse


def _wide_read_inputs(query, keys, writes, next_writes, cocktail, bank_cocktail, key_bias,
                      admission, idx, valid):
    if query.dtype != torch.bfloat16:
        raise TypeError(f"dabsn_b200: states wider than {NARROW_READ_MAX_H} units are read in "
                        "bfloat16 only (use autocast)")
    bf = torch.bfloat16
    big = [t.to(bf).contiguous() for t in (query, keys, writes, next_writes, cocktail,
                                             bank_cocktail)]
    small = [t.to(torch.float32).contiguous() for t in (key_bias, admission)]
    return big, small, idx.to(torch.int64).contiguous(), valid.to(torch.bool).contiguous()


def _read_wide_forward(query, keys, writes, next_writes, cocktail, bank_cocktail, key_bias,
                       admission, scale, idx, valid, gains, mode, total_steps):
    dev = query.device
    B, T, H = query.shape
    Nb = keys.shape[1]
    big, small, idx, valid = _wide_read_inputs(query, keys, writes, next_writes, cocktail,
                                               bank_cocktail, key_bias, admission, idx, valid)
    lib = N.load()
    ld = int(lib.dabsn_read_wide_ld(max(Nb, 1)))
    out = torch.empty((B, T, H), device=dev, dtype=torch.bfloat16)
    compat = torch.empty((B, T, ld), device=dev, dtype=torch.bfloat16)
    lse = torch.empty((B, T, 3), device=dev, dtype=torch.float32)
    if Nb == 0 or T == 0 or B == 0:
        out.zero_()
        lse.fill_(float("inf"))
        return out, compat, lse
    ws = torch.empty(int(lib.dabsn_read_wide_fwd_workspace(B, T, Nb)), device=dev,
                     dtype=torch.uint8)
    with torch.cuda.device(dev), _timed("read_fwd", dev, launches=4):
        st = lib.dabsn_read_wide_fwd(
            B, T, Nb, H, mode, total_steps, *[_ptr(t) for t in big], *[_ptr(t) for t in small],
            _ptr(scale), _ptr(idx), _ptr(valid), _ptr(gains), _ptr(out), _ptr(compat), _ptr(lse),
            _ptr(ws), ws.numel(), _stream(dev),
        )
    N.check(st, "read_wide_fwd")
    return out, compat, lse


def read_backward(
    query: Tensor, keys: Tensor, writes: Tensor, next_writes: Tensor, cocktail: Tensor,
    bank_cocktail: Tensor, key_bias: Tensor, admission: Tensor, scale: Tensor, idx: Tensor,
    valid: Tensor, gains: Tensor, mode: int, total_steps: int, streams: Tensor, lse: Tensor,
    gout: Tensor,
):
    """Returns (dq, dcocktail, dkeys, dwrites, dnext, dbias, dbank_cocktail,
    d scale, d gains[4])."""
    dev = _require_cuda(query)
    B, T, H = query.shape
    Nb = keys.shape[1]
    if H > NARROW_READ_MAX_H:
        return _read_wide_backward(query, keys, writes, next_writes, cocktail, bank_cocktail,
                                   key_bias, admission, scale, idx, valid, gains, mode,
                                   total_steps, streams, lse, gout)
    dt = query.dtype
    code = act_code(dt)
    key_bias = key_bias.to(dt).contiguous()
    admission = admission.to(dt).contiguous()
    go = gout.detach().float().contiguous()
    u3 = torch.empty((B, T, 3), device=dev, dtype=torch.float32)
    dq = torch.empty((B, T, H), device=dev, dtype=dt)
    dcq = torch.empty((B, T, 4), device=dev, dtype=torch.float32)
    dk = torch.empty((B, Nb, H), device=dev, dtype=dt)
    dv = torch.empty_like(dk)
    dn = torch.empty_like(dk)
    db = torch.empty((B, Nb), device=dev, dtype=torch.float32)
    dck = torch.empty((B, Nb, 4), device=dev, dtype=torch.float32)
    nqt = (T + 31) // 32
    partial = torch.empty((B, nqt, 2), device=dev, dtype=torch.float32)
    if Nb == 0 or T == 0 or B == 0:
        for t in (u3, dq, dcq, dk, dv, dn, db, dck, partial):
            t.zero_()
    else:
        lib = N.load()
        with torch.cuda.device(dev), _timed("read_bwd", dev, launches=2):
            st = lib.dabsn_read_bwd(
                code, B, T, Nb, H, mode, total_steps, _ptr(query), _ptr(keys), _ptr(writes),
                _ptr(next_writes), _ptr(cocktail), _ptr(bank_cocktail), _ptr(key_bias),
                _ptr(admission), _ptr(scale), _ptr(idx), _ptr(valid), _ptr(gains),
                _ptr(streams), _ptr(lse), _ptr(go), _ptr(u3), _ptr(dq), _ptr(dcq), _ptr(dk),
                _ptr(dv), _ptr(dn), _ptr(db), _ptr(dck), _ptr(partial), _stream(dev),
            )
        N.check(st, "read_bwd")
    psum = partial.sum(dim=(0, 1))
    usum = u3.sum(dim=(0, 1))
    dgains = torch.stack([usum[0], usum[1], usum[2], psum[1]])
    return dq, dcq, dk, dv, dn, db, dck, psum[0], dgains


def _read_wide_backward(query, keys, writes, next_writes, cocktail, bank_cocktail, key_bias,
                        admission, scale, idx, valid, gains, mode, total_steps, compat, lse, gout):
    dev = query.device
    B, T, H = query.shape
    Nb = keys.shape[1]
    big, small, idx, valid = _wide_read_inputs(query, keys, writes, next_writes, cocktail,
                                               bank_cocktail, key_bias, admission, idx, valid)
    go = gout.detach().to(torch.bfloat16).contiguous()
    bf = torch.bfloat16
    u3 = torch.zeros((B, T, 3), device=dev, dtype=torch.float32)
    # dq, dk, dv, dn are GEMM outputs whose every tile the GEMM writes (zeros
    # for a tile with no live slice); the small accumulators start at zero
    dq = torch.empty((B, T, H), device=dev, dtype=bf)
    dcq = torch.zeros((B, T, 4), device=dev, dtype=torch.float32)
    dk = torch.empty((B, Nb, H), device=dev, dtype=bf)
    dv = torch.empty_like(dk)
    dn = torch.empty_like(dk)
    db = torch.zeros((B, Nb), device=dev, dtype=torch.float32)
    dck = torch.zeros((B, Nb, 4), device=dev, dtype=torch.float32)
    rowpart = torch.zeros((B, T, 2), device=dev, dtype=torch.float32)
    if Nb > 0 and T > 0 and B > 0:
        lib = N.load()
        ws = torch.empty(int(lib.dabsn_read_wide_bwd_workspace(B, T, Nb)), device=dev,
                         dtype=torch.uint8)
        with torch.cuda.device(dev), _timed("read_bwd", dev, launches=6):
            st = lib.dabsn_read_wide_bwd(
                B, T, Nb, H, mode, total_steps, *[_ptr(t) for t in big],
                *[_ptr(t) for t in small], _ptr(scale), _ptr(idx), _ptr(valid), _ptr(gains),
                _ptr(compat), _ptr(lse), _ptr(go), _ptr(u3), _ptr(dq), _ptr(dcq), _ptr(dk),
                _ptr(dv), _ptr(dn), _ptr(db), _ptr(dck), _ptr(rowpart), _ptr(ws), ws.numel(),
                _stream(dev),
            )
        N.check(st, "read_wide_bwd")
    else:
        for t in (dq, dk, dv, dn):
            t.zero_()
    usum = u3.sum(dim=(0, 1))
    rsum = rowpart.sum(dim=(0, 1))
    dgains = torch.stack([usum[0], usum[1], usum[2], rsum[1]])
    return dq, dcq, dk, dv, dn, db, dck, rsum[0], dgains


# ---------------------------------------------------------------------------
# Read admission and admitted bank (read.py:152-303 semantics)
# ---------------------------------------------------------------------------
def admission_forward(expression: Tensor, novelty: Tensor, plasticity: Tensor, energy: Tensor,
                      saturation: Tensor, params: Tensor, window: Tensor, mode: int,
                      query_dtype: torch.dtype = torch.float32):
    """Token statistics, membership and the stable partition of positions.

    Returns ``(query [B,T,H] in query_dtype, key_bias [B,T], admission [B,T],
    cocktail [B,T,4], stats [B,T,8], order int64 [B,T], counts int64 [B],
    inv int32 [B,T])``."""
    dev = _require_cuda(expression)
    B, T, H = expression.shape
    dt = expression.dtype
    code = act_code(dt)
    tapes = [t.detach().to(dt).contiguous() for t in (expression, novelty, plasticity, energy,
                                                      saturation)]
    f32 = torch.float32
    query = torch.empty((B, T, H), device=dev, dtype=query_dtype)
    kb = torch.empty((B, T), device=dev, dtype=f32)
    adm = torch.empty((B, T), device=dev, dtype=f32)
    cocktail = torch.empty((B, T, 4), device=dev, dtype=f32)
    stats = torch.empty((B, T, 8), device=dev, dtype=f32)
    order = torch.empty((B, T), device=dev, dtype=torch.int64)
    counts = torch.empty((B,), device=dev, dtype=torch.int64)
    inv = torch.empty((B, T), device=dev, dtype=torch.int32)
    lib = N.load()
    with torch.cuda.device(dev), _timed("admission_fwd", dev, launches=2):
        st = lib.dabsn_admission_fwd(
            code, B, T, H, mode, *[_ptr(t) for t in tapes], _ptr(params), _ptr(window),
            act_code(query_dtype), _ptr(query), _ptr(kb), _ptr(adm), _ptr(cocktail),
            _ptr(stats), _ptr(order), _ptr(counts), _ptr(inv), _stream(dev),
        )
    N.check(st, "admission_fwd")
    return query, kb, adm, cocktail, stats, order, counts, inv


def bank_gather(write: Tensor, kb: Tensor, adm: Tensor, cocktail: Tensor, order: Tensor,
                counts: Tensor, n: int, key_dtype: torch.dtype = torch.float32):
    """The first ``n`` bank entries: ``(bank_writes, bank_keys in key_dtype, next_writes,
    bank_cocktail, bank_bias, bank_admission, bank_idx int64, bank_valid bool,
    key_norm)``."""
    dev = _require_cuda(write)
    B, T, H = write.shape
    dt = write.dtype
    write = write.detach().contiguous()
    f32 = torch.float32
    bw = torch.empty((B, n, H), device=dev, dtype=dt)
    bk = torch.empty((B, n, H), device=dev, dtype=key_dtype)
    nw = torch.empty((B, n, H), device=dev, dtype=dt)
    bc = torch.empty((B, n, 4), device=dev, dtype=f32)
    bb = torch.empty((B, n), device=dev, dtype=f32)
    ba = torch.empty((B, n), device=dev, dtype=f32)
    bi = torch.empty((B, n), device=dev, dtype=torch.int64)
    bv = torch.empty((B, n), device=dev, dtype=torch.bool)
    kn = torch.empty((B, n), device=dev, dtype=f32)
    lib = N.load()
    with torch.cuda.device(dev), _timed("bank_gather", dev):
        st = lib.dabsn_bank_gather(
            act_code(dt), B, T, H, n, _ptr(write), _ptr(kb), _ptr(adm), _ptr(cocktail),
            _ptr(order), _ptr(counts), _ptr(bw), act_code(key_dtype), _ptr(bk), _ptr(nw),
            _ptr(bc), _ptr(bb), _ptr(ba), _ptr(bi), _ptr(bv), _ptr(kn), _stream(dev),
        )
    N.check(st, "bank_gather")
    return bw, bk, nw, bc, bb, ba, bi, bv, kn


def admission_backward(expression: Tensor, write: Tensor, stats: Tensor, cocktail: Tensor,
                       params: Tensor, inv: Tensor, key_norm: Tensor, n: int, grads):
    """Gradients of the token statistics and the bank gathers.

    ``grads`` = (d query, d cocktail, d keys, d writes, d next writes,
    d bank cocktail, d bank bias, d bank admission), any None.  The four
    [.,.,H] gradients are read in BF16 when the activations are BF16 and all
    of them arrive in BF16, else in FP32; the rest in FP32.  Query and keys
    are recomputed from ``expression``, ``write``, ``stats`` and ``key_norm``.
    Returns ``(d expression, d write, d_means [B,T,4] (per-unit gradient of
    plasticity, novelty, energy, saturation), param_part [B,T,8])``."""
    dev = _require_cuda(expression)
    B, T, H = expression.shape
    dt = expression.dtype
    wide = [grads[i] for i in (0, 2, 3, 4)]
    gdt = (torch.bfloat16 if dt == torch.bfloat16
           and all(g is None or g.dtype == torch.bfloat16 for g in wide) else torch.float32)
    gs = [None if g is None else g.detach().to(gdt if i in (0, 2, 3, 4) else torch.float32)
          .contiguous() for i, g in enumerate(grads)]
    d_expr = torch.empty((B, T, H), device=dev, dtype=dt)
    d_write = torch.empty((B, T, H), device=dev, dtype=write.dtype)
    d_means = torch.empty((B, T, 4), device=dev, dtype=torch.float32)
    part = torch.empty((B, T, 8), device=dev, dtype=torch.float32)
    if write.dtype != dt:
        raise TypeError("admission backward: expression and write must share a dtype")
    lib = N.load()
    with torch.cuda.device(dev), _timed("admission_bwd", dev):
        st = lib.dabsn_admission_bwd(
            act_code(dt), B, T, H, n, _ptr(expression), _ptr(write), _ptr(stats), _ptr(cocktail),
            _ptr(params), _ptr(inv), _ptr(key_norm), act_code(gdt), _ptr(gs[0]), _ptr(gs[1]),
            _ptr(gs[2]), _ptr(gs[3]), _ptr(gs[4]), _ptr(gs[5]), _ptr(gs[6]), _ptr(gs[7]),
            _ptr(d_expr), _ptr(d_write), _ptr(d_means), _ptr(part), _stream(dev),
        )
    N.check(st, "admission_bwd")
    return d_expr, d_write, d_means, part


# ---------------------------------------------------------------------------
# Primitives: permanent delta scan, local field gather
# ---------------------------------------------------------------------------
def permanent_delta_forward(k: Tensor, v: Tensor, beta: Tensor, ckpt: Tensor | None = None) -> Tensor:
    """``dabsn::permanent_delta_scan`` forward: reconstructions [B,T,h]."""
    dev = _require_cuda(k)
    B, T, h = k.shape
    dt = k.dtype
    k, v, beta = (x.detach().to(dt).contiguous() for x in (k, v, beta))
    out = torch.empty((B, T, h), device=dev, dtype=dt)
    if T == 0 or B == 0:
        return out
    lib = N.load()
    with torch.cuda.device(dev), _timed("permanent_delta_fwd", dev):
        st = lib.dabsn_permanent_delta_fwd(act_code(dt), B, T, h, _ptr(k), _ptr(v), _ptr(beta),
                                           _ptr(out), _ptr(ckpt), _stream(dev))
    N.check(st, "permanent_delta_fwd")
    return out


def permanent_delta_backward(k: Tensor, v: Tensor, beta: Tensor, grad_out: Tensor):
    """Gradients (dk, dv, dbeta): the forward is re-run storing the state every
    64 steps, then the reverse walks back from the checkpoints."""
    dev = _require_cuda(k)
    B, T, h = k.shape
    dt = k.dtype
    k, v, beta = (x.detach().to(dt).contiguous() for x in (k, v, beta))
    dk, dv, dbeta = torch.zeros_like(k), torch.zeros_like(v), torch.zeros_like(beta)
    if T == 0 or B == 0 or grad_out is None:
        return dk, dv, dbeta
    lib = N.load()
    ckpt = torch.empty(int(lib.dabsn_delta_ckpt_floats(B, T, h)), device=dev, dtype=torch.float32)
    recon = permanent_delta_forward(k, v, beta, ckpt)
    g = grad_out.detach().float().contiguous()
    with torch.cuda.device(dev), _timed("permanent_delta_bwd", dev):
        st = lib.dabsn_permanent_delta_bwd(act_code(dt), B, T, h, _ptr(k), _ptr(v), _ptr(beta),
                                           _ptr(recon), _ptr(g), _ptr(ckpt), _ptr(dk), _ptr(dv),
                                           _ptr(dbeta), _stream(dev))
    N.check(st, "permanent_delta_bwd")
    return dk, dv, dbeta


def local_field_gather(x: Tensor, patch: Tensor) -> Tensor:
    """``dabsn::local_field_gather``: x [B,C,D], patch [N,K] -> [B,N,K,D]."""
    dev = _require_cuda(x)
    B, C, D = x.shape
    Np, K = patch.shape
    x = x.detach().contiguous()
    p = patch.detach().to(device=dev, dtype=torch.int64).contiguous()
    out = torch.empty((B, Np, K, D), device=dev, dtype=x.dtype)
    lib = N.load()
    with torch.cuda.device(dev), _timed("local_field_gather", dev):
        st = lib.dabsn_local_field_gather(act_code(x.dtype), B, C, Np, K, D, _ptr(x), _ptr(p),
                                          _ptr(out), _stream(dev))
    N.check(st, "local_field_gather")
    return out


def local_field_scatter(grad_out: Tensor, patch: Tensor, cells: int) -> Tensor:
    """Reverse of the gather: per source cell, the sum of the gradients of the
    slots that read it (inverse index built here; no atomics)."""
    dev = _require_cuda(grad_out)
    B, Np, K, D = grad_out.shape
    g = grad_out.detach().contiguous()
    flat = patch.detach().to(device=dev, dtype=torch.int64).reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=cells)
    offsets = torch.zeros(cells + 1, device=dev, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    gx = torch.empty((B, cells, D), device=dev, dtype=g.dtype)
    lib = N.load()
    with torch.cuda.device(dev), _timed("local_field_scatter", dev):
        st = lib.dabsn_local_field_scatter(act_code(g.dtype), B, cells, Np, K, D, _ptr(g),
                                           _ptr(order), _ptr(offsets), _ptr(gx), _stream(dev))
    N.check(st, "local_field_scatter")
    return gx


def read_out_grad_prep(grad: Tensor, long_channel: Tensor, long_gain: Tensor):
    """One pass over the read output projection's FP32 gradient [R, H]:
    returns (grad BF16 [R, H], dlong FP32 [R, H] = long_gain * grad, bias
    gradient FP32 [H] (column sums of the BF16 copy), gain gradient FP32 []
    (sum of grad * long))."""
    dev = _require_cuda(grad)
    R, H = grad.shape
    lib = N.load()
    nb = int(lib.dabsn_glue_blocks(R))
    gb = torch.empty((R, H), device=dev, dtype=torch.bfloat16)
    dlong = torch.empty((R, H), device=dev, dtype=torch.float32)
    colpart = torch.empty((nb, H), device=dev, dtype=torch.float32)
    dotpart = torch.empty(nb, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev), _timed("read_out_glue", dev):
        st = lib.dabsn_read_out_grad_prep(R, H, _ptr(grad), _ptr(long_channel), _ptr(long_gain),
                                          _ptr(gb), _ptr(dlong), _ptr(colpart), _ptr(dotpart),
                                          _stream(dev))
    N.check(st, "read_out_grad_prep")
    return gb, dlong, colpart.sum(dim=0), dotpart.sum()


def colsum_bf16(x: Tensor) -> Tensor:
    """Column sums (FP32 [H]) of a BF16 [R, H] matrix with H a multiple of 8."""
    dev = _require_cuda(x)
    R, H = x.shape
    lib = N.load()
    colpart = torch.empty((int(lib.dabsn_glue_blocks(R)), H), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        st = lib.dabsn_colsum_bf16(R, H, _ptr(x), _ptr(colpart), _stream(dev))
    N.check(st, "colsum_bf16")
    return colpart.sum(dim=0)


# ---------------------------------------------------------------------------
# Readout + cross-entropy (runtime/loss.py:52-231 semantics)
# ---------------------------------------------------------------------------
def linear_ce_forward(hidden: Tensor, weight: Tensor, bias: Tensor | None, targets: Tensor,
                      ignore_index: int, round_bf16: bool):
    """Returns (lse [rows] FP32, target logit [rows] FP32)."""
    dev = _require_cuda(hidden)
    rows, D = hidden.shape
    V = weight.shape[0]
    lib = N.load()
    lse = torch.empty(rows, device=dev, dtype=torch.float32)
    tgt = torch.zeros(rows, device=dev, dtype=torch.float32)
    ws = torch.empty(int(lib.dabsn_linear_ce_workspace_floats(rows, V)), device=dev,
                     dtype=torch.float32)
    with torch.cuda.device(dev), _timed("linear_ce_fwd", dev, launches=2):
        st = lib.dabsn_linear_ce_fwd(rows, V, D, _ptr(hidden), _ptr(weight), _ptr(bias),
                                     _ptr(targets), ignore_index, int(round_bf16), _ptr(lse),
                                     _ptr(tgt), _ptr(ws), _stream(dev))
    N.check(st, "linear_ce_fwd")
    return lse, tgt


def linear_ce_backward(hidden: Tensor, weight: Tensor, bias: Tensor | None, targets: Tensor,
                       ignore_index: int, round_bf16: bool, lse: Tensor, scale: Tensor,
                       row_chunk: int | None = None):
    """Returns (dhidden BF16 [rows,D], dweight FP32 [V,D], dbias FP32 [V] or None).

    The reverse runs over chunks of ``row_chunk`` rows (all rows when None):
    each chunk's dlogits [chunk, ld] BF16 live in one reused workspace and
    dweight accumulates across chunks in FP32."""
    dev = _require_cuda(hidden)
    rows, D = hidden.shape
    V = weight.shape[0]
    lib = N.load()
    ld = int(lib.dabsn_linear_ce_ld(V))
    chunk = rows if row_chunk is None else max(1, min(int(row_chunk), rows))
    dlogits = torch.empty((chunk, ld), device=dev, dtype=torch.bfloat16)
    dh = torch.empty((rows, D), device=dev, dtype=torch.bfloat16)
    dw = torch.empty((V, D), device=dev, dtype=torch.float32)
    db = torch.zeros(V, device=dev, dtype=torch.float32) if bias is not None else None
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        dl = dlogits[: r1 - r0]
        with torch.cuda.device(dev), _timed("linear_ce_bwd", dev, launches=3):
            st = lib.dabsn_linear_ce_bwd(
                r1 - r0, V, D, _ptr(hidden[r0:r1]), _ptr(weight), _ptr(bias),
                _ptr(targets[r0:r1]), ignore_index, int(round_bf16), _ptr(lse[r0:r1]),
                _ptr(scale), _ptr(dl), _ptr(dh[r0:r1]), _ptr(dw), int(r0 > 0), _stream(dev))
        N.check(st, "linear_ce_bwd")
        if db is not None:
            db += dl[:, :V].float().sum(dim=0)
    return dh, dw, db


# ---------------------------------------------------------------------------
# Cross-entropy over materialised logits (runtime/loss.py:187-231 semantics)
# ---------------------------------------------------------------------------
def ce_logits_forward(logits: Tensor, targets: Tensor, ignore_index: int):
    """logits [rows, V] (FP32/BF16, rows contiguous), targets [rows] int64.
    Returns (lse [rows] FP32, target logit [rows] FP32)."""
    dev = _require_cuda(logits)
    rows, V = logits.shape
    lse = torch.empty(rows, device=dev, dtype=torch.float32)
    tgt = torch.empty(rows, device=dev, dtype=torch.float32)
    lib = N.load()
    with torch.cuda.device(dev), _timed("ce_logits_fwd", dev):
        st = lib.dabsn_ce_logits_fwd(act_code(logits.dtype), rows, V, logits.stride(0),
                                     _ptr(logits), _ptr(targets), int(ignore_index), _ptr(lse),
                                     _ptr(tgt), _stream(dev))
    N.check(st, "ce_logits_fwd")
    return lse, tgt


def ce_logits_backward(logits: Tensor, targets: Tensor, ignore_index: int, lse: Tensor,
                       scale: Tensor) -> Tensor:
    """dlogits [rows, V] in the logits' dtype: scale (softmax - onehot)."""
    dev = _require_cuda(logits)
    rows, V = logits.shape
    dl = torch.empty((rows, V), device=dev, dtype=logits.dtype)
    lib = N.load()
    with torch.cuda.device(dev), _timed("ce_logits_bwd", dev):
        st = lib.dabsn_ce_logits_bwd(act_code(logits.dtype), rows, V, logits.stride(0),
                                     _ptr(logits), _ptr(targets), int(ignore_index), _ptr(lse),
                                     _ptr(scale), _ptr(dl), _stream(dev))
    N.check(st, "ce_logits_bwd")
    return dl


# ---------------------------------------------------------------------------
# Dense products around the scan on the tcgen05 GEMM (BF16)
# ---------------------------------------------------------------------------
def input_proj_forward(x: Tensor, W: Tensor, Wg: Tensor, bias_g: Tensor | None):
    """x [M, D] BF16 (rows contiguous), W / Wg [H, D] BF16, bias FP32 [H] or
    None -> (Wx, Wgx) [M, H] BF16."""
    dev = _require_cuda(x, W, Wg)
    M, D = x.shape
    H = W.shape[0]
    wx = torch.empty((M, H), device=dev, dtype=torch.bfloat16)
    wgx = torch.empty_like(wx)
    lib = N.load()
    with torch.cuda.device(dev), _timed("input_proj_fwd", dev):
        st = lib.dabsn_input_proj_fwd(M, D, H, _ptr(x), x.stride(0), _ptr(W), _ptr(Wg),
                                      _ptr(bias_g), _ptr(wx), _ptr(wgx), _stream(dev))
    N.check(st, "input_proj_fwd")
    return wx, wgx


def input_proj_backward(x: Tensor, W: Tensor, Wg: Tensor, gWx: Tensor, gWgx: Tensor,
                        need_dx: bool):
    """-> (dx [M, D] or None, dW [H, D], dWg [H, D]), all BF16."""
    dev = _require_cuda(x, W, Wg, gWx, gWgx)
    M, D = x.shape
    H = W.shape[0]
    dx = torch.empty((M, D), device=dev, dtype=torch.bfloat16) if need_dx else None
    dW = torch.empty((H, D), device=dev, dtype=torch.bfloat16)
    dWg = torch.empty_like(dW)
    lib = N.load()
    with torch.cuda.device(dev), _timed("input_proj_bwd", dev, launches=2 if need_dx else 1):
        st = lib.dabsn_input_proj_bwd(M, D, H, _ptr(x), x.stride(0), _ptr(W), _ptr(Wg), _ptr(gWx),
                                      _ptr(gWgx), _ptr(dx), _ptr(dW), _ptr(dWg), _stream(dev))
    N.check(st, "input_proj_bwd")
    return dx, dW, dWg


def rec_grad(y: Tensor, gWgx: Tensor, day: Tensor):
    """y [M, H] BF16 (row stride free), dWgx / dA [M, H] BF16 -> (grad Ug,
    grad A) [H, H] BF16."""
    dev = _require_cuda(y, gWgx, day)
    M, H = gWgx.shape
    gUg = torch.empty((H, H), device=dev, dtype=torch.bfloat16)
    gA = torch.empty_like(gUg)
    lib = N.load()
    with torch.cuda.device(dev), _timed("rec_grad", dev):
        st = lib.dabsn_rec_grad(M, H, _ptr(y), y.stride(0), _ptr(gWgx), _ptr(day), _ptr(gUg),
                                _ptr(gA), _stream(dev))
    N.check(st, "rec_grad")
    return gUg, gA


def _rows(t: Tensor) -> Tensor:
    """[..., H] with unit inner stride as a [rows, H] view (row stride kept)."""
    return t.reshape(-1, t.shape[-1])


def read_out_forward(y: Tensor, bud: Tensor, ret: Tensor, W: Tensor, bias: Tensor | None,
                     addend: Tensor, add_scale: Tensor) -> Tensor:
    """FP32 [rows, H] = bf16(cat[y, b, r] W^T + bias) + add_scale * addend."""
    dev = _require_cuda(y, bud, ret, W, addend)
    y2, b2, r2 = _rows(y), _rows(bud), _rows(ret)
    M, H = y2.shape
    out = torch.empty((M, H), device=dev, dtype=torch.float32)
    lib = N.load()
    with torch.cuda.device(dev), _timed("read_out_fwd", dev):
        st = lib.dabsn_read_out_fwd(M, H, _ptr(y2), y2.stride(0), _ptr(b2), b2.stride(0), _ptr(r2),
                                    r2.stride(0), _ptr(W), _ptr(bias), _ptr(addend),
                                    _ptr(add_scale), _ptr(out), _stream(dev))
    N.check(st, "read_out_fwd")
    return out


def read_out_backward(y: Tensor, bud: Tensor, ret: Tensor, W: Tensor, gout: Tensor):
    """-> (dy, db, dr [rows, H] BF16, dW [H, 3H] BF16) for gout [rows, H] BF16."""
    dev = _require_cuda(y, bud, ret, W, gout)
    y2, b2, r2 = _rows(y), _rows(bud), _rows(ret)
    M, H = y2.shape
    dy = torch.empty((M, H), device=dev, dtype=torch.bfloat16)
    db = torch.empty_like(dy)
    dr = torch.empty_like(dy)
    dW = torch.empty((H, 3 * H), device=dev, dtype=torch.bfloat16)
    lib = N.load()
    with torch.cuda.device(dev), _timed("read_out_bwd", dev, launches=2):
        st = lib.dabsn_read_out_bwd(M, H, _ptr(y2), y2.stride(0), _ptr(b2), b2.stride(0), _ptr(r2),
                                    r2.stride(0), _ptr(W), _ptr(gout), _ptr(dy), _ptr(db), _ptr(dr),
                                    _ptr(dW), _stream(dev))
    N.check(st, "read_out_bwd")
    return dy, db, dr, dW

