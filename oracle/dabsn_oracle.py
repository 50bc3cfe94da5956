"""CPU oracle for the DABSN scan + read hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the ``dabsn_b200`` package imports this
module: it is the checker that ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` compare the CUDA kernels against.  It is a
plain, loop-based PyTorch restatement of the reference mathematics, written to
run in float64 (or float32) on the CPU; gradients come from PyTorch autograd
through these loops, so the oracle's backward is independent of the analytic
reverse scans in the reference and in the CUDA kernels.

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference
package itself, records its outputs and gradients on seeded inputs into
``tests/golden/*.pt``, and ``tests/test_oracle_golden.py`` checks every function
below against those fixtures.

Reference citations are ``path:line`` inside the reference project
(BleedingXiko/dabsn v0.1.8).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

CORE_PARAM_NAMES = (
    "beta",
    "log_kappa",
    "logit_recover",
    "k_s",
    "k_y",
    "k_b",
    "k_n",
    "k_bias",
    "r_s",
    "r_y",
    "r_b",
    "r_n",
    "r_bias",
    "logit_c_decay",
    "k_c",
    "r_c",
)
CORE_SCALAR_NAMES = ("logit_alpha", "log_lambda", "logit_c_suppress")


class _HardsigmoidTapeMask(torch.autograd.Function):
    """hardsigmoid whose derivative mask is taken from the gate rounded to the
    tape dtype: the reference's reverse scan reads the stored gate tape
    (batched_runtime.py:539, mask ``(gate > 0) & (gate < 1)`` at :392),
    so with BF16 tapes a gate of 0.999 (stored as 1.0) has zero derivative."""

    @staticmethod
    def forward(ctx, x, tape_dtype):
        s = F.hardsigmoid(x)
        st = s.to(tape_dtype).to(s.dtype)
        ctx.save_for_backward(((st > 0) & (st < 1)).to(s.dtype))
        return s

    @staticmethod
    def backward(ctx, g):
        (mask,) = ctx.saved_tensors
        return g * mask / 6.0, None


def _round(x: Tensor, dtype: torch.dtype | None) -> Tensor:
    """Round through ``dtype`` and back (models an activation-dtype store)."""
    if dtype is None or dtype == x.dtype:
        return x
    return x.to(dtype).to(x.dtype)


# ---------------------------------------------------------------------------
# A.1  core recurrence  (src/dabsn/core.py:171-221,
#                        src/dabsn/kernels/batched_runtime.py:38-158)
# ---------------------------------------------------------------------------
def core_scan(
    Wx: Tensor,
    Wgx: Tensor,
    Ug: Tensor,
    A: Tensor,
    beta: Tensor,
    log_kappa: Tensor,
    logit_recover: Tensor,
    k_s: Tensor,
    k_y: Tensor,
    k_b: Tensor,
    k_n: Tensor,
    k_bias: Tensor,
    r_s: Tensor,
    r_y: Tensor,
    r_b: Tensor,
    r_n: Tensor,
    r_bias: Tensor,
    logit_c_decay: Tensor,
    k_c: Tensor,
    r_c: Tensor,
    logit_alpha: Tensor,
    log_lambda: Tensor,
    logit_c_suppress: Tensor,
    initial_b: Tensor,
    initial_e: Tensor,
    initial_c: Tensor,
    *,
    gemm_dtype: torch.dtype | None = None,
    state_dtype: torch.dtype | None = None,
) -> tuple[Tensor, ...]:
    """The registered ``dabsn::core_scan_batched`` operator, restated.

    Same 26 inputs and 11 outputs as the reference schema
    (batched_runtime.py:1507-1566): ``U=[y,b'] [B,T,2H]``, novelty, plasticity,
    expression, write, energy (pre-update), saturation (post-update), gate, and
    the final budget/energy/saturation.  By default the state chain runs in
    the promoted input dtype (exact mathematics, e.g. float64).  With
    ``state_dtype=torch.float32`` it follows the reference's precision policy:
    an FP32 state chain whatever the activation dtype, and the recurrent
    product formed in the activation dtype (batched_runtime.py:168-186,
    1123-1131).  ``gemm_dtype`` models the
    reference's reduced-precision recurrent product: ``y`` and ``[Ug;A]`` are
    rounded to it and so is the product (batched_runtime.py:96-101, 1123).
    """
    B, T, H = Wx.shape
    if state_dtype is None:
        dt = torch.promote_types(Wx.dtype, initial_b.dtype)
        dt = torch.promote_types(dt, Ug.dtype)
    else:
        dt = state_dtype
    act = Wx.dtype
    rec = torch.cat([Ug, A], dim=0).to(act if state_dtype is not None else dt)
    rec = _round(rec, gemm_dtype)
    b = initial_b.to(dt)
    e = initial_e.to(dt)
    c = initial_c.to(dt)
    alpha = torch.sigmoid(logit_alpha.to(dt))
    lam = F.softplus(log_lambda.to(dt))
    suppress = torch.sigmoid(logit_c_suppress.to(dt))
    decay = torch.sigmoid(logit_c_decay.to(dt))
    kappa = F.softplus(log_kappa.to(dt))
    recover = torch.sigmoid(logit_recover.to(dt))
    outs: dict[str, list[Tensor]] = {k: [] for k in ("y", "b", "n", "p", "a", "w", "e", "c", "s")}
    for t in range(T):
        y = torch.tanh(Wx[:, t].to(dt) + b)
        prod = _round(y.to(rec.dtype), gemm_dtype) @ rec.T
        prod = _round(prod, gemm_dtype).to(dt)
        g_r, a = prod[:, :H], prod[:, H:]
        if gemm_dtype is None:
            s = F.hardsigmoid(Wgx[:, t].to(dt) + g_r)
        else:
            s = _HardsigmoidTapeMask.apply(Wgx[:, t].to(dt) + g_r, gemm_dtype)
        n = torch.tanh((a - b).abs())
        c = decay * c + (1.0 - decay) * (n * (1.0 - e))
        n_eff = n * (1.0 - suppress * c)
        tb = torch.tanh(b)
        k_sig = k_s * s + k_y * y + k_b * tb + k_n * n_eff + k_bias + k_c * c
        r_sig = r_s * s + r_y * y + r_b * tb + r_n * n_eff + r_bias + r_c * c
        write_cost = kappa * torch.exp(0.5 * torch.tanh(k_sig))
        recovery = torch.clamp(recover * torch.exp(0.5 * torch.tanh(r_sig)), 0.0, 1.0)
        p = s * e
        w = p * a
        outs["e"].append(e)
        b = (1.0 - alpha) * b + beta + lam * w
        e = torch.clamp(e + recovery * (1.0 - e) - write_cost * p, 0.0, 1.0)
        outs["y"].append(y)
        outs["b"].append(b)
        outs["n"].append(n)
        outs["p"].append(p)
        outs["a"].append(a)
        outs["w"].append(w)
        outs["c"].append(c)
        outs["s"].append(s)
    st = {k: torch.stack(v, dim=1) for k, v in outs.items()}
    U = torch.cat([st["y"], st["b"]], dim=-1)
    res = (U, st["n"], st["p"], st["a"], st["w"], st["e"], st["c"], st["s"], b, e, c)
    if state_dtype is not None:
        res = tuple(r.to(act) for r in res)
    return res


# ---------------------------------------------------------------------------
# A.2  three-way admitted read  (src/dabsn/kernels/compact_admitted.py:16-80,
#                                src/dabsn/kernels/admitted.py:16-64)
# ---------------------------------------------------------------------------
def three_way_read(
    query: Tensor,
    bank_keys: Tensor,
    bank_writes: Tensor,
    next_writes: Tensor,
    cocktail: Tensor,
    bank_cocktail: Tensor,
    bank_key_bias: Tensor,
    bank_admission: Tensor,
    scale: Tensor,
    bank_idx: Tensor,
    bank_valid: Tensor,
    *,
    mode: str,
    short_gain: Tensor,
    pad_gain: Tensor,
    induct_gain: Tensor,
    cocktail_gain: Tensor,
    total_steps: int | None = None,
    score_dtype: torch.dtype | None = None,
) -> Tensor:
    """Dense masked restatement of the exact admitted read.

    ``S = scale*q.k + key_bias + admission``; ``P = S + cocktail_gain*cc``;
    short/permanent read ``bank_writes`` under the causal mask
    ``idx <= t`` (seq) or all valid entries (field); induction reads
    ``next_writes`` under ``idx < t`` (seq) or ``idx < T-1`` (field).  Rows with
    no eligible entry read zero.  ``score_dtype=torch.float32`` follows the
    reference's precision policy (scores, softmax and the gain-weighted sum
    in FP32, value products in the activation dtype;
    compact_admitted.py:40-80).
    """
    Bsz, T, H = query.shape
    N = bank_keys.shape[1]
    full = T if total_steps is None else int(total_steps)
    act = query.dtype
    dt = act if score_dtype is None else score_dtype
    scores = scale.to(dt) * torch.einsum("bth,bnh->btn", query, bank_keys.to(act)).to(dt)
    short = scores + (bank_key_bias.to(dt) + bank_admission.to(dt)).unsqueeze(1)
    cc = torch.einsum("btc,bnc->btn", cocktail.to(dt), bank_cocktail.to(dt))
    perm = short + cocktail_gain.to(dt) * cc
    valid = bank_valid.unsqueeze(1)
    pos = bank_idx.unsqueeze(1)
    if mode == "seq":
        tq = torch.arange(T).view(1, T, 1)
        allow = valid & (pos <= tq)
        induct_allow = valid & (pos < tq)
    elif mode == "field":
        allow = valid.expand(Bsz, T, N)
        induct_allow = (valid & (pos < full - 1)).expand(Bsz, T, N)
    else:
        raise ValueError("mode must be seq or field")

    def read(sc: Tensor, values: Tensor, mask: Tensor) -> Tensor:
        eligible = mask.any(dim=-1, keepdim=True)
        masked = sc.masked_fill(~mask, float("-inf")).masked_fill(~eligible, 0.0)
        weights = torch.softmax(masked, dim=-1)
        weights = torch.where(eligible, weights, torch.zeros_like(weights))
        return (weights.to(act) @ values.to(act)).to(dt)

    out = (
        short_gain.to(dt) * read(short, bank_writes, allow)
        + pad_gain.to(dt) * read(perm, bank_writes, allow)
        + induct_gain.to(dt) * read(short, next_writes, induct_allow)
    )
    return out.to(act)


# ---------------------------------------------------------------------------
# A.3  long-memory channel  (src/dabsn/read.py:577-640,
#                            src/dabsn/kernels/long.py:492-579)
# ---------------------------------------------------------------------------
def long_scan(
    write: Tensor,
    plasticity: Tensor,
    logit_retain: Tensor,
    logit_expect_retain: Tensor,
    logit_retention_decay: Tensor,
    logit_retention_strength: Tensor,
    initial_state: tuple[Tensor, Tensor, Tensor] | None = None,
    *,
    return_final_state: bool = False,
):
    """Expected / retention / long diagonal recurrences, one step at a time."""
    B, T, H = write.shape
    dt = torch.promote_types(write.dtype, logit_retain.dtype)
    if initial_state is None:
        L = torch.zeros(B, H, dtype=dt)
        E = torch.zeros(B, H, dtype=dt)
        Q = torch.ones(B, H, dtype=dt)
    else:
        L, E, Q = (s.to(dt) for s in initial_state)
    R = torch.sigmoid(logit_retain.to(dt))
    re = torch.sigmoid(logit_expect_retain.to(dt))
    rd = torch.sigmoid(logit_retention_decay.to(dt))
    rs = torch.sigmoid(logit_retention_strength.to(dt))
    outs = []
    for t in range(T):
        w = write[:, t].to(dt)
        pe = torch.tanh((w - E).abs())
        sal = plasticity[:, t].to(dt) * pe
        E = re * E + (1.0 - re) * w
        Q = rd * Q + (1.0 - rd) * (1.0 - pe)
        eta = R + (1.0 - R) * rs * Q
        L = eta * L + (1.0 - eta) * (sal * w)
        outs.append(L)
    out = torch.stack(outs, dim=1)
    if return_final_state:
        return out, (L, E, Q)
    return out


# ---------------------------------------------------------------------------
# Admission and bank construction  (src/dabsn/read.py:152-303)
# ---------------------------------------------------------------------------
def admitted_bank(
    expression: Tensor,
    write: Tensor,
    novelty: Tensor,
    plasticity: Tensor,
    energy: Tensor,
    saturation: Tensor,
    read_params: dict[str, Tensor],
    *,
    geometry: str = "seq",
):
    """Admission scores, bank selection and gathered bank tensors.

    Returns a dict with everything :func:`three_way_read` consumes plus the
    bank width ``n_max``.
    """
    Bsz, T, H = expression.shape
    rp = read_params
    query = F.normalize(expression, dim=-1)
    scale = (F.softplus(rp["log_temp"]) + 1.0) * (H**0.5)
    p_mean = plasticity.mean(dim=-1)
    n_mean = novelty.mean(dim=-1)
    e_mean = energy.mean(dim=-1)
    c_mean = saturation.mean(dim=-1)
    key_bias = rp["p_gain"] * torch.log1p(p_mean * H) + rp["novelty_gain"] * n_mean + rp["null_bias"]
    admission = (
        rp["adm_p_gain"] * torch.log1p(p_mean * H)
        + rp["adm_novelty_gain"] * n_mean
        + rp["adm_saturation_gain"] * c_mean
        + rp["adm_energy_gain"] * e_mean
        + rp["adm_bias"]
    )
    cocktail = F.normalize(torch.stack([e_mean, c_mean, n_mean, p_mean], dim=-1), dim=-1)
    window = F.softplus(rp["admit_window"])
    if geometry == "seq":
        floor = torch.cummax(admission, dim=1).values - window
    else:
        floor = admission.max(dim=1, keepdim=True).values - window
    member = admission >= floor
    counts = member.sum(dim=1)
    order = torch.argsort(member.to(query.dtype), dim=1, descending=True, stable=True)
    n_max = max(int(counts.max().item()), 1)
    idx = order[:, :n_max]
    valid = torch.arange(n_max).unsqueeze(0) < counts.clamp_min(1).unsqueeze(1)
    gh = idx.unsqueeze(-1).expand(-1, -1, H)
    bank_writes = torch.gather(write, 1, gh)
    bank_keys = F.normalize(bank_writes, dim=-1)
    bank_cocktail = torch.gather(cocktail, 1, idx.unsqueeze(-1).expand(-1, -1, 4))
    bank_key_bias = torch.gather(key_bias, 1, idx)
    bank_admission = torch.gather(admission, 1, idx)
    nidx = (idx + 1).clamp(max=T - 1)
    next_writes = torch.gather(write, 1, nidx.unsqueeze(-1).expand(-1, -1, H))
    return {
        "query": query,
        "bank_keys": bank_keys,
        "bank_writes": bank_writes,
        "next_writes": next_writes,
        "cocktail": cocktail,
        "bank_cocktail": bank_cocktail,
        "bank_key_bias": bank_key_bias,
        "bank_admission": bank_admission,
        "scale": scale,
        "bank_idx": idx,
        "bank_valid": valid,
        "n_max": n_max,
    }


# ---------------------------------------------------------------------------
# A.4  one seq block  (src/dabsn/model.py:309-372, 179-195)
# ---------------------------------------------------------------------------
def block_forward(
    params: dict[str, Tensor],
    x: Tensor,
    *,
    residual: bool = False,
    core_state_dtype: torch.dtype | None = None,
) -> Tensor:
    """One ``DABSNBlock.forward_world`` for the seq geometry, no MLP.

    ``params`` uses the reference module's ``state_dict`` names
    (``core.W.weight``, ``read.short_read.out.bias`` ...), so a reference
    checkpoint's parameters feed it unchanged.
    """
    P = params
    Bsz, T, _ = x.shape
    H = P["core.Ug.weight"].shape[0]
    Wx = x @ P["core.W.weight"].T
    Wgx = x @ P["core.Wg.weight"].T + P["core.Wg.bias"]
    core_args = [Wx, Wgx, P["core.Ug.weight"], P["core.A.weight"]]
    core_args += [P[f"core.{n}"] for n in ("beta", "log_kappa", "logit_recover", "k_s", "k_y", "k_b", "k_n", "k_bias", "r_s", "r_y", "r_b", "r_n", "r_bias")]
    core_args.append(P["core.logit_saturation_decay"].expand(H))
    core_args += [P["core.k_saturation"], P["core.r_saturation"]]
    core_args += [P["core.logit_alpha"].reshape(()), P["core.log_lambda"].reshape(()), P["core.logit_saturation_suppress"].reshape(())]
    dt = x.dtype
    core_args += [torch.zeros(Bsz, H, dtype=dt), torch.ones(Bsz, H, dtype=dt), torch.zeros(Bsz, H, dtype=dt)]
    U, n, p, a, w, e, c, s, *_ = core_scan(*core_args, state_dtype=core_state_dtype)
    y, b = U[..., :H], U[..., H:]
    rp = {k: P[f"read.short_read.{k}"] for k in ("log_temp", "p_gain", "novelty_gain", "null_bias", "adm_p_gain", "adm_novelty_gain", "adm_saturation_gain", "adm_energy_gain", "adm_bias")}
    rp["admit_window"] = P["read.admit_window"]
    bank = admitted_bank(a, w, n, p, e, c, rp, geometry="seq")
    retrieved = three_way_read(
        bank["query"], bank["bank_keys"], bank["bank_writes"], bank["next_writes"],
        bank["cocktail"], bank["bank_cocktail"], bank["bank_key_bias"], bank["bank_admission"],
        bank["scale"], bank["bank_idx"], bank["bank_valid"], mode="seq",
        short_gain=P["read.short_gain"], pad_gain=P["read.pad_gain"],
        induct_gain=P["read.induct_gain"], cocktail_gain=P["read.cocktail_gain"],
    )
    out = torch.cat([y, b, retrieved], dim=-1) @ P["read.short_read.out.weight"].T + P["read.short_read.out.bias"]
    long = long_scan(w, p, P["read.logit_retain"], P["read.logit_expect_retain"], P["read.logit_retention_decay"], P["read.logit_retention_strength"])
    read = out + P["read.long_gain"] * long
    hidden = y + P["read_gain"] * read
    if residual:
        hidden = x + hidden
    return hidden


def linrec(a: Tensor, g: Tensor, y_init: Tensor) -> Tensor:
    """``y_t = a_t*y_{t-1} + g_t`` (src/dabsn/kernels/long.py:24-32)."""
    y = y_init
    outs = []
    for t in range(a.shape[1]):
        y = a[:, t] * y + g[:, t]
        outs.append(y)
    return torch.stack(outs, dim=1)


def softplus(x: float) -> float:
    return math.log1p(math.exp(x))


# ---------------------------------------------------------------------------
# Primitives of the dabsn.kernels surface
# ---------------------------------------------------------------------------
def permanent_delta_scan(k: Tensor, v: Tensor, beta: Tensor) -> Tensor:
    """Delta-rule scan of ``dabsn::permanent_delta_scan``
    (src/dabsn/kernels/permanent.py:56-67): S starts at zero;
    r_t = S k_t, S <- S + beta_t (v_t - r_t) k_t^T; returns r.  Gradients by
    autograd through the loop (the reference's analytic reverse,
    permanent.py:70-110, is its twin)."""
    B, T, h = k.shape
    S = k.new_zeros(B, h, h)
    outs = []
    for t in range(T):
        kt = k[:, t]
        r = torch.einsum("bvk,bk->bv", S, kt)
        outs.append(r)
        S = S + beta[:, t].view(B, 1, 1) * torch.einsum("bv,bk->bvk", v[:, t] - r, kt)
    return torch.stack(outs, dim=1)


def local_field_gather(x: Tensor, patch: Tensor) -> Tensor:
    """``dabsn::local_field_gather`` (src/dabsn/kernels/local_field.py:208-214):
    out[b, n, k, :] = x[b, patch[n, k], :]."""
    return x[:, patch]


# ---------------------------------------------------------------------------
# Readout + cross-entropy (the training loss after the blocks)
# ---------------------------------------------------------------------------
def linear_cross_entropy(hidden: Tensor, weight: Tensor, bias: Tensor | None, targets: Tensor,
                         ignore_index: int = -100, empty: str = "zero",
                         logits_dtype: torch.dtype | None = None) -> Tensor:
    """Mean cross-entropy of ``dabsn.runtime.chunked_linear_cross_entropy``
    (src/dabsn/runtime/loss.py:57-96, chunked; :165-180, single shot).

    logits = hidden W^T + b, rounded to ``logits_dtype`` when given (the BF16
    logits that F.linear gives under autocast), then in float64; the loss sums
    logsumexp(logits) - logits[target] over the rows whose target is not
    ``ignore_index`` and divides by their number.  With no such row the
    chunked branch divides by 1 (``empty="zero"``: loss 0) and the single-shot
    branch (F.cross_entropy's mean) gives NaN (``empty="nan"``).  Gradients by
    autograd (the reference's chunked reverse, loss.py:98-135, is its twin)."""
    logits = hidden @ weight.transpose(0, 1)
    if bias is not None:
        logits = logits + bias
    if logits_dtype is not None:
        logits = logits.to(logits_dtype)
    logits = logits.to(torch.float64)
    valid = targets != ignore_index
    safe = torch.where(valid, targets, torch.zeros_like(targets))
    nll = torch.logsumexp(logits, dim=-1) - logits.gather(-1, safe.unsqueeze(-1)).squeeze(-1)
    total = (nll * valid.to(nll.dtype)).sum()
    count = valid.sum()
    if int(count) == 0 and empty == "nan":
        return total * float("nan")
    return total / max(int(count), 1)
