// Per-element mathematics of the DABSN core recurrence, shared by the
// register-resident scans (core_scan.cu) and the grid-wide scans
// (core_scan_wide.cu).  Reference: src/dabsn/kernels/batched_runtime.py:38-158
// (forward step) and :299-466 (reverse step).
#pragma once

#include "common.cuh"

namespace dabsn {

struct CoreParams {
  // Per-unit parameters, FP32 [H].
  const float* beta;
  const float* log_kappa;
  const float* logit_recover;
  const float* k_s;
  const float* k_y;
  const float* k_b;
  const float* k_n;
  const float* k_bias;
  const float* r_s;
  const float* r_y;
  const float* r_b;
  const float* r_n;
  const float* r_bias;
  const float* logit_c_decay;
  const float* k_c;
  const float* r_c;
  // Scalars, FP32 [1].
  const float* logit_alpha;
  const float* log_lambda;
  const float* logit_c_suppress;
};

// Derived per-unit constants of one state element.
struct UnitConsts {
  float kappa, recover, decay, beta, sigk;
  float ks, ky, kb, kn, kbias, kc, rs, ry, rb, rn, rbias, rc;
};

__device__ __forceinline__ UnitConsts load_unit(const CoreParams& p, int u) {
  UnitConsts c;
  c.kappa = softplusf_(p.log_kappa[u]);
  c.sigk = sigmoidf_(p.log_kappa[u]);
  c.recover = sigmoidf_(p.logit_recover[u]);
  c.decay = sigmoidf_(p.logit_c_decay[u]);
  c.beta = p.beta[u];
  c.ks = p.k_s[u];
  c.ky = p.k_y[u];
  c.kb = p.k_b[u];
  c.kn = p.k_n[u];
  c.kbias = p.k_bias[u];
  c.kc = p.k_c[u];
  c.rs = p.r_s[u];
  c.ry = p.r_y[u];
  c.rb = p.r_b[u];
  c.rn = p.r_n[u];
  c.rbias = p.r_bias[u];
  c.rc = p.r_c[u];
  return c;
}

// Everything the reverse step t reads for one (sequence, unit) element.
struct StepIn {
  float y, b_prev, e_prev, c_prev, gate, p, ay, c_t;
  float gy0, gb, gc, gnov, gp, gay, gw, ge;
};

// The part of a reverse step that depends only on saved tapes and parameters,
// not on the adjoints carried from later steps.
struct StepPre {
  StepIn in;
  float nov, tanh_b, neff, tanh_k, tanh_r, exp_k, exp_r, wcost, rec_pre, recov, rec_cg;
  float emask, gmask, stress, c_new, dnov_scale;
};

__device__ __forceinline__ StepPre pre_step(const StepIn& in, const UnitConsts& uc,
                                            float suppress) {
  StepPre r;
  r.in = in;
  r.nov = tanh_fast(fabsf(in.ay - in.b_prev));
  r.tanh_b = tanh_fast(in.b_prev);
  r.neff = r.nov * (1.0f - suppress * in.c_t);
  const float ksig = uc.ks * in.gate + uc.ky * in.y + uc.kb * r.tanh_b + uc.kn * r.neff +
                     uc.kbias + uc.kc * in.c_t;
  const float rsig = uc.rs * in.gate + uc.ry * in.y + uc.rb * r.tanh_b + uc.rn * r.neff +
                     uc.rbias + uc.rc * in.c_t;
  r.tanh_k = tanh_fast(ksig);
  r.tanh_r = tanh_fast(rsig);
  r.exp_k = exp_fast(0.5f * r.tanh_k);
  r.exp_r = exp_fast(0.5f * r.tanh_r);
  r.wcost = uc.kappa * r.exp_k;
  r.rec_pre = uc.recover * r.exp_r;
  r.recov = clamp01(r.rec_pre);
  r.rec_cg = (r.rec_pre >= 0.f && r.rec_pre <= 1.f) ? 1.f : 0.f;
  const float e_pre = in.e_prev + r.recov * (1.0f - in.e_prev) - r.wcost * in.p;
  r.emask = (e_pre >= 0.f && e_pre <= 1.f) ? 1.f : 0.f;
  r.gmask = (in.gate > 0.f && in.gate < 1.f) ? (1.0f / 6.0f) : 0.f;
  r.stress = r.nov * (1.0f - in.e_prev);
  r.c_new = uc.decay * in.c_prev + (1.0f - uc.decay) * r.stress;
  r.dnov_scale = (1.0f - r.nov * r.nov) * signf_(in.ay - in.b_prev);
  return r;
}


// One forward step of one state element (batched_runtime.py:95-158), with
// the product (g_r, a) already formed.  Returns the tapes of the step and the
// next state; y_next needs the next step's pre-activation wx_next.
struct FwdPoint {
  float s, n, c, pl, w, bn, enew;
};

// The part of the step the next recurrent vector depends on: gate,
// plasticity, write and the new b.
__device__ __forceinline__ void fwd_gate(float b, float e, float wgx, float gr, float a,
                                         const UnitConsts& uc, float alpha, float lam,
                                         FwdPoint& r) {
  r.s = hardsigmoidf_(wgx + gr);
  r.pl = r.s * e;
  r.w = r.pl * a;
  r.bn = (1.0f - alpha) * b + uc.beta + lam * r.w;
}

// The rest of the step: novelty, saturation and the energy update.
__device__ __forceinline__ void fwd_rest(float y, float b, float e, float c_prev, float a,
                                         const UnitConsts& uc, float suppress, FwdPoint& r) {
  r.n = tanh_fast(fabsf(a - b));
  r.c = uc.decay * c_prev + (1.0f - uc.decay) * (r.n * (1.0f - e));
  const float neff = r.n * (1.0f - suppress * r.c);
  const float tb = tanh_fast(b);
  const float ksig = uc.ks * r.s + uc.ky * y + uc.kb * tb + uc.kn * neff + uc.kbias + uc.kc * r.c;
  const float rsig = uc.rs * r.s + uc.ry * y + uc.rb * tb + uc.rn * neff + uc.rbias + uc.rc * r.c;
  const float wcost = uc.kappa * exp_fast(0.5f * tanh_fast(ksig));
  const float recov = clamp01(uc.recover * exp_fast(0.5f * tanh_fast(rsig)));
  r.enew = clamp01(e + recov * (1.0f - e) - wcost * r.pl);
}

__device__ __forceinline__ FwdPoint fwd_point(float y, float b, float e, float c_prev, float wgx,
                                              float gr, float a, const UnitConsts& uc,
                                              float alpha, float lam, float suppress) {
  FwdPoint r;
  fwd_gate(b, e, wgx, gr, a, uc, alpha, lam, r);
  fwd_rest(y, b, e, c_prev, a, uc, suppress, r);
  return r;
}

// The carried-adjoint part of one reverse step (batched_runtime.py:358-466):
// given the step's carry-independent values and the adjoints flowing in from
// later steps, the exchanged pair (dgate_pre, d_expr), the values the second
// half of the step needs, the next carries and the parameter-gradient terms.
struct BwdCarry {
  float dgate_pre, d_expr;
  float gy_rest;   // gy0 + gy_energy (the recurrent adjoint is added later)
  float gb_rest;   // next_gb before - d_nov + gpre: g_bprev_state + gb_energy - d_nov
  float ge_next, gc_next;
  float p[16];
  float s0, s1, s2;
};

__device__ __forceinline__ void bwd_carry(const StepPre& pre, const UnitConsts& uc, float gbn,
                                          float gen, float gcn, float alpha, float lam,
                                          float sig_lam, float suppress, BwdCarry& o) {
  const StepIn& in = pre.in;
  const float gb_new = in.gb + gbn;
  const float gc_new = gcn + in.gc;
  const float ge_pre = gen * pre.emask;
  const float g_bprev_state = gb_new * (1.0f - alpha);
  const float g_eprev_state = ge_pre * (1.0f - pre.recov);
  float gp = in.gp + gb_new * lam * in.ay - ge_pre * pre.wcost;
  const float gayv = in.gay + gb_new * lam * in.p;
  const float g_wcost = -ge_pre * in.p;
  const float g_recov = ge_pre * (1.0f - in.e_prev);
  const float d_expr_main = gayv + in.gw * in.p;
  gp = gp + in.gw * in.ay;
  const float g_ksig = g_wcost * pre.wcost * 0.5f * (1.0f - pre.tanh_k * pre.tanh_k);
  const float g_rec_pre = g_recov * pre.rec_cg;
  const float g_rsig = g_rec_pre * pre.rec_pre * 0.5f * (1.0f - pre.tanh_r * pre.tanh_r);
  const float g_gate_energy = g_ksig * uc.ks + g_rsig * uc.rs;
  const float gnov_eff = g_ksig * uc.kn + g_rsig * uc.rn;
  const float gc_energy = g_ksig * uc.kc + g_rsig * uc.rc;
  o.dgate_pre = (gp * in.e_prev + g_gate_energy) * pre.gmask;
  const float g_c_new = gc_new + gc_energy - gnov_eff * pre.nov * suppress;
  const float g_stress = g_c_new * (1.0f - uc.decay);
  const float g_nov = gnov_eff * (1.0f - suppress * pre.c_new) + g_stress * (1.0f - in.e_prev);
  const float d_nov = (in.gnov + g_nov) * pre.dnov_scale;
  o.d_expr = d_expr_main + d_nov;
  const float gy_energy = g_ksig * uc.ky + g_rsig * uc.ry;
  const float gb_energy = (g_ksig * uc.kb + g_rsig * uc.rb) * (1.0f - pre.tanh_b * pre.tanh_b);
  o.gy_rest = in.gy0 + gy_energy;
  o.gb_rest = g_bprev_state + gb_energy - d_nov;
  o.ge_next = g_eprev_state + gp * in.gate - g_stress * pre.nov + in.ge;
  o.gc_next = g_c_new * uc.decay;
  o.p[0] = gb_new;
  o.p[1] = g_wcost * pre.exp_k * uc.sigk;
  o.p[2] = g_rec_pre * pre.exp_r * uc.recover * (1.0f - uc.recover);
  o.p[3] = g_ksig * in.gate;
  o.p[4] = g_ksig * in.y;
  o.p[5] = g_ksig * pre.tanh_b;
  o.p[6] = g_ksig * pre.neff;
  o.p[7] = g_ksig;
  o.p[8] = g_rsig * in.gate;
  o.p[9] = g_rsig * in.y;
  o.p[10] = g_rsig * pre.tanh_b;
  o.p[11] = g_rsig * pre.neff;
  o.p[12] = g_rsig;
  o.p[13] = g_c_new * (in.c_prev - pre.stress) * uc.decay * (1.0f - uc.decay);
  o.p[14] = g_ksig * in.c_t;
  o.p[15] = g_rsig * in.c_t;
  o.s0 = gb_new * (-in.b_prev) * alpha * (1.0f - alpha);
  o.s1 = gb_new * (in.p * in.ay) * sig_lam;
  o.s2 = gnov_eff * pre.nov * (-pre.c_new) * suppress * (1.0f - suppress);
}

}  // namespace dabsn
