// Fused long-memory channel: the three diagonal recurrences of the DABSN read
// (expected E, retention Q, long L) and their elementwise glue in one pass.
//
// Reference: src/dabsn/read.py:597-640 (loop form) and
// src/dabsn/kernels/long.py:492-579 (three `dabsn::linear_recurrence` launches
// plus ATen glue, with the Triton kernels at long.py:106-212).  Per element:
//
//   pi_t  = tanh|w_t - E_{t-1}|          sal_t = p_t * pi_t
//   E_t   = re*E_{t-1} + (1-re)*w_t
//   Q_t   = rd*Q_{t-1} + (1-rd)*(1-pi_t)
//   eta_t = R + (1-R)*rs*Q_t
//   L_t   = eta_t*L_{t-1} + (1-eta_t)*sal_t*w_t
//
// Every (sequence, unit) pair is independent, so one thread owns one pair for
// the whole sequence; consecutive threads own consecutive units (coalesced).
// The forward loads KCH steps of (w, p) ahead into registers.  In training it
// also stores (L, E, Q) at the start of every KCH-step chunk; the reverse pass
// recomputes one chunk forward in registers from that checkpoint and then
// runs the adjoint back through it, so no [B,T,H] intermediate is stored.
#include "../../include/dabsn_b200.h"
#include "common.cuh"

namespace dabsn {
namespace {

constexpr int KCH = 8;  // steps per chunk (prefetch depth and checkpoint stride)
constexpr int LTHREADS = 128;

struct LongScalars {
  float R, re, rd, rs;
};

__device__ __forceinline__ LongScalars load_scalars(const float* logits) {
  LongScalars s;
  s.R = sigmoidf_(logits[0]);
  s.re = sigmoidf_(logits[1]);
  s.rd = sigmoidf_(logits[2]);
  s.rs = sigmoidf_(logits[3]);
  return s;
}

template <typename Act>
__global__ void __launch_bounds__(LTHREADS) long_fwd_kernel(
    int B, int T, int H, const Act* __restrict__ w, const Act* __restrict__ p,
    const float* __restrict__ logits, const float* __restrict__ init, float* __restrict__ out,
    float* __restrict__ ckpt, float* __restrict__ fin) {
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)B * H) return;
  const int b = (int)(gid / H), h = (int)(gid % H);
  const LongScalars sc = load_scalars(logits);
  const size_t bs = (size_t)b * H + h;
  const size_t BH = (size_t)B * H;
  float L = init ? init[bs] : 0.f;
  float E = init ? init[BH + bs] : 0.f;
  float Q = init ? init[2 * BH + bs] : 1.f;
  const int nchunks = (T + KCH - 1) / KCH;
  const size_t base = (size_t)b * T * H + h;
  float wn[KCH], pn[KCH];
#pragma unroll
  for (int k = 0; k < KCH; ++k) {
    const bool ok = k < T;
    wn[k] = ok ? to_f<Act>(w[base + (size_t)k * H]) : 0.f;
    pn[k] = ok ? to_f<Act>(p[base + (size_t)k * H]) : 0.f;
  }
  for (int c = 0; c < nchunks; ++c) {
    float wc[KCH], pc[KCH];
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      wc[k] = wn[k];
      pc[k] = pn[k];
    }
    // Prefetch the next chunk while this one is computed.
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      const int t = (c + 1) * KCH + k;
      const bool ok = t < T;
      wn[k] = ok ? to_f<Act>(w[base + (size_t)t * H]) : 0.f;
      pn[k] = ok ? to_f<Act>(p[base + (size_t)t * H]) : 0.f;
    }
    if (ckpt) {
      float* dst = ckpt + ((size_t)b * nchunks + c) * 3 * H + h;
      dst[0] = L;
      dst[H] = E;
      dst[2 * H] = Q;
    }
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      const int t = c * KCH + k;
      if (t < T) {
        const float wt = wc[k];
        const float pe = tanhf(fabsf(wt - E));
        const float sal = pc[k] * pe;
        E = sc.re * E + (1.0f - sc.re) * wt;
        Q = sc.rd * Q + (1.0f - sc.rd) * (1.0f - pe);
        const float eta = sc.R + (1.0f - sc.R) * sc.rs * Q;
        L = eta * L + (1.0f - eta) * (sal * wt);
        out[base + (size_t)t * H] = L;
      }
    }
  }
  if (fin) {
    fin[bs] = L;
    fin[BH + bs] = E;
    fin[2 * BH + bs] = Q;
  }
}

template <typename Act>
__global__ void __launch_bounds__(LTHREADS) long_bwd_kernel(
    int B, int T, int H, const Act* __restrict__ w, const Act* __restrict__ p,
    const float* __restrict__ logits, const float* __restrict__ ckpt,
    const float* __restrict__ gout, const float* __restrict__ gfin, Act* __restrict__ dw,
    Act* __restrict__ dp, float* __restrict__ ginit, float* __restrict__ partial) {
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)B * H) return;
  const int b = (int)(gid / H), h = (int)(gid % H);
  const LongScalars sc = load_scalars(logits);
  const size_t bs = (size_t)b * H + h;
  const size_t BH = (size_t)B * H;
  const int nchunks = (T + KCH - 1) / KCH;
  const size_t base = (size_t)b * T * H + h;
  // Adjoints of the state after the current step, flowing in from the future.
  float gL = gfin ? gfin[bs] : 0.f;
  float gE = gfin ? gfin[BH + bs] : 0.f;
  float gQ = gfin ? gfin[2 * BH + bs] : 0.f;
  float dR = 0.f, dre = 0.f, drd = 0.f, drs = 0.f;
  // The inputs of chunk c - 1 are loaded while chunk c is computed.
  float nwc[KCH], npc[KCH], ngo[KCH], nL, nE, nQ;
  auto fetch = [&](int c) {
    const float* src = ckpt + ((size_t)b * nchunks + c) * 3 * H + h;
    nL = src[0];
    nE = src[H];
    nQ = src[2 * H];
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      const int t = c * KCH + k;
      const bool ok = t < T;
      nwc[k] = ok ? to_f<Act>(w[base + (size_t)t * H]) : 0.f;
      npc[k] = ok ? to_f<Act>(p[base + (size_t)t * H]) : 0.f;
      ngo[k] = ok ? gout[base + (size_t)t * H] : 0.f;
    }
  };
  fetch(nchunks - 1);
  for (int c = nchunks - 1; c >= 0; --c) {
    float L = nL, E = nE, Q = nQ;
    float wc[KCH], pc[KCH], go[KCH], Lp[KCH], Ep[KCH], Qp[KCH];
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      wc[k] = nwc[k];
      pc[k] = npc[k];
      go[k] = ngo[k];
    }
    if (c > 0) fetch(c - 1);
    // Recompute the chunk, keeping the state before every step.
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      Lp[k] = L;
      Ep[k] = E;
      Qp[k] = Q;
      const float wt = wc[k];
      const float pe = tanhf(fabsf(wt - E));
      E = sc.re * E + (1.0f - sc.re) * wt;
      Q = sc.rd * Q + (1.0f - sc.rd) * (1.0f - pe);
      const float eta = sc.R + (1.0f - sc.R) * sc.rs * Q;
      L = eta * L + (1.0f - eta) * (pc[k] * pe * wt);
    }
#pragma unroll
    for (int k = KCH - 1; k >= 0; --k) {
      const int t = c * KCH + k;
      if (t < T) {
        const float wt = wc[k], pt = pc[k];
        const float Em = Ep[k], Qm = Qp[k], Lm = Lp[k];
        const float diff = wt - Em;
        const float pe = tanhf(fabsf(diff));
        const float sal = pt * pe;
        const float Qt = sc.rd * Qm + (1.0f - sc.rd) * (1.0f - pe);
        const float eta = sc.R + (1.0f - sc.R) * sc.rs * Qt;
        const float lamL = go[k] + gL;
        const float deta = lamL * (Lm - sal * wt);
        const float dsal = lamL * (1.0f - eta) * wt;
        float dwt = lamL * (1.0f - eta) * sal;
        const float lamQ = gQ + deta * (1.0f - sc.R) * sc.rs;
        dR += deta * (1.0f - sc.rs * Qt);
        drs += deta * (1.0f - sc.R) * Qt;
        drd += lamQ * (Qm - (1.0f - pe));
        float dpe = -lamQ * (1.0f - sc.rd) + dsal * pt;
        const float dpt = dsal * pe;
        // E_t = re*E_{t-1} + (1-re)*w_t
        dwt += gE * (1.0f - sc.re);
        dre += gE * (Em - wt);
        float gEm = gE * sc.re;
        const float dd = dpe * (1.0f - pe * pe) * signf_(diff);
        dwt += dd;
        gEm -= dd;
        dw[base + (size_t)t * H] = from_f<Act>(dwt);
        dp[base + (size_t)t * H] = from_f<Act>(dpt);
        gL = lamL * eta;
        gQ = lamQ * sc.rd;
        gE = gEm;
      }
    }
  }
  if (ginit) {
    ginit[bs] = gL;
    ginit[BH + bs] = gE;
    ginit[2 * BH + bs] = gQ;
  }
  // d/dlogit = d/dsigmoid * s(1-s)
  float* dst = partial + (size_t)gid * 4;
  dst[0] = dR * sc.R * (1.0f - sc.R);
  dst[1] = dre * sc.re * (1.0f - sc.re);
  dst[2] = drd * sc.rd * (1.0f - sc.rd);
  dst[3] = drs * sc.rs * (1.0f - sc.rs);
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int dabsn_long_chunk(void) { return KCH; }

extern "C" int dabsn_long_fwd(int dtype, int64_t B, int64_t T, int64_t H, const void* write,
                              const void* plasticity, const float* logits, const float* init,
                              float* out, float* ckpt, float* fin, void* stream) {
  if (B < 0 || T < 0 || H <= 0) {
    set_error("long_fwd: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  if (B == 0 || T == 0) return DABSN_OK;
  const long long n = (long long)B * H;
  const dim3 grid((unsigned)((n + LTHREADS - 1) / LTHREADS));
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32) {
    long_fwd_kernel<float><<<grid, LTHREADS, 0, st>>>((int)B, (int)T, (int)H, (const float*)write,
                                                      (const float*)plasticity, logits, init, out,
                                                      ckpt, fin);
  } else if (dtype == DABSN_BF16) {
    long_fwd_kernel<__nv_bfloat16><<<grid, LTHREADS, 0, st>>>(
        (int)B, (int)T, (int)H, (const __nv_bfloat16*)write, (const __nv_bfloat16*)plasticity,
        logits, init, out, ckpt, fin);
  } else {
    set_error("long_fwd: unsupported dtype %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("long_fwd");
}

extern "C" int dabsn_long_bwd(int dtype, int64_t B, int64_t T, int64_t H, const void* write,
                              const void* plasticity, const float* logits, const float* ckpt,
                              const float* gout, const float* gfin, void* dwrite, void* dplast,
                              float* ginit, float* partial, void* stream) {
  if (B < 0 || T < 0 || H <= 0) {
    set_error("long_bwd: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  if (B == 0 || T == 0) return DABSN_OK;
  const long long n = (long long)B * H;
  const dim3 grid((unsigned)((n + LTHREADS - 1) / LTHREADS));
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32) {
    long_bwd_kernel<float><<<grid, LTHREADS, 0, st>>>(
        (int)B, (int)T, (int)H, (const float*)write, (const float*)plasticity, logits, ckpt, gout,
        gfin, (float*)dwrite, (float*)dplast, ginit, partial);
  } else if (dtype == DABSN_BF16) {
    long_bwd_kernel<__nv_bfloat16><<<grid, LTHREADS, 0, st>>>(
        (int)B, (int)T, (int)H, (const __nv_bfloat16*)write, (const __nv_bfloat16*)plasticity,
        logits, ckpt, gout, gfin, (__nv_bfloat16*)dwrite, (__nv_bfloat16*)dplast, ginit, partial);
  } else {
    set_error("long_bwd: unsupported dtype %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("long_bwd");
}
