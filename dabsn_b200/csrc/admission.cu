// Read admission and admitted-bank construction, forward and backward.
//
// Reference: src/dabsn/read.py:152-303 (`DABSNRead._unified_forward`) and
// :58-72 (`_AdmittedReadParameters.admission`).  Per token (b, t), over the
// state width H:
//
//   query      = expression / max(|expression|, 1e-12)
//   mp, mn, me, mc = means of plasticity, novelty, energy, saturation
//   lg         = log1p(mp * H)
//   key_bias   = p_gain lg + novelty_gain mn + null_bias
//   admission  = adm_p_gain lg + adm_novelty_gain mn + adm_saturation_gain mc
//              + adm_energy_gain me + adm_bias
//   cocktail   = normalize([me, mc, mn, mp])
//   member     = admission >= cummax_{u<=t} admission_u - softplus(window)   (seq)
//              = admission >= max_u admission_u - softplus(window)          (field)
//
// The bank lists members in ascending position, then the other positions in
// ascending position (a stable partition, what the reference's stable argsort
// of the membership flags yields); its first n_max entries are gathered:
// writes, keys = normalize(writes), next writes (position + 1, clamped),
// cocktails, key biases and admissions.
//
// With BF16 activations the statistics follow the reference under autocast:
// the means and mp * H are rounded to BF16, log1p and the rest run in FP32.
//
// Kernels: token statistics (one warp per token), membership and stable
// partition (one CTA per sequence), bank gather (one warp per bank entry);
// backward: one warp per token assembles every input gradient of that token
// from the bank entries that read it (an inverse map, no atomics).
#include <climits>

#include "../../include/dabsn_b200.h"
#include "common.cuh"

namespace dabsn {
namespace {

typedef __nv_bfloat16 bf16;
constexpr float kNormEps = 1e-12f;

template <typename Act>
__device__ __forceinline__ float round_stat(float v) {
  return to_f<Act>(from_f<Act>(v));
}

// params: p_gain, novelty_gain, null_bias, adm_p_gain, adm_novelty_gain,
//         adm_saturation_gain, adm_energy_gain, adm_bias
template <typename Act>
__global__ void __launch_bounds__(256) adm_stats_kernel(int B, int T, int H, const Act* expr,
                                                        const Act* nov, const Act* plast,
                                                        const Act* energy, const Act* sat,
                                                        const float* params, float* query,
                                                        float* kb, float* adm, float* cocktail,
                                                        float* stats) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= (long long)B * T) return;
  const size_t o = (size_t)row * H;
  float sq = 0.f, sp = 0.f, sn = 0.f, se = 0.f, sc = 0.f;
  for (int h = lane; h < H; h += 32) {
    const float x = to_f<Act>(expr[o + h]);
    sq = fmaf(x, x, sq);
    sp += to_f<Act>(plast[o + h]);
    sn += to_f<Act>(nov[o + h]);
    se += to_f<Act>(energy[o + h]);
    sc += to_f<Act>(sat[o + h]);
  }
  sq = warp_sum(sq);
  sp = warp_sum(sp);
  sn = warp_sum(sn);
  se = warp_sum(se);
  sc = warp_sum(sc);
  const float inv_h = 1.0f / (float)H;
  const float mp = round_stat<Act>(sp * inv_h), mn = round_stat<Act>(sn * inv_h);
  const float me = round_stat<Act>(se * inv_h), mc = round_stat<Act>(sc * inv_h);
  const float norm = sqrtf(sq);
  const float den = fmaxf(norm, kNormEps);
  for (int h = lane; h < H; h += 32) query[o + h] = to_f<Act>(expr[o + h]) / den;
  if (lane == 0) {
    const float mpH = round_stat<Act>(mp * (float)H);
    const float lg = log1pf(mpH);
    kb[row] = params[0] * lg + params[1] * mn + params[2];
    adm[row] = params[3] * lg + params[4] * mn + params[5] * mc + params[6] * me + params[7];
    const float cn = sqrtf(me * me + mc * mc + mn * mn + mp * mp);
    const float cd = fmaxf(cn, kNormEps);
    float* c = cocktail + row * 4;
    c[0] = me / cd;
    c[1] = mc / cd;
    c[2] = mn / cd;
    c[3] = mp / cd;
    float* s = stats + row * 8;
    s[0] = mp; s[1] = mn; s[2] = me; s[3] = mc;
    s[4] = lg; s[5] = mpH; s[6] = norm; s[7] = cn;
  }
}

// Inclusive scans over one CTA of 1024 threads (warp shuffles + one smem pass).
constexpr int OT = 1024;

__device__ __forceinline__ float block_scan_max(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = fmaxf(v, n);
  }
  if (lane == 31) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w = fmaxf(w, n);
    }
    sh[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v = fmaxf(v, sh[warp - 1]);
  __syncthreads();
  return v;
}

__device__ __forceinline__ int block_scan_sum(int v, int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    sh[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += sh[warp - 1];
  __syncthreads();
  return v;
}

// One CTA per sequence: membership, member count, the stable partition
// `order` (members, then the others, each in ascending position) and the
// inverse map inv[t] = bank slot of t if t is a member, else -1.
__global__ void __launch_bounds__(OT) adm_order_kernel(int T, int mode, const float* adm,
                                                       const float* window, int64_t* order,
                                                       int64_t* counts, int* inv) {
  __shared__ float shf[32];
  __shared__ int shi[32];
  __shared__ float s_carry_f;
  __shared__ int s_carry_i;
  const int b = blockIdx.x;
  const float* a = adm + (size_t)b * T;
  int* iv = inv + (size_t)b * T;
  int64_t* od = order + (size_t)b * T;
  const float w = window[0];

  float gmax = -INFINITY;
  if (mode != 0) {
    float m = -INFINITY;
    for (int t = threadIdx.x; t < T; t += OT) m = fmaxf(m, a[t]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) shf[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = shf[threadIdx.x];
      v = warp_max(v);
      if (threadIdx.x == 0) s_carry_f = v;
    }
    __syncthreads();
    gmax = s_carry_f;
    __syncthreads();
  }
  // pass 1: membership (kept in inv as 0/1) and the member count
  if (threadIdx.x == 0) {
    s_carry_f = -INFINITY;
    s_carry_i = 0;
  }
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += OT) {
    const int t = t0 + threadIdx.x;
    const float v = t < T ? a[t] : -INFINITY;
    float floor_v;
    if (mode == 0) {
      float pm = block_scan_max(v, shf);
      pm = fmaxf(pm, s_carry_f);
      floor_v = pm - w;
      __syncthreads();
      if (threadIdx.x == OT - 1) s_carry_f = pm;
    } else {
      floor_v = gmax - w;
    }
    const int mem = (t < T && v >= floor_v) ? 1 : 0;
    if (t < T) iv[t] = mem;
    const int cnt = block_scan_sum(mem, shi);
    if (threadIdx.x == OT - 1) s_carry_i += cnt;
    __syncthreads();
  }
  const int total = s_carry_i;
  __syncthreads();
  // pass 2: slots
  if (threadIdx.x == 0) s_carry_i = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += OT) {
    const int t = t0 + threadIdx.x;
    const int mem = t < T ? iv[t] : 0;
    const int incl = block_scan_sum(mem, shi);
    const int before = s_carry_i + incl - mem;  // members before t
    if (t < T) {
      const int slot = mem ? before : total + (t - before);
      od[slot] = t;
      iv[t] = mem ? before : -1;
    }
    __syncthreads();
    if (threadIdx.x == OT - 1) s_carry_i += incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[b] = total;
}

// One warp per bank entry (b, j < n): gathers and key normalisation.
template <typename Act>
__global__ void __launch_bounds__(256) bank_gather_kernel(
    int B, int T, int H, int n, const Act* write, const float* kb, const float* adm,
    const float* cocktail, const int64_t* order, const int64_t* counts, Act* bank_writes,
    float* bank_keys, Act* next_writes, float* bank_cocktail, float* bank_bias,
    float* bank_adm, int64_t* bank_idx, bool* bank_valid, float* key_norm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long e = (long long)blockIdx.x * 8 + warp;
  if (e >= (long long)B * n) return;
  const int b = (int)(e / n), j = (int)(e % n);
  const int t = (int)order[(size_t)b * T + j];
  const int tn = min(t + 1, T - 1);
  const Act* src = write + ((size_t)b * T + t) * H;
  const Act* srcn = write + ((size_t)b * T + tn) * H;
  float sq = 0.f;
  for (int h = lane; h < H; h += 32) {
    const float x = to_f<Act>(src[h]);
    sq = fmaf(x, x, sq);
  }
  sq = warp_sum(sq);
  const float norm = sqrtf(sq);
  const float den = fmaxf(norm, kNormEps);
  Act* bw = bank_writes + (size_t)e * H;
  float* bk = bank_keys + (size_t)e * H;
  Act* nw = next_writes + (size_t)e * H;
  for (int h = lane; h < H; h += 32) {
    const Act x = src[h];
    bw[h] = x;
    bk[h] = to_f<Act>(x) / den;
    nw[h] = srcn[h];
  }
  if (lane < 4) bank_cocktail[(size_t)e * 4 + lane] = cocktail[((size_t)b * T + t) * 4 + lane];
  if (lane == 0) {
    bank_bias[e] = kb[(size_t)b * T + t];
    bank_adm[e] = adm[(size_t)b * T + t];
    bank_idx[e] = t;
    const long long c = counts[b] > 0 ? counts[b] : 1;
    bank_valid[e] = j < c;
    key_norm[e] = norm;
  }
}

// Backward, one warp per token (b, t).  Bank slots that read position t:
// j = inv[t] (its write and key), inv[t-1] (next write of t-1) and, at
// t = T-1, inv[T-1] again (the next write of the last position is itself).
// Slots at or beyond n (not gathered) contribute nothing.
template <typename Act>
__global__ void __launch_bounds__(256) adm_bwd_kernel(
    int B, int T, int H, int n, const Act* expr, const Act* write, const float* stats,
    const float* query, const float* cocktail, const float* params, const int* inv,
    const float* key_norm, const float* bank_keys, const float* d_query, const float* d_cocktail,
    const float* d_keys, const float* d_writes, const float* d_next, const float* d_bcocktail,
    const float* d_bbias, const float* d_badm, Act* d_expr, Act* d_write, float* d_means,
    float* param_part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= (long long)B * T) return;
  const int b = (int)(row / T), t = (int)(row % T);
  const int* iv = inv + (size_t)b * T;
  int j = iv[t];
  int jp = t >= 1 ? iv[t - 1] : -1;
  int jl = t == T - 1 ? iv[t] : -1;
  if (j >= n) j = -1;
  if (jp >= n) jp = -1;
  if (jl >= n) jl = -1;
  const size_t o = (size_t)row * H;
  const size_t ej = (size_t)b * n + (j < 0 ? 0 : j);
  const size_t ep = (size_t)b * n + (jp < 0 ? 0 : jp);
  const size_t el = (size_t)b * n + (jl < 0 ? 0 : jl);

  // query normalisation
  const float* s = stats + row * 8;
  const float qnorm = s[6];
  float dot = 0.f;
  if (d_query) {
    for (int h = lane; h < H; h += 32) dot = fmaf(query[o + h], d_query[o + h], dot);
    dot = warp_sum(dot);
  }
  // key normalisation of slot j
  float kdot = 0.f;
  const float knorm = j >= 0 ? key_norm[ej] : 0.f;
  if (j >= 0 && d_keys) {
    for (int h = lane; h < H; h += 32)
      kdot = fmaf(bank_keys[ej * H + h], d_keys[ej * H + h], kdot);
    kdot = warp_sum(kdot);
  }
  for (int h = lane; h < H; h += 32) {
    float ge = 0.f;
    if (d_query) {
      const float g = d_query[o + h];
      ge = qnorm > kNormEps ? (g - query[o + h] * dot) / qnorm : g / kNormEps;
    }
    d_expr[o + h] = from_f<Act>(ge);
    float gw = 0.f;
    if (j >= 0) {
      if (d_writes) gw += d_writes[ej * H + h];
      if (d_keys) {
        const float g = d_keys[ej * H + h];
        gw += knorm > kNormEps ? (g - bank_keys[ej * H + h] * kdot) / knorm : g / kNormEps;
      }
    }
    if (jp >= 0 && d_next) gw += d_next[ep * H + h];
    if (jl >= 0 && d_next) gw += d_next[el * H + h];
    d_write[o + h] = from_f<Act>(gw);
  }
  if (lane == 0) {
    const float dkb = (j >= 0 && d_bbias) ? d_bbias[ej] : 0.f;
    const float dad = (j >= 0 && d_badm) ? d_badm[ej] : 0.f;
    float dc[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      dc[c] = (d_cocktail ? d_cocktail[row * 4 + c] : 0.f) +
              ((j >= 0 && d_bcocktail) ? d_bcocktail[ej * 4 + c] : 0.f);
    }
    const float* cc = cocktail + row * 4;
    const float cn = s[7];
    float dv[4];
    if (cn > kNormEps) {
      const float cdot = cc[0] * dc[0] + cc[1] * dc[1] + cc[2] * dc[2] + cc[3] * dc[3];
#pragma unroll
      for (int c = 0; c < 4; ++c) dv[c] = (dc[c] - cc[c] * cdot) / cn;
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) dv[c] = dc[c] / kNormEps;
    }
    const float mp = s[0], mn = s[1], me = s[2], mc = s[3], lg = s[4], mpH = s[5];
    const float dlg = params[0] * dkb + params[3] * dad;
    const float dmp = dlg * (float)H / (1.0f + mpH) + dv[3];
    const float dmn = params[1] * dkb + params[4] * dad + dv[2];
    const float dme = params[6] * dad + dv[0];
    const float dmc = params[5] * dad + dv[1];
    const float inv_h = 1.0f / (float)H;
    float* dm = d_means + row * 4;
    dm[0] = dmp * inv_h;  // d plasticity (each unit)
    dm[1] = dmn * inv_h;  // d novelty
    dm[2] = dme * inv_h;  // d energy
    dm[3] = dmc * inv_h;  // d saturation
    float* pp = param_part + row * 8;
    pp[0] = lg * dkb;
    pp[1] = mn * dkb;
    pp[2] = dkb;
    pp[3] = lg * dad;
    pp[4] = mn * dad;
    pp[5] = mc * dad;
    pp[6] = me * dad;
    pp[7] = dad;
  }
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;
using dabsn::bf16;

extern "C" int dabsn_admission_fwd(int dtype, int64_t B, int64_t T, int64_t H, int mode,
                                   const void* expression, const void* novelty,
                                   const void* plasticity, const void* energy,
                                   const void* saturation, const float* params,
                                   const float* window, float* query, float* key_bias,
                                   float* admission, float* cocktail, float* stats,
                                   int64_t* order, int64_t* counts, int* inv, void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || (mode != 0 && mode != 1)) {
    set_error("admission_fwd: bad sizes or mode (B=%lld T=%lld H=%lld mode=%d)", (long long)B,
              (long long)T, (long long)H, mode);
    return DABSN_ERR_SHAPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((B * T + 7) / 8);
  if (dtype == DABSN_F32) {
    adm_stats_kernel<float><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (const float*)expression, (const float*)novelty,
        (const float*)plasticity, (const float*)energy, (const float*)saturation, params, query,
        key_bias, admission, cocktail, stats);
  } else if (dtype == DABSN_BF16) {
    adm_stats_kernel<bf16><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (const bf16*)expression, (const bf16*)novelty,
        (const bf16*)plasticity, (const bf16*)energy, (const bf16*)saturation, params, query,
        key_bias, admission, cocktail, stats);
  } else {
    set_error("admission_fwd: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  int rc = launch_status("admission_stats");
  if (rc) return rc;
  adm_order_kernel<<<(unsigned)B, OT, 0, st>>>((int)T, mode, admission, window, order, counts,
                                               inv);
  return launch_status("admission_order");
}

extern "C" int dabsn_bank_gather(int dtype, int64_t B, int64_t T, int64_t H, int64_t n,
                                 const void* write, const float* key_bias,
                                 const float* admission, const float* cocktail,
                                 const int64_t* order, const int64_t* counts, void* bank_writes,
                                 float* bank_keys, void* next_writes, float* bank_cocktail,
                                 float* bank_bias, float* bank_admission, int64_t* bank_idx,
                                 void* bank_valid, float* key_norm, void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || n <= 0 || n > T) {
    set_error("bank_gather: bad sizes (B=%lld T=%lld H=%lld n=%lld)", (long long)B, (long long)T,
              (long long)H, (long long)n);
    return DABSN_ERR_SHAPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((B * n + 7) / 8);
  if (dtype == DABSN_F32) {
    bank_gather_kernel<float><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (int)n, (const float*)write, key_bias, admission, cocktail, order,
        counts, (float*)bank_writes, bank_keys, (float*)next_writes, bank_cocktail, bank_bias,
        bank_admission, bank_idx, (bool*)bank_valid, key_norm);
  } else if (dtype == DABSN_BF16) {
    bank_gather_kernel<bf16><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (int)n, (const bf16*)write, key_bias, admission, cocktail, order,
        counts, (bf16*)bank_writes, bank_keys, (bf16*)next_writes, bank_cocktail, bank_bias,
        bank_admission, bank_idx, (bool*)bank_valid, key_norm);
  } else {
    set_error("bank_gather: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("bank_gather");
}

extern "C" int dabsn_admission_bwd(int dtype, int64_t B, int64_t T, int64_t H, int64_t n,
                                   const void* expression, const void* write, const float* stats,
                                   const float* query, const float* cocktail,
                                   const float* params, const int* inv, const float* key_norm,
                                   const float* bank_keys, const float* d_query,
                                   const float* d_cocktail, const float* d_keys,
                                   const float* d_writes, const float* d_next,
                                   const float* d_bank_cocktail, const float* d_bank_bias,
                                   const float* d_bank_admission, void* d_expression,
                                   void* d_write, float* d_means, float* param_part,
                                   void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || n <= 0 || n > T) {
    set_error("admission_bwd: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((B * T + 7) / 8);
  if (dtype == DABSN_F32) {
    adm_bwd_kernel<float><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (int)n, (const float*)expression, (const float*)write, stats,
        query, cocktail, params, inv, key_norm, bank_keys, d_query, d_cocktail, d_keys, d_writes,
        d_next, d_bank_cocktail, d_bank_bias, d_bank_admission, (float*)d_expression,
        (float*)d_write, d_means, param_part);
  } else if (dtype == DABSN_BF16) {
    adm_bwd_kernel<bf16><<<grid, 256, 0, st>>>(
        (int)B, (int)T, (int)H, (int)n, (const bf16*)expression, (const bf16*)write, stats, query,
        cocktail, params, inv, key_norm, bank_keys, d_query, d_cocktail, d_keys, d_writes, d_next,
        d_bank_cocktail, d_bank_bias, d_bank_admission, (bf16*)d_expression, (bf16*)d_write,
        d_means, param_part);
  } else {
    set_error("admission_bwd: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("admission_bwd");
}
