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
// backward: one CTA (or CTA slice) per token assembles every input gradient
// of that token from the bank entries that read it (an inverse map, no
// atomics).  The query and the bank keys are written in the read's compute
// dtype only; the backward recomputes their FP32 values from the expression
// and write rows and the stored norms with the same division, so the values
// it uses are the ones the forward rounded.  Rows whose width is a multiple
// of 8 move as 16-byte words.
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


// 8 consecutive elements moved as 16-byte words (one for BF16, two for FP32).
template <typename T>
struct Pack8 {
  uint4 w[sizeof(T) / 2];
};

template <typename T>
__device__ __forceinline__ Pack8<T> ld8(const T* p) {
  Pack8<T> v;
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(T) / 2); ++i) v.w[i] = q[i];
  return v;
}

template <typename T>
__device__ __forceinline__ float el8(const Pack8<T>& v, int i) {
  return to_f<T>(reinterpret_cast<const T*>(v.w)[i]);
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&f)[8]) {
  Pack8<T> v;
  T* e = reinterpret_cast<T*>(v.w);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f<T>(f[i]);
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(T) / 2); ++i) q[i] = v.w[i];
}

// The normalised value the forward stores and the backward recomputes.
__device__ __forceinline__ float normed(float x, float den) { return x / den; }

// params: p_gain, novelty_gain, null_bias, adm_p_gain, adm_novelty_gain,
//         adm_saturation_gain, adm_energy_gain, adm_bias
// One warp per token; `query` is written in Q (the read's compute dtype).
template <typename Act, typename Q>
__global__ void __launch_bounds__(256) adm_stats_kernel(int B, int T, int H, const Act* expr,
                                                        const Act* nov, const Act* plast,
                                                        const Act* energy, const Act* sat,
                                                        const float* params, Q* query,
                                                        float* kb, float* adm, float* cocktail,
                                                        float* stats) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= (long long)B * T) return;
  const size_t o = (size_t)row * H;
  const bool vec = (H & 7) == 0;
  float sq = 0.f, sp = 0.f, sn = 0.f, se = 0.f, sc = 0.f;
  if (vec) {
    for (int h = lane * 8; h < H; h += 256) {
      const Pack8<Act> x = ld8(expr + o + h), p = ld8(plast + o + h), n = ld8(nov + o + h),
                       e = ld8(energy + o + h), c = ld8(sat + o + h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xv = el8(x, i);
        sq = fmaf(xv, xv, sq);
        sp += el8(p, i);
        sn += el8(n, i);
        se += el8(e, i);
        sc += el8(c, i);
      }
    }
  } else {
    for (int h = lane; h < H; h += 32) {
      const float x = to_f<Act>(expr[o + h]);
      sq = fmaf(x, x, sq);
      sp += to_f<Act>(plast[o + h]);
      sn += to_f<Act>(nov[o + h]);
      se += to_f<Act>(energy[o + h]);
      sc += to_f<Act>(sat[o + h]);
    }
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
  if (vec) {
    for (int h = lane * 8; h < H; h += 256) {
      const Pack8<Act> x = ld8(expr + o + h);
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = normed(el8(x, i), den);
      st8(query + o + h, f);
    }
  } else {
    for (int h = lane; h < H; h += 32)
      query[o + h] = from_f<Q>(normed(to_f<Act>(expr[o + h]), den));
  }
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

// One warp per bank entry (b, j < n): gathers and key normalisation; the keys
// are written in K (the read's compute dtype).
template <typename Act, typename K>
__global__ void __launch_bounds__(256) bank_gather_kernel(
    int B, int T, int H, int n, const Act* write, const float* kb, const float* adm,
    const float* cocktail, const int64_t* order, const int64_t* counts, Act* bank_writes,
    K* bank_keys, Act* next_writes, float* bank_cocktail, float* bank_bias,
    float* bank_adm, int64_t* bank_idx, bool* bank_valid, float* key_norm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long e = (long long)blockIdx.x * 8 + warp;
  if (e >= (long long)B * n) return;
  const int b = (int)(e / n), j = (int)(e % n);
  const int t = (int)order[(size_t)b * T + j];
  const int tn = min(t + 1, T - 1);
  const Act* src = write + ((size_t)b * T + t) * H;
  const Act* srcn = write + ((size_t)b * T + tn) * H;
  Act* bw = bank_writes + (size_t)e * H;
  K* bk = bank_keys + (size_t)e * H;
  Act* nw = next_writes + (size_t)e * H;
  const bool vec = (H & 7) == 0;
  float sq = 0.f;
  if (vec) {
    for (int h = lane * 8; h < H; h += 256) {
      const Pack8<Act> x = ld8(src + h);
#pragma unroll
      for (int i = 0; i < 8; ++i) sq = fmaf(el8(x, i), el8(x, i), sq);
    }
  } else {
    for (int h = lane; h < H; h += 32) {
      const float x = to_f<Act>(src[h]);
      sq = fmaf(x, x, sq);
    }
  }
  sq = warp_sum(sq);
  const float norm = sqrtf(sq);
  const float den = fmaxf(norm, kNormEps);
  if (vec) {
    for (int h = lane * 8; h < H; h += 256) {
      const Pack8<Act> x = ld8(src + h), xn = ld8(srcn + h);
#pragma unroll
      for (int i = 0; i < (int)(sizeof(Act) / 2); ++i) {
        reinterpret_cast<uint4*>(bw + h)[i] = x.w[i];
        reinterpret_cast<uint4*>(nw + h)[i] = xn.w[i];
      }
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = normed(el8(x, i), den);
      st8(bk + h, f);
    }
  } else {
    for (int h = lane; h < H; h += 32) {
      const Act x = src[h];
      bw[h] = x;
      bk[h] = from_f<K>(normed(to_f<Act>(x), den));
      nw[h] = srcn[h];
    }
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

// Backward.  Bank slots that read position t: j = inv[t] (its write and
// key), inv[t-1] (next write of t-1) and, at t = T-1, inv[T-1] again (the
// next write of the last position is itself).  Slots at or beyond n (not
// gathered) contribute nothing.  The query of t is expr[t] / max(|expr[t]|,
// eps) and the key of slot j = inv[t] is write[t] / max(key_norm[j], eps),
// both recomputed here.
struct AdmTok {
  int j, jp, jl;
  size_t o, ej, ep, el;
};

__device__ __forceinline__ AdmTok adm_token(long long row, int T, int n, const int* inv) {
  AdmTok k;
  const int b = (int)(row / T), t = (int)(row % T);
  const int* iv = inv + (size_t)b * T;
  k.j = iv[t];
  k.jp = t >= 1 ? iv[t - 1] : -1;
  k.jl = t == T - 1 ? iv[t] : -1;
  if (k.j >= n) k.j = -1;
  if (k.jp >= n) k.jp = -1;
  if (k.jl >= n) k.jl = -1;
  k.ej = (size_t)b * n + (k.j < 0 ? 0 : k.j);
  k.ep = (size_t)b * n + (k.jp < 0 ? 0 : k.jp);
  k.el = (size_t)b * n + (k.jl < 0 ? 0 : k.jl);
  return k;
}

// The per-token scalar gradients: cocktail, key bias, admission -> d_means
// and the parameter terms.
__device__ __forceinline__ void adm_token_tail(long long row, int H, const AdmTok& k,
                                               const float* s, const float* cocktail,
                                               const float* params, const float* d_cocktail,
                                               const float* d_bcocktail, const float* d_bbias,
                                               const float* d_badm, float* d_means,
                                               float* param_part) {
  const int j = k.j;
  const float dkb = (j >= 0 && d_bbias) ? d_bbias[k.ej] : 0.f;
  const float dad = (j >= 0 && d_badm) ? d_badm[k.ej] : 0.f;
  float dc[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    dc[c] = (d_cocktail ? d_cocktail[row * 4 + c] : 0.f) +
            ((j >= 0 && d_bcocktail) ? d_bcocktail[k.ej * 4 + c] : 0.f);
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

__device__ __forceinline__ float grad_expr(float g, float q, float dot, float qnorm) {
  return qnorm > kNormEps ? (g - q * dot) / qnorm : g / kNormEps;
}

struct AdmBwdArgs {
  int B, T, H, n;
  const void* expr;
  const void* write;
  const float* stats;
  const float* cocktail;
  const float* params;
  const int* inv;
  const float* key_norm;
  const void* d_query;
  const float* d_cocktail;
  const void* d_keys;
  const void* d_writes;
  const void* d_next;
  const float* d_bcocktail;
  const float* d_bbias;
  const float* d_badm;
  void* d_expr;
  void* d_write;
  float* d_means;
  float* param_part;
};

// Rows whose width is a multiple of 8: 2^lg_tpr threads per token (32..256),
// each holding NV 8-element words of the expression, write and the two
// normalised-gradient rows in registers between the two reductions and the
// output pass.  Every thread of the CTA reaches the reductions.
template <typename Act, typename G, int NV>
__global__ void __launch_bounds__(256) adm_bwd_vec_kernel(AdmBwdArgs a, int lg_tpr) {
  __shared__ float red[8][2];
  const int tpr = 1 << lg_tpr;
  const int sub = threadIdx.x >> lg_tpr, tid = threadIdx.x & (tpr - 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (256 >> lg_tpr) + sub;
  const bool ok = row < (long long)a.B * a.T;
  const int H = a.H;
  const Act* expr = static_cast<const Act*>(a.expr);
  const Act* write = static_cast<const Act*>(a.write);
  const G* dq = static_cast<const G*>(a.d_query);
  const G* dk = static_cast<const G*>(a.d_keys);
  const G* dw = static_cast<const G*>(a.d_writes);
  const G* dn = static_cast<const G*>(a.d_next);
  AdmTok k{};
  float qnorm = 0.f, knorm = 0.f;
  if (ok) {
    k = adm_token(row, a.T, a.n, a.inv);
    k.o = (size_t)row * H;
    qnorm = a.stats[row * 8 + 6];
    knorm = k.j >= 0 ? a.key_norm[k.ej] : 0.f;
  }
  const float qden = fmaxf(qnorm, kNormEps), kden = fmaxf(knorm, kNormEps);
  const bool use_k = ok && k.j >= 0 && dk != nullptr;
  Pack8<Act> xe[NV], xw[NV];
  Pack8<G> gq[NV], gk[NV];
  float dot = 0.f, kdot = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int h = (v * tpr + tid) * 8;
    if (ok && h < H) {
      xe[v] = ld8(expr + k.o + h);
      if (dq) {
        gq[v] = ld8(dq + k.o + h);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(normed(el8(xe[v], i), qden), el8(gq[v], i), dot);
      }
      if (use_k) {
        xw[v] = ld8(write + k.o + h);
        gk[v] = ld8(dk + k.ej * H + h);
#pragma unroll
        for (int i = 0; i < 8; ++i) kdot = fmaf(normed(el8(xw[v], i), kden), el8(gk[v], i), kdot);
      }
    }
  }
  dot = warp_sum(dot);
  kdot = warp_sum(kdot);
  if (tpr > 32) {
    if (lane == 0) {
      red[warp][0] = dot;
      red[warp][1] = kdot;
    }
    __syncthreads();
    const int w0 = (sub << lg_tpr) >> 5, nw = tpr >> 5;
    dot = 0.f;
    kdot = 0.f;
    for (int w = 0; w < nw; ++w) {
      dot += red[w0 + w][0];
      kdot += red[w0 + w][1];
    }
  }
  if (!ok) return;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int h = (v * tpr + tid) * 8;
    if (h >= H) continue;
    float ge[8], gw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ge[i] = dq ? grad_expr(el8(gq[v], i), normed(el8(xe[v], i), qden), dot, qnorm) : 0.f;
      gw[i] = 0.f;
    }
    if (k.j >= 0 && dw) {
      const Pack8<G> g = ld8(dw + k.ej * H + h);
#pragma unroll
      for (int i = 0; i < 8; ++i) gw[i] += el8(g, i);
    }
    if (use_k) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        gw[i] += grad_expr(el8(gk[v], i), normed(el8(xw[v], i), kden), kdot, knorm);
    }
    if (k.jp >= 0 && dn) {
      const Pack8<G> g = ld8(dn + k.ep * H + h);
#pragma unroll
      for (int i = 0; i < 8; ++i) gw[i] += el8(g, i);
    }
    if (k.jl >= 0 && dn) {
      const Pack8<G> g = ld8(dn + k.el * H + h);
#pragma unroll
      for (int i = 0; i < 8; ++i) gw[i] += el8(g, i);
    }
    st8(static_cast<Act*>(a.d_expr) + k.o + h, ge);
    st8(static_cast<Act*>(a.d_write) + k.o + h, gw);
  }
  if (tid == 0)
    adm_token_tail(row, H, k, a.stats + row * 8, a.cocktail, a.params, a.d_cocktail,
                   a.d_bcocktail, a.d_bbias, a.d_badm, a.d_means, a.param_part);
}

// Any width: one warp per token, element by element (the rows are re-read
// from L1/L2 for the output pass).
template <typename Act, typename G>
__global__ void __launch_bounds__(256) adm_bwd_kernel(AdmBwdArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= (long long)a.B * a.T) return;
  const int H = a.H;
  const Act* expr = static_cast<const Act*>(a.expr);
  const Act* write = static_cast<const Act*>(a.write);
  const G* dq = static_cast<const G*>(a.d_query);
  const G* dk = static_cast<const G*>(a.d_keys);
  const G* dw = static_cast<const G*>(a.d_writes);
  const G* dn = static_cast<const G*>(a.d_next);
  Act* d_expr = static_cast<Act*>(a.d_expr);
  Act* d_write = static_cast<Act*>(a.d_write);
  AdmTok k = adm_token(row, a.T, a.n, a.inv);
  k.o = (size_t)row * H;
  const size_t o = k.o;
  const float qnorm = a.stats[row * 8 + 6];
  const float qden = fmaxf(qnorm, kNormEps);
  const float knorm = k.j >= 0 ? a.key_norm[k.ej] : 0.f;
  const float kden = fmaxf(knorm, kNormEps);
  float dot = 0.f;
  if (dq) {
    for (int h = lane; h < H; h += 32)
      dot = fmaf(normed(to_f<Act>(expr[o + h]), qden), to_f<G>(dq[o + h]), dot);
    dot = warp_sum(dot);
  }
  float kdot = 0.f;
  if (k.j >= 0 && dk) {
    for (int h = lane; h < H; h += 32)
      kdot = fmaf(normed(to_f<Act>(write[o + h]), kden), to_f<G>(dk[k.ej * H + h]), kdot);
    kdot = warp_sum(kdot);
  }
  for (int h = lane; h < H; h += 32) {
    const float ge = dq ? grad_expr(to_f<G>(dq[o + h]), normed(to_f<Act>(expr[o + h]), qden),
                                    dot, qnorm)
                        : 0.f;
    d_expr[o + h] = from_f<Act>(ge);
    float gw = 0.f;
    if (k.j >= 0) {
      if (dw) gw += to_f<G>(dw[k.ej * H + h]);
      if (dk)
        gw += grad_expr(to_f<G>(dk[k.ej * H + h]), normed(to_f<Act>(write[o + h]), kden), kdot,
                        knorm);
    }
    if (k.jp >= 0 && dn) gw += to_f<G>(dn[k.ep * H + h]);
    if (k.jl >= 0 && dn) gw += to_f<G>(dn[k.el * H + h]);
    d_write[o + h] = from_f<Act>(gw);
  }
  if (lane == 0)
    adm_token_tail(row, H, k, a.stats + row * 8, a.cocktail, a.params, a.d_cocktail,
                   a.d_bcocktail, a.d_bbias, a.d_badm, a.d_means, a.param_part);
}

template <typename Act, typename G>
void launch_adm_bwd(const AdmBwdArgs& a, cudaStream_t st) {
  const long long rows = (long long)a.B * a.T;
  const int h8 = a.H / 8;
  if ((a.H & 7) == 0 && h8 <= 1024) {
    const int nv = h8 <= 256 ? 1 : (h8 <= 512 ? 2 : 4);
    int lg = 5;
    while ((1 << lg) * nv < h8) ++lg;  // threads per token: 32..256
    const long long per = 256 >> lg;
    const unsigned grid = (unsigned)((rows + per - 1) / per);
    if (nv == 1) adm_bwd_vec_kernel<Act, G, 1><<<grid, 256, 0, st>>>(a, lg);
    else if (nv == 2) adm_bwd_vec_kernel<Act, G, 2><<<grid, 256, 0, st>>>(a, lg);
    else adm_bwd_vec_kernel<Act, G, 4><<<grid, 256, 0, st>>>(a, lg);
  } else {
    adm_bwd_kernel<Act, G><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a);
  }
}

template <typename Act, typename Q>
void launch_stats(int64_t B, int64_t T, int64_t H, const void* e, const void* nv, const void* pl,
                  const void* en, const void* sa, const float* params, void* query, float* kb,
                  float* adm, float* cocktail, float* stats, cudaStream_t st) {
  const unsigned grid = (unsigned)((B * T + 7) / 8);
  adm_stats_kernel<Act, Q><<<grid, 256, 0, st>>>(
      (int)B, (int)T, (int)H, (const Act*)e, (const Act*)nv, (const Act*)pl, (const Act*)en,
      (const Act*)sa, params, (Q*)query, kb, adm, cocktail, stats);
}

template <typename Act, typename K>
void launch_gather(int64_t B, int64_t T, int64_t H, int64_t n, const void* write,
                   const float* key_bias, const float* admission, const float* cocktail,
                   const int64_t* order, const int64_t* counts, void* bank_writes,
                   void* bank_keys, void* next_writes, float* bank_cocktail, float* bank_bias,
                   float* bank_admission, int64_t* bank_idx, void* bank_valid, float* key_norm,
                   cudaStream_t st) {
  const unsigned grid = (unsigned)((B * n + 7) / 8);
  bank_gather_kernel<Act, K><<<grid, 256, 0, st>>>(
      (int)B, (int)T, (int)H, (int)n, (const Act*)write, key_bias, admission, cocktail, order,
      counts, (Act*)bank_writes, (K*)bank_keys, (Act*)next_writes, bank_cocktail, bank_bias,
      bank_admission, bank_idx, (bool*)bank_valid, key_norm);
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;
using dabsn::bf16;

static bool float_code(int c) { return c == DABSN_F32 || c == DABSN_BF16; }

extern "C" int dabsn_admission_fwd(int dtype, int64_t B, int64_t T, int64_t H, int mode,
                                   const void* expression, const void* novelty,
                                   const void* plasticity, const void* energy,
                                   const void* saturation, const float* params,
                                   const float* window, int query_dtype, void* query,
                                   float* key_bias, float* admission, float* cocktail,
                                   float* stats, int64_t* order, int64_t* counts, int* inv,
                                   void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || (mode != 0 && mode != 1)) {
    set_error("admission_fwd: bad sizes or mode (B=%lld T=%lld H=%lld mode=%d)", (long long)B,
              (long long)T, (long long)H, mode);
    return DABSN_ERR_SHAPE;
  }
  if (!float_code(dtype) || !float_code(query_dtype)) {
    set_error("admission_fwd: dtype codes %d / %d", dtype, query_dtype);
    return DABSN_ERR_DTYPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const bool a32 = dtype == DABSN_F32, q32 = query_dtype == DABSN_F32;
  auto go = [&](auto act, auto q) {
    using A = decltype(act);
    using Q = decltype(q);
    launch_stats<A, Q>(B, T, H, expression, novelty, plasticity, energy, saturation, params,
                       query, key_bias, admission, cocktail, stats, st);
  };
  if (a32 && q32) go(float{}, float{});
  else if (a32) go(float{}, bf16{});
  else if (q32) go(bf16{}, float{});
  else go(bf16{}, bf16{});
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
                                 int key_dtype, void* bank_keys, void* next_writes,
                                 float* bank_cocktail, float* bank_bias, float* bank_admission,
                                 int64_t* bank_idx, void* bank_valid, float* key_norm,
                                 void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || n <= 0 || n > T) {
    set_error("bank_gather: bad sizes (B=%lld T=%lld H=%lld n=%lld)", (long long)B, (long long)T,
              (long long)H, (long long)n);
    return DABSN_ERR_SHAPE;
  }
  if (!float_code(dtype) || !float_code(key_dtype)) {
    set_error("bank_gather: dtype codes %d / %d", dtype, key_dtype);
    return DABSN_ERR_DTYPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const bool a32 = dtype == DABSN_F32, k32 = key_dtype == DABSN_F32;
  auto go = [&](auto act, auto kk) {
    using A = decltype(act);
    using K = decltype(kk);
    launch_gather<A, K>(B, T, H, n, write, key_bias, admission, cocktail, order, counts,
                        bank_writes, bank_keys, next_writes, bank_cocktail, bank_bias,
                        bank_admission, bank_idx, bank_valid, key_norm, st);
  };
  if (a32 && k32) go(float{}, float{});
  else if (a32) go(float{}, bf16{});
  else if (k32) go(bf16{}, float{});
  else go(bf16{}, bf16{});
  return launch_status("bank_gather");
}

extern "C" int dabsn_admission_bwd(int dtype, int64_t B, int64_t T, int64_t H, int64_t n,
                                   const void* expression, const void* write, const float* stats,
                                   const float* cocktail, const float* params, const int* inv,
                                   const float* key_norm, int grad_dtype, const void* d_query,
                                   const float* d_cocktail, const void* d_keys,
                                   const void* d_writes, const void* d_next,
                                   const float* d_bank_cocktail, const float* d_bank_bias,
                                   const float* d_bank_admission, void* d_expression,
                                   void* d_write, float* d_means, float* param_part,
                                   void* stream) {
  if (B <= 0 || T <= 0 || H <= 0 || n <= 0 || n > T) {
    set_error("admission_bwd: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  if (!float_code(dtype) || !float_code(grad_dtype) ||
      (dtype == DABSN_F32 && grad_dtype == DABSN_BF16)) {
    set_error("admission_bwd: dtype codes %d / %d (BF16 gradients need BF16 activations)", dtype,
              grad_dtype);
    return DABSN_ERR_DTYPE;
  }
  AdmBwdArgs a{(int)B, (int)T, (int)H, (int)n, expression, write, stats, cocktail, params, inv,
               key_norm, d_query, d_cocktail, d_keys, d_writes, d_next, d_bank_cocktail,
               d_bank_bias, d_bank_admission, d_expression, d_write, d_means, param_part};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32) launch_adm_bwd<float, float>(a, st);
  else if (grad_dtype == DABSN_F32) launch_adm_bwd<bf16, float>(a, st);
  else launch_adm_bwd<bf16, bf16>(a, st);
  return launch_status("admission_bwd");
}
