// Exact three-way admitted read (short / permanent / induction), forward and
// backward, tiled flash-style: the [T, N] score matrices are never stored.
//
// Reference: src/dabsn/kernels/compact_admitted.py:16-80
// (`dense_bmm_three_way_read_exact`, the CUDA training path reached from
// src/dabsn/kernels/triton.py:314-406) and its analytic twin
// src/dabsn/kernels/admitted.py:16-246.  For query row t and bank entry j:
//
//   S_tj = scale * q_t.k_j + key_bias_j + admission_j
//   P_tj = S_tj + cocktail_gain * (c_t . c_j)
//   short_t  = softmax_{j in allow(t)}  (S_t.) . W
//   perm_t   = softmax_{j in allow(t)}  (P_t.) . W
//   induct_t = softmax_{j in induct(t)} (S_t.) . Wnext
//   out_t    = short_gain*short_t + pad_gain*perm_t + induct_gain*induct_t
//
// allow(t) = valid_j & idx_j <= t (seq) | valid_j (field);
// induct(t) = valid_j & idx_j < t (seq) | valid_j & idx_j < T-1 (field).
// A row with no eligible entry reads zero.
//
// Tiles: 32 query rows x 32 bank entries per step, 256 threads.  Score tiles
// are computed 2x2 per thread from float4 shared-memory reads; the value
// products give each warp 4 query rows and each lane a strided set of
// columns.  Entries are skipped tile by tile when no query of the tile may see
// them (their smallest position exceeds the tile's last query).
#include <math_constants.h>

#include <algorithm>
#include <cstdlib>

#include "../../include/dabsn_b200.h"
#include "common.cuh"

namespace dabsn {
namespace {

constexpr int RT = 32;        // query rows per tile
constexpr int NT = 32;        // bank entries per tile
constexpr int RTHREADS = 256;
constexpr int SLD = NT + 1;   // leading dimension of score tiles in smem

struct ReadArgs {
  int B, T, N, H, Hp, ld;  // ld = Hp + 4
  int mode;                // 0 seq, 1 field
  int total_steps;         // for the field induction mask
  const void* q;           // [B,T,H]
  const void* k;           // [B,N,H]
  const void* v;           // [B,N,H]  bank writes
  const void* vn;          // [B,N,H]  next writes
  const void* cq;          // [B,T,4]  query cocktail
  const void* ck;          // [B,N,4]  bank cocktail
  const void* kb;          // [B,N]    key bias
  const void* adm;         // [B,N]    admission
  const float* scale;      // [1]
  const int64_t* idx;      // [B,N]
  const uint8_t* valid;    // [B,N]
  const float* gains;      // [4]: short, pad, induct, cocktail
  // forward outputs
  void* out;               // [B,T,H] activation dtype
  float* o3;               // [B,T,3,H] per-stream normalised reads (saved)
  float* lse;              // [B,T,3] log-sum-exp per stream (+inf: empty row)
  // backward
  const float* gout;       // [B,T,H] FP32 upstream gradient
  float* u3;               // [B,T,3]  gout . o_stream (unscaled)
  void* dq;                // [B,T,H]
  float* dcq;              // [B,T,4]
  void* dk;                // [B,N,H]
  void* dv;                // [B,N,H]
  void* dvn;               // [B,N,H]
  float* dbias;            // [B,N]  gradient of key_bias (= of admission)
  float* dck;              // [B,N,4]
  float* partial_q;        // [B, T/RT, 2]: d scale, d cocktail_gain partials
};

// Row tiles are loaded with several independent global loads in flight per
// thread (a load-then-store loop would wait out one memory latency per
// element).  Rows >= nrows and columns >= H are zero-filled.
constexpr int LOAD_BATCH = 8;

template <typename T>
__device__ __forceinline__ void load_rows_any(float* dst, int ld, const T* src, int row0,
                                              int nrows, int H, int Hp) {
  const int total = RT * Hp;
  for (int base = threadIdx.x; base < total; base += blockDim.x * LOAD_BATCH) {
    float v[LOAD_BATCH];
#pragma unroll
    for (int u = 0; u < LOAD_BATCH; ++u) {
      const int i = base + u * blockDim.x;
      const int r = i / Hp, h = i % Hp;
      v[u] = (i < total && r < nrows && h < H) ? to_f<T>(src[(size_t)(row0 + r) * H + h]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < LOAD_BATCH; ++u) {
      const int i = base + u * blockDim.x;
      if (i < total) dst[(i / Hp) * ld + i % Hp] = v[u];
    }
  }
}

template <typename Act>
__device__ __forceinline__ void load_rows(float* dst, int ld, const Act* src, int row0, int nrows,
                                          int H, int Hp) {
  load_rows_any<Act>(dst, ld, src, row0, nrows, H, Hp);
}

__device__ __forceinline__ void load_rows_f32(float* dst, int ld, const float* src, int row0,
                                              int nrows, int H, int Hp) {
  load_rows_any<float>(dst, ld, src, row0, nrows, H, Hp);
}

// The same rows of three bank arrays (keys, writes, next writes) at once.
template <typename Act>
__device__ __forceinline__ void load_rows3(float* d0, float* d1, float* d2, int ld, const Act* s0,
                                           const Act* s1, const Act* s2, int row0, int nrows,
                                           int H, int Hp) {
  constexpr int NB = LOAD_BATCH / 2;
  const int total = RT * Hp;
  for (int base = threadIdx.x; base < total; base += blockDim.x * NB) {
    float v0[NB], v1[NB], v2[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int i = base + u * blockDim.x;
      const int r = i / Hp, h = i % Hp;
      const bool ok = i < total && r < nrows && h < H;
      const size_t o = (size_t)(row0 + r) * H + h;
      v0[u] = ok ? to_f<Act>(s0[o]) : 0.f;
      v1[u] = ok ? to_f<Act>(s1[o]) : 0.f;
      v2[u] = ok ? to_f<Act>(s2[o]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int i = base + u * blockDim.x;
      if (i < total) {
        const int o = (i / Hp) * ld + i % Hp;
        d0[o] = v0[u];
        d1[o] = v1[u];
        d2[o] = v2[u];
      }
    }
  }
}

// Query rows (activation dtype) and upstream-gradient rows (FP32) at once.
template <typename Act>
__device__ __forceinline__ void load_rows_qg(float* dq, float* dg, int ld, const Act* q,
                                             const float* g, int row0, int nrows, int H, int Hp) {
  constexpr int NB = LOAD_BATCH / 2;
  const int total = RT * Hp;
  for (int base = threadIdx.x; base < total; base += blockDim.x * NB) {
    float v0[NB], v1[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int i = base + u * blockDim.x;
      const int r = i / Hp, h = i % Hp;
      const bool ok = i < total && r < nrows && h < H;
      const size_t o = (size_t)(row0 + r) * H + h;
      v0[u] = ok ? to_f<Act>(q[o]) : 0.f;
      v1[u] = ok ? g[o] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      const int i = base + u * blockDim.x;
      if (i < total) {
        const int o = (i / Hp) * ld + i % Hp;
        dq[o] = v0[u];
        dg[o] = v1[u];
      }
    }
  }
}

// 2x2 tile of A . B^T: rows {r, r+16} of A, rows {c, c+16} of B.
__device__ __forceinline__ void dot2x2(const float* A, const float* Bm, int ld, int Hp, int r, int c,
                                       float o[4]) {
  float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
  const float* a0 = A + r * ld;
  const float* a1 = A + (r + 16) * ld;
  const float* b0 = Bm + c * ld;
  const float* b1 = Bm + (c + 16) * ld;
  for (int h = 0; h < Hp; h += 4) {
    const float4 x0 = *reinterpret_cast<const float4*>(a0 + h);
    const float4 x1 = *reinterpret_cast<const float4*>(a1 + h);
    const float4 y0 = *reinterpret_cast<const float4*>(b0 + h);
    const float4 y1 = *reinterpret_cast<const float4*>(b1 + h);
    a00 = fmaf(x0.x, y0.x, fmaf(x0.y, y0.y, fmaf(x0.z, y0.z, fmaf(x0.w, y0.w, a00))));
    a01 = fmaf(x0.x, y1.x, fmaf(x0.y, y1.y, fmaf(x0.z, y1.z, fmaf(x0.w, y1.w, a01))));
    a10 = fmaf(x1.x, y0.x, fmaf(x1.y, y0.y, fmaf(x1.z, y0.z, fmaf(x1.w, y0.w, a10))));
    a11 = fmaf(x1.x, y1.x, fmaf(x1.y, y1.y, fmaf(x1.z, y1.z, fmaf(x1.w, y1.w, a11))));
  }
  o[0] = a00;
  o[1] = a01;
  o[2] = a10;
  o[3] = a11;
}

struct BankMeta {
  int pos[NT];
  uint8_t ok[NT];
  float bias[NT];
  float c4[NT][4];
};

template <typename Act>
__device__ __forceinline__ void load_bank_meta(BankMeta& m, const ReadArgs& a, int b, int j0) {
  const Act* kb = reinterpret_cast<const Act*>(a.kb);
  const Act* adm = reinterpret_cast<const Act*>(a.adm);
  const Act* ck = reinterpret_cast<const Act*>(a.ck);
  for (int j = threadIdx.x; j < NT; j += blockDim.x) {
    const int jj = j0 + j;
    const bool in = jj < a.N;
    const size_t o = (size_t)b * a.N + jj;
    m.ok[j] = in ? a.valid[o] : 0;
    m.pos[j] = in ? (int)a.idx[o] : 0x7fffffff;
    m.bias[j] = in ? to_f<Act>(kb[o]) + to_f<Act>(adm[o]) : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) m.c4[j][c] = in ? to_f<Act>(ck[o * 4 + c]) : 0.f;
  }
}

__device__ __forceinline__ bool allow_main(const ReadArgs& a, const BankMeta& m, int j, int t) {
  return m.ok[j] && (a.mode == 1 || m.pos[j] <= t);
}
__device__ __forceinline__ bool allow_induct(const ReadArgs& a, const BankMeta& m, int j, int t) {
  return m.ok[j] && (a.mode == 1 ? m.pos[j] < a.total_steps - 1 : m.pos[j] < t);
}

// Smallest position among the valid entries of a bank tile (INT_MAX if none).
__device__ __forceinline__ int tile_min_pos(const BankMeta& m, int* red) {
  if (threadIdx.x < 32) {
    int v = m.ok[threadIdx.x] ? m.pos[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) *red = v;
  }
  __syncthreads();
  return *red;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename Act, int HC>
__global__ void __launch_bounds__(RTHREADS, 1) read_fwd_kernel(const ReadArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * RT;
  const int nq = min(RT, a.T - t0);
  const int ld = a.ld;
  float* Qs = reinterpret_cast<float*>(smem_raw);
  float* Ks = Qs + RT * ld;
  float* Vs = Ks + NT * ld;
  float* Ns = Vs + NT * ld;
  float* Ss = Ns + NT * ld;    // [RT][SLD] short/induct scores
  float* Ps = Ss + RT * SLD;   // [RT][SLD] permanent scores
  float* W3 = Ps + RT * SLD;   // [3][RT][SLD] probabilities
  float* rowst = W3 + 3 * RT * SLD;  // [3][RT] m, [3][RT] l, [3][RT] alpha, [RT][4] cq
  float* m_ = rowst;
  float* l_ = m_ + 3 * RT;
  float* al_ = l_ + 3 * RT;
  float* cq_ = al_ + 3 * RT;
  BankMeta* meta = reinterpret_cast<BankMeta*>(cq_ + 4 * RT);
  int* red = reinterpret_cast<int*>(meta + 1);

  const Act* q = reinterpret_cast<const Act*>(a.q) + (size_t)b * a.T * a.H;
  const Act* k = reinterpret_cast<const Act*>(a.k) + (size_t)b * a.N * a.H;
  const Act* v = reinterpret_cast<const Act*>(a.v) + (size_t)b * a.N * a.H;
  const Act* vn = reinterpret_cast<const Act*>(a.vn) + (size_t)b * a.N * a.H;
  const Act* cq = reinterpret_cast<const Act*>(a.cq);
  const float scale = a.scale[0];
  const float cg = a.gains[3];

  load_rows<Act>(Qs, ld, q, t0, nq, a.H, a.Hp);
  for (int i = threadIdx.x; i < 3 * RT; i += blockDim.x) {
    m_[i] = -CUDART_INF_F;
    l_[i] = 0.f;
  }
  for (int i = threadIdx.x; i < RT * 4; i += blockDim.x) {
    const int r = i / 4, c = i % 4;
    cq_[i] = r < nq ? to_f<Act>(cq[((size_t)b * a.T + t0 + r) * 4 + c]) : 0.f;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.z * HC;  // first 32-column block of this CTA's share of H
  float acc[3][4][HC];
#pragma unroll
  for (int s = 0; s < 3; ++s)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < HC; ++c) acc[s][i][c] = 0.f;

  const int tmax = t0 + nq - 1;
  for (int j0 = 0; j0 < a.N; j0 += NT) {
    __syncthreads();
    load_bank_meta<Act>(*meta, a, b, j0);
    __syncthreads();
    const int minpos = tile_min_pos(*meta, red);
    if (minpos == 0x7fffffff || (a.mode == 0 && minpos > tmax)) continue;
    const int nk = min(NT, a.N - j0);
    load_rows3<Act>(Ks, Vs, Ns, ld, k, v, vn, j0, nk, a.H, a.Hp);
    __syncthreads();
    {
      const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
      float o[4];
      dot2x2(Qs, Ks, ld, a.Hp, r, c, o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = r + (i >> 1) * 16, cc = c + (i & 1) * 16;
        const float qk = round_act<Act>(o[i]);
        const float s = qk * scale + meta->bias[cc];
        float ccv = 0.f;
#pragma unroll
        for (int z = 0; z < 4; ++z) ccv = fmaf(cq_[rr * 4 + z], meta->c4[cc][z], ccv);
        ccv = round_act<Act>(ccv);
        Ss[rr * SLD + cc] = s;
        Ps[rr * SLD + cc] = s + ccv * cg;
      }
    }
    __syncthreads();
    // Online softmax statistics: warp w owns rows 4w..4w+3, lane = entry.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i;
      const int t = t0 + r;
      const bool am = (r < nq) && allow_main(a, *meta, lane, t);
      const bool ai = (r < nq) && allow_induct(a, *meta, lane, t);
      const float sv = Ss[r * SLD + lane];
      const float pv = Ps[r * SLD + lane];
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const bool ok = (s == 2) ? ai : am;
        const float x = ok ? (s == 1 ? pv : sv) : -CUDART_INF_F;
        const float mold = m_[s * RT + r];
        const float mnew = fmaxf(mold, warp_max(x));
        const float pr = ok ? expf(x - mnew) : 0.f;
        const float sum = warp_sum(pr);
        W3[(s * RT + r) * SLD + lane] = pr;
        if (lane == 0) {
          const float alpha = (mnew == -CUDART_INF_F) ? 1.f : expf(mold - mnew);
          al_[s * RT + r] = alpha;
          l_[s * RT + r] = l_[s * RT + r] * alpha + sum;
          m_[s * RT + r] = mnew;
        }
      }
    }
    __syncthreads();
    // Rescale and accumulate P . V for the three streams.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i;
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const float al = al_[s * RT + r];
#pragma unroll
        for (int c = 0; c < HC; ++c) acc[s][i][c] *= al;
      }
    }
    for (int j = 0; j < nk; ++j) {
      float vv[HC], nn[HC];
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        vv[c] = Vs[j * ld + lane + 32 * (cb + c)];
        nn[c] = Ns[j * ld + lane + 32 * (cb + c)];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = warp * 4 + i;
        const float ps = W3[(0 * RT + r) * SLD + j];
        const float pp = W3[(1 * RT + r) * SLD + j];
        const float pi = W3[(2 * RT + r) * SLD + j];
#pragma unroll
        for (int c = 0; c < HC; ++c) {
          acc[0][i][c] = fmaf(ps, vv[c], acc[0][i][c]);
          acc[1][i][c] = fmaf(pp, vv[c], acc[1][i][c]);
          acc[2][i][c] = fmaf(pi, nn[c], acc[2][i][c]);
        }
      }
    }
  }
  __syncthreads();
  const float g0 = a.gains[0], g1 = a.gains[1], g2 = a.gains[2];
  Act* out = reinterpret_cast<Act*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
    if (r >= nq) continue;
    const size_t row = (size_t)b * a.T + t0 + r;
    float inv[3];
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const float l = l_[s * RT + r];
      inv[s] = l > 0.f ? 1.0f / l : 0.f;
    }
#pragma unroll
    for (int c = 0; c < HC; ++c) {
      const int h = lane + 32 * (cb + c);
      if (h < a.H) {
        const float os = acc[0][i][c] * inv[0];
        const float op = acc[1][i][c] * inv[1];
        const float oi = acc[2][i][c] * inv[2];
        out[row * a.H + h] = from_f<Act>(g0 * os + g1 * op + g2 * oi);
        float* o3 = a.o3 + row * 3 * a.H + h;
        o3[0] = os;
        o3[a.H] = op;
        o3[2 * a.H] = oi;
      }
    }
    if (lane < 3 && blockIdx.z == 0) {
      const float l = l_[lane * RT + r];
      a.lse[row * 3 + lane] = l > 0.f ? m_[lane * RT + r] + logf(l) : CUDART_INF_F;
    }
  }
}

// ---------------------------------------------------------------------------
// Backward, query-parallel: dq, d(query cocktail), u = gout . o_stream and the
// scalar partials for scale and cocktail_gain.
// ---------------------------------------------------------------------------
template <typename Act, int HC>
__global__ void __launch_bounds__(RTHREADS, 1) read_bwd_q_kernel(const ReadArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * RT;
  const int nq = min(RT, a.T - t0);
  const int ld = a.ld;
  float* Qs = reinterpret_cast<float*>(smem_raw);
  float* Gs = Qs + RT * ld;   // gout rows
  float* Ks = Gs + RT * ld;
  float* Vs = Ks + NT * ld;
  float* Ns = Vs + NT * ld;
  float* DS = Ns + NT * ld;   // [RT][SLD] dS_total
  float* DP = DS + RT * SLD;  // [RT][SLD] dS_perm
  float* lse_ = DP + RT * SLD;  // [3][RT]
  float* D_ = lse_ + 3 * RT;    // [3][RT]
  float* cq_ = D_ + 3 * RT;     // [RT][4]
  float* redf = cq_ + 4 * RT;   // [2 * 8]
  BankMeta* meta = reinterpret_cast<BankMeta*>(redf + 16);
  int* red = reinterpret_cast<int*>(meta + 1);

  const Act* q = reinterpret_cast<const Act*>(a.q) + (size_t)b * a.T * a.H;
  const Act* k = reinterpret_cast<const Act*>(a.k) + (size_t)b * a.N * a.H;
  const Act* v = reinterpret_cast<const Act*>(a.v) + (size_t)b * a.N * a.H;
  const Act* vn = reinterpret_cast<const Act*>(a.vn) + (size_t)b * a.N * a.H;
  const Act* cq = reinterpret_cast<const Act*>(a.cq);
  const float scale = a.scale[0];
  const float g0 = a.gains[0], g1 = a.gains[1], g2 = a.gains[2], cg = a.gains[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.z * HC;  // first 32-column block of this CTA's share of H

  load_rows_qg<Act>(Qs, Gs, ld, q, a.gout + (size_t)b * a.T * a.H, t0, nq, a.H, a.Hp);
  for (int i = threadIdx.x; i < RT * 4; i += blockDim.x) {
    const int r = i / 4, c = i % 4;
    cq_[i] = r < nq ? to_f<Act>(cq[((size_t)b * a.T + t0 + r) * 4 + c]) : 0.f;
  }
  __syncthreads();
  // u_s = gout . o_s per row (warp w: rows 4w..4w+3); D_s = gain_s * u_s.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
    float u[3] = {0.f, 0.f, 0.f};
    if (r < nq) {
      const size_t row = (size_t)b * a.T + t0 + r;
      for (int h = lane; h < a.H; h += 32) {
        const float gv = Gs[r * ld + h];
        const float* o3 = a.o3 + row * 3 * a.H + h;
        u[0] = fmaf(gv, o3[0], u[0]);
        u[1] = fmaf(gv, o3[a.H], u[1]);
        u[2] = fmaf(gv, o3[2 * a.H], u[2]);
      }
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) u[s] = warp_sum(u[s]);
    if (lane < 3) {
      const float us = lane == 0 ? u[0] : (lane == 1 ? u[1] : u[2]);
      const float gs = lane == 0 ? g0 : (lane == 1 ? g1 : g2);
      D_[lane * RT + r] = gs * us;
      lse_[lane * RT + r] =
          r < nq ? a.lse[((size_t)b * a.T + t0 + r) * 3 + lane] : CUDART_INF_F;
      if (r < nq && blockIdx.z == 0) a.u3[((size_t)b * a.T + t0 + r) * 3 + lane] = us;
    }
  }
  float dqa[4][HC];
  float dcz[4];  // lanes 0..3: cocktail component z = lane of rows 4w..4w+3
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int c = 0; c < HC; ++c) dqa[i][c] = 0.f;
    dcz[i] = 0.f;
  }
  float dscale = 0.f, dcg = 0.f;
  const int tmax = t0 + nq - 1;
  for (int j0 = 0; j0 < a.N; j0 += NT) {
    __syncthreads();
    load_bank_meta<Act>(*meta, a, b, j0);
    __syncthreads();
    const int minpos = tile_min_pos(*meta, red);
    if (minpos == 0x7fffffff || (a.mode == 0 && minpos > tmax)) continue;
    const int nk = min(NT, a.N - j0);
    load_rows3<Act>(Ks, Vs, Ns, ld, k, v, vn, j0, nk, a.H, a.Hp);
    __syncthreads();
    {
      const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
      float qk[4], gv[4], gn[4];
      dot2x2(Qs, Ks, ld, a.Hp, r, c, qk);
      dot2x2(Gs, Vs, ld, a.Hp, r, c, gv);
      dot2x2(Gs, Ns, ld, a.Hp, r, c, gn);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = r + (i >> 1) * 16, cc = c + (i & 1) * 16;
        const int t = t0 + rr;
        const float qkr = round_act<Act>(qk[i]);
        const float s = qkr * scale + meta->bias[cc];
        float ccv = 0.f;
#pragma unroll
        for (int z = 0; z < 4; ++z) ccv = fmaf(cq_[rr * 4 + z], meta->c4[cc][z], ccv);
        ccv = round_act<Act>(ccv);
        const float pv = s + ccv * cg;
        const bool live = rr < nq;
        const bool am = live && allow_main(a, *meta, cc, t);
        const bool ai = live && allow_induct(a, *meta, cc, t);
        const float ps = am ? expf(s - lse_[0 * RT + rr]) : 0.f;
        const float pp = am ? expf(pv - lse_[1 * RT + rr]) : 0.f;
        const float pi = ai ? expf(s - lse_[2 * RT + rr]) : 0.f;
        const float ds_s = ps * (g0 * gv[i] - D_[0 * RT + rr]);
        const float ds_p = pp * (g1 * gv[i] - D_[1 * RT + rr]);
        const float ds_i = pi * (g2 * gn[i] - D_[2 * RT + rr]);
        const float dst = ds_s + ds_p + ds_i;
        DS[rr * SLD + cc] = dst;
        DP[rr * SLD + cc] = ds_p;
        dscale = fmaf(dst, qkr, dscale);
        dcg = fmaf(ds_p, ccv, dcg);
      }
    }
    __syncthreads();
    // dq[r] += scale * sum_j dS[r][j] k_j ; dcq[r] += cg * sum_j dSp[r][j] c_j
    for (int j = 0; j < nk; ++j) {
      float kk[HC];
#pragma unroll
      for (int c = 0; c < HC; ++c) kk[c] = Ks[j * ld + lane + 32 * (cb + c)];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = warp * 4 + i;
        const float d = DS[r * SLD + j];
#pragma unroll
        for (int c = 0; c < HC; ++c) dqa[i][c] = fmaf(d, kk[c], dqa[i][c]);
      }
    }
    if (lane < 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = warp * 4 + i;
        float sacc = 0.f;
        for (int j = 0; j < nk; ++j) sacc = fmaf(DP[r * SLD + j], meta->c4[j][lane], sacc);
        dcz[i] += sacc;
      }
    }
  }
  Act* dq = reinterpret_cast<Act*>(a.dq);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
    if (r >= nq) continue;
    const size_t row = (size_t)b * a.T + t0 + r;
#pragma unroll
    for (int c = 0; c < HC; ++c) {
      const int h = lane + 32 * (cb + c);
      if (h < a.H) dq[row * a.H + h] = from_f<Act>(scale * dqa[i][c]);
    }
    if (lane < 4 && blockIdx.z == 0) a.dcq[row * 4 + lane] = cg * dcz[i];
  }
  // Block-reduce the two scalar partials.
  dscale = warp_sum(dscale);
  dcg = warp_sum(dcg);
  __syncthreads();
  if (lane == 0) {
    redf[warp] = dscale;
    redf[8 + warp] = dcg;
  }
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.z == 0) {
    float s0 = 0.f, s1 = 0.f;
    for (int w = 0; w < 8; ++w) {
      s0 += redf[w];
      s1 += redf[8 + w];
    }
    float* dst = a.partial_q + ((size_t)b * gridDim.x + blockIdx.x) * 2;
    dst[0] = s0;
    dst[1] = s1;
  }
}

// ---------------------------------------------------------------------------
// Backward, bank-parallel: dk, dv (writes), dvn (next writes), d bias and
// d(bank cocktail).
// ---------------------------------------------------------------------------
template <typename Act, int HC>
__global__ void __launch_bounds__(RTHREADS, 1) read_bwd_kv_kernel(const ReadArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.y;
  const int j0 = blockIdx.x * NT;
  const int nk = min(NT, a.N - j0);
  const int ld = a.ld;
  float* Ks = reinterpret_cast<float*>(smem_raw);
  float* Vs = Ks + NT * ld;
  float* Ns = Vs + NT * ld;
  float* Qs = Ns + NT * ld;
  float* Gs = Qs + RT * ld;
  float* DS = Gs + RT * ld;    // [RT][SLD] dS_total
  float* PA = DS + RT * SLD;   // [RT][SLD] g0*Ps + g1*Pp
  float* PI = PA + RT * SLD;   // [RT][SLD] g2*Pi
  float* DP = PI + RT * SLD;   // [RT][SLD] dS_perm
  float* lse_ = DP + RT * SLD; // [3][RT]
  float* D_ = lse_ + 3 * RT;   // [3][RT]
  float* cq_ = D_ + 3 * RT;    // [RT][4]
  BankMeta* meta = reinterpret_cast<BankMeta*>(cq_ + 4 * RT);
  int* red = reinterpret_cast<int*>(meta + 1);

  const Act* q = reinterpret_cast<const Act*>(a.q) + (size_t)b * a.T * a.H;
  const Act* k = reinterpret_cast<const Act*>(a.k) + (size_t)b * a.N * a.H;
  const Act* v = reinterpret_cast<const Act*>(a.v) + (size_t)b * a.N * a.H;
  const Act* vn = reinterpret_cast<const Act*>(a.vn) + (size_t)b * a.N * a.H;
  const Act* cq = reinterpret_cast<const Act*>(a.cq);
  const float scale = a.scale[0];
  const float g0 = a.gains[0], g1 = a.gains[1], g2 = a.gains[2], cg = a.gains[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.z * HC;  // first 32-column block of this CTA's share of H

  load_bank_meta<Act>(*meta, a, b, j0);
  load_rows3<Act>(Ks, Vs, Ns, ld, k, v, vn, j0, nk, a.H, a.Hp);
  __syncthreads();
  const int minpos = tile_min_pos(*meta, red);

  // Warp w accumulates bank entries 4w..4w+3; lane owns columns lane+32c.
  float dka[4][HC], dva[4][HC], dna[4][HC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < HC; ++c) dka[i][c] = dva[i][c] = dna[i][c] = 0.f;
  float dbias_acc = 0.f;  // thread (entry = lane), summed over row groups
  float dck_acc[4] = {0.f, 0.f, 0.f, 0.f};

  if (minpos != 0x7fffffff) {
    // positions may be negative (bank entries before a query window): those
    // entries are visible from the first query row on
    const int tstart = a.mode == 0 ? max(0, (minpos / RT) * RT) : 0;
    for (int t0 = tstart; t0 < a.T; t0 += RT) {
      const int nq = min(RT, a.T - t0);
      __syncthreads();
      load_rows_qg<Act>(Qs, Gs, ld, q, a.gout + (size_t)b * a.T * a.H, t0, nq, a.H, a.Hp);
      for (int i = threadIdx.x; i < RT * 4; i += blockDim.x) {
        const int r = i / 4, c = i % 4;
        cq_[i] = r < nq ? to_f<Act>(cq[((size_t)b * a.T + t0 + r) * 4 + c]) : 0.f;
      }
      for (int i = threadIdx.x; i < 3 * RT; i += blockDim.x) {
        const int s = i / RT, r = i % RT;
        const size_t row = (size_t)b * a.T + t0 + r;
        const float gs = s == 0 ? g0 : (s == 1 ? g1 : g2);
        lse_[i] = r < nq ? a.lse[row * 3 + s] : CUDART_INF_F;
        D_[i] = r < nq ? gs * a.u3[row * 3 + s] : 0.f;
      }
      __syncthreads();
      {
        const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
        float qk[4], gv[4], gn[4];
        dot2x2(Qs, Ks, ld, a.Hp, r, c, qk);
        dot2x2(Gs, Vs, ld, a.Hp, r, c, gv);
        dot2x2(Gs, Ns, ld, a.Hp, r, c, gn);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = r + (i >> 1) * 16, cc = c + (i & 1) * 16;
          const int t = t0 + rr;
          const float qkr = round_act<Act>(qk[i]);
          const float s = qkr * scale + meta->bias[cc];
          float ccv = 0.f;
#pragma unroll
          for (int z = 0; z < 4; ++z) ccv = fmaf(cq_[rr * 4 + z], meta->c4[cc][z], ccv);
          ccv = round_act<Act>(ccv);
          const float pv = s + ccv * cg;
          const bool live = rr < nq;
          const bool am = live && allow_main(a, *meta, cc, t);
          const bool ai = live && allow_induct(a, *meta, cc, t);
          const float ps = am ? expf(s - lse_[0 * RT + rr]) : 0.f;
          const float pp = am ? expf(pv - lse_[1 * RT + rr]) : 0.f;
          const float pi = ai ? expf(s - lse_[2 * RT + rr]) : 0.f;
          const float ds_s = ps * (g0 * gv[i] - D_[0 * RT + rr]);
          const float ds_p = pp * (g1 * gv[i] - D_[1 * RT + rr]);
          const float ds_i = pi * (g2 * gn[i] - D_[2 * RT + rr]);
          DS[rr * SLD + cc] = ds_s + ds_p + ds_i;
          DP[rr * SLD + cc] = ds_p;
          PA[rr * SLD + cc] = g0 * ps + g1 * pp;
          PI[rr * SLD + cc] = g2 * pi;
        }
      }
      __syncthreads();
      for (int r = 0; r < nq; ++r) {
        float qq[HC], gg[HC];
#pragma unroll
        for (int c = 0; c < HC; ++c) {
          qq[c] = Qs[r * ld + lane + 32 * (cb + c)];
          gg[c] = Gs[r * ld + lane + 32 * (cb + c)];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = warp * 4 + i;
          const float d = DS[r * SLD + j];
          const float pa = PA[r * SLD + j];
          const float pi = PI[r * SLD + j];
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            dka[i][c] = fmaf(d, qq[c], dka[i][c]);
            dva[i][c] = fmaf(pa, gg[c], dva[i][c]);
            dna[i][c] = fmaf(pi, gg[c], dna[i][c]);
          }
        }
      }
      if (warp == 0) {
        for (int r = 0; r < nq; ++r) {
          const float d = DS[r * SLD + lane];
          const float dp = DP[r * SLD + lane];
          dbias_acc += d;
#pragma unroll
          for (int z = 0; z < 4; ++z) dck_acc[z] = fmaf(dp, cq_[r * 4 + z], dck_acc[z]);
        }
      }
    }
  }
  Act* dk = reinterpret_cast<Act*>(a.dk);
  Act* dv = reinterpret_cast<Act*>(a.dv);
  Act* dvn = reinterpret_cast<Act*>(a.dvn);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = warp * 4 + i;
    if (j >= nk) continue;
    const size_t row = (size_t)b * a.N + j0 + j;
#pragma unroll
    for (int c = 0; c < HC; ++c) {
      const int h = lane + 32 * (cb + c);
      if (h < a.H) {
        dk[row * a.H + h] = from_f<Act>(scale * dka[i][c]);
        dv[row * a.H + h] = from_f<Act>(dva[i][c]);
        dvn[row * a.H + h] = from_f<Act>(dna[i][c]);
      }
    }
  }
  if (warp == 0 && lane < nk && blockIdx.z == 0) {
    const size_t row = (size_t)b * a.N + j0 + lane;
    a.dbias[row] = dbias_acc;
#pragma unroll
    for (int z = 0; z < 4; ++z) a.dck[row * 4 + z] = cg * dck_acc[z];
  }
}

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

size_t fwd_smem(int ld) {
  return sizeof(float) * ((size_t)RT * ld + 3 * (size_t)NT * ld + 5 * RT * SLD + 9 * RT + 4 * RT) +
         sizeof(BankMeta) + 16;
}
size_t bwdq_smem(int ld) {
  return sizeof(float) * (2 * (size_t)RT * ld + 3 * (size_t)NT * ld + 2 * RT * SLD + 6 * RT +
                          4 * RT + 16) +
         sizeof(BankMeta) + 16;
}
size_t bwdkv_smem(int ld) {
  return sizeof(float) * (3 * (size_t)NT * ld + 2 * (size_t)RT * ld + 4 * RT * SLD + 6 * RT +
                          4 * RT) +
         sizeof(BankMeta) + 16;
}

template <typename Kern>
int launch_read(Kern kernel, dim3 grid, size_t smem, const ReadArgs& a, cudaStream_t st,
                const char* what) {
  if (smem > 227 * 1024) {
    set_error("%s: hidden width %d needs %zu bytes of shared memory", what, a.H, smem);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (!kernel_prepared((const void*)kernel, (int)smem)) return DABSN_ERR_LAUNCH;
  kernel<<<grid, RTHREADS, smem, st>>>(a);
  return launch_status(what);
}

// HC = 32-column blocks of H per thread.  When one CTA per (sequence, tile)
// would leave most SMs idle (short sequences, small banks), the H columns of
// the value / gradient accumulations are split over two CTAs (grid z): both
// compute the full-width scores and softmax, each accumulates and writes half
// of the columns, and only z = 0 writes the per-row and per-entry outputs
// (DABSN_B200_READ_SPLIT=0 turns the split off).
template <typename Act, int HC>
int read_launch(int which, const ReadArgs& a, cudaStream_t st, int split) {
  if (which == 0) {
    dim3 grid((a.T + RT - 1) / RT, a.B, split);
    return launch_read(read_fwd_kernel<Act, HC>, grid, fwd_smem(a.ld), a, st, "read_fwd");
  }
  dim3 gq((a.T + RT - 1) / RT, a.B, split);
  int rc = launch_read(read_bwd_q_kernel<Act, HC>, gq, bwdq_smem(a.ld), a, st, "read_bwd_q");
  if (rc != DABSN_OK) return rc;
  dim3 gk((a.N + NT - 1) / NT, a.B, split);
  return launch_read(read_bwd_kv_kernel<Act, HC>, gk, bwdkv_smem(a.ld), a, st, "read_bwd_kv");
}

template <typename Act, int HC>
int read_dispatch(int which, const ReadArgs& a, cudaStream_t st) {
  const char* e = getenv("DABSN_B200_READ_SPLIT");  // "0": never split
  if constexpr (HC >= 2) {
    if (e && e[0] == '0') return read_launch<Act, HC>(which, a, st, 1);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
    const long long ctas = (long long)a.B * std::max((a.T + RT - 1) / RT, (a.N + NT - 1) / NT);
    if (2 * ctas <= sms) return read_launch<Act, HC / 2>(which, a, st, 2);
  }
  return read_launch<Act, HC>(which, a, st, 1);
}

template <typename Act>
int read_run(int which, ReadArgs& a, cudaStream_t st) {
  if (a.H <= 32) return read_dispatch<Act, 1>(which, a, st);
  if (a.H <= 64) return read_dispatch<Act, 2>(which, a, st);
  if (a.H <= 128) return read_dispatch<Act, 4>(which, a, st);
  if (a.H <= 256) return read_dispatch<Act, 8>(which, a, st);
  set_error("three-way read: hidden width %d > 256 is not supported by the SIMT read", a.H);
  return DABSN_ERR_UNSUPPORTED;
}

int read_entry(int which, int dtype, ReadArgs& a, void* stream) {
  if (a.B < 0 || a.T < 0 || a.N < 0 || a.H <= 0) {
    set_error("three-way read: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  a.Hp = round_up(a.H, 32);
  a.ld = a.Hp + 4;
  if (a.B == 0 || a.T == 0) return DABSN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32) return read_run<float>(which, a, st);
  if (dtype == DABSN_BF16) return read_run<__nv_bfloat16>(which, a, st);
  set_error("three-way read: unsupported dtype %d", dtype);
  return DABSN_ERR_DTYPE;
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int dabsn_read_fwd(int dtype, int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                              int64_t total_steps, const void* query, const void* bank_keys,
                              const void* bank_writes, const void* next_writes,
                              const void* cocktail, const void* bank_cocktail,
                              const void* bank_key_bias, const void* bank_admission,
                              const float* scale, const int64_t* bank_idx,
                              const uint8_t* bank_valid, const float* gains, void* out,
                              float* streams, float* lse, void* stream) {
  ReadArgs a = {};
  a.B = (int)B;
  a.T = (int)T;
  a.N = (int)N;
  a.H = (int)H;
  a.mode = mode;
  a.total_steps = (int)total_steps;
  a.q = query;
  a.k = bank_keys;
  a.v = bank_writes;
  a.vn = next_writes;
  a.cq = cocktail;
  a.ck = bank_cocktail;
  a.kb = bank_key_bias;
  a.adm = bank_admission;
  a.scale = scale;
  a.idx = bank_idx;
  a.valid = bank_valid;
  a.gains = gains;
  a.out = out;
  a.o3 = streams;
  a.lse = lse;
  return read_entry(0, dtype, a, stream);
}

extern "C" int dabsn_read_bwd(int dtype, int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                              int64_t total_steps, const void* query, const void* bank_keys,
                              const void* bank_writes, const void* next_writes,
                              const void* cocktail, const void* bank_cocktail,
                              const void* bank_key_bias, const void* bank_admission,
                              const float* scale, const int64_t* bank_idx,
                              const uint8_t* bank_valid, const float* gains,
                              const float* streams, const float* lse, const float* gout,
                              float* u3, void* dquery, float* dcocktail, void* dkeys,
                              void* dwrites, void* dnext, float* dbias, float* dbank_cocktail,
                              float* partial, void* stream) {
  ReadArgs a = {};
  a.B = (int)B;
  a.T = (int)T;
  a.N = (int)N;
  a.H = (int)H;
  a.mode = mode;
  a.total_steps = (int)total_steps;
  a.q = query;
  a.k = bank_keys;
  a.v = bank_writes;
  a.vn = next_writes;
  a.cq = cocktail;
  a.ck = bank_cocktail;
  a.kb = bank_key_bias;
  a.adm = bank_admission;
  a.scale = scale;
  a.idx = bank_idx;
  a.valid = bank_valid;
  a.gains = gains;
  a.o3 = const_cast<float*>(streams);
  a.lse = const_cast<float*>(lse);
  a.gout = gout;
  a.u3 = u3;
  a.dq = dquery;
  a.dcq = dcocktail;
  a.dk = dkeys;
  a.dv = dwrites;
  a.dvn = dnext;
  a.dbias = dbias;
  a.dck = dbank_cocktail;
  a.partial_q = partial;
  return read_entry(1, dtype, a, stream);
}
