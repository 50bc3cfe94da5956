// Three-way admitted read for wide states (BF16, H > 256) on tensor cores.
//
// Reference: src/dabsn/kernels/compact_admitted.py:16-80
// (`dense_bmm_three_way_read_exact`), the path the reference trains through
// under BF16 autocast: BF16 batched products with FP32 accumulation, scores and
// softmax in FP32, the softmax weights rounded to BF16 for the value products.
// Same mathematics as read.cu:
//
//   C_tj = bf16(q_t . k_j)                      (stored, [B, T, Np] BF16)
//   S_tj = scale * C_tj + key_bias_j + admission_j
//   P_tj = S_tj + cocktail_gain * bf16(c_t . c_j)
//   out_t = sum_j (g_s softmax_allow(S)_tj + g_p softmax_allow(P)_tj) W_j
//         + sum_j  g_i softmax_induct(S)_tj Wnext_j
//
// At H >= 512 every score costs 2H multiply-adds and every value product 2H
// more, so the read is a chain of batched BF16 GEMMs around two row kernels
// that own the softmaxes.  The GEMMs run on the tcgen05 tensor cores with
// TMA-staged operands and TMEM accumulators (tc_gemm.cuh); the mma.sync
// kernel below (m16n8k16, 128 x 128 x 32 CTA tiles, three-stage cp.async
// pipeline) is kept behind DABSN_B200_TCGEN05=0 as the cross-check:
//
//   forward : prep (bank positions / biases / cocktails, per-32-entry minimum
//             position) -> C = Q K^T -> row softmax (log-sum-exps, BF16
//             weights Pw = g_s p_s + g_p p_p and Pi = g_i p_i)
//             -> out = Pw W + Pi Wnext (one GEMM over both pairs)
//   backward: prep -> G = gout W^T, Gn = gout Wnext^T -> row backward
//             (dC = bf16(scale dS), Pw / Pi over G / Gn, row and column
//             partials) -> column reduction -> dQ = dC K
//             -> dK = dC^T Q, dW = Pw^T gout, dWnext = Pi^T gout
//
// The short and permanent streams read the same values, so their weights are
// combined before the value product (two value GEMMs instead of three; the
// BF16 rounding of each stream's output is replaced by one rounding of the
// sum).  Causal structure (seq mode) is used at tile granularity: a score tile
// whose bank entries all sit after its last query is never computed, and the
// value / gradient GEMMs skip the k-tiles that cannot contribute.  Entries of
// skipped score tiles are never read as numbers: the row kernels select on
// the masks before using a value and write every weight / gradient entry of
// their rows (zeros where masked), so the GEMM operands are always defined.
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "../../include/dabsn_b200.h"
#include "common.cuh"
#include "tc_gemm.cuh"
#include "tc_mma.cuh"

namespace dabsn {
namespace {

using tc::bf16;

constexpr int GBM = 128, GBN = 128, GBK = 32, GSTAGES = 3, GTHREADS = 256;
constexpr int ROW_LD = GBK + 8;   // [rows][k] tile row (80 B: conflict-free ldmatrix)
constexpr int COL_LD = GBM + 8;   // [k][cols] tile row (272 B)
constexpr int TILE_ELEMS = (GBM * ROW_LD > GBK * COL_LD) ? GBM * ROW_LD : GBK * COL_LD;
constexpr int MAX_KT = 1024;      // live k-tile list capacity
constexpr size_t GEMM_SMEM = (size_t)2 * GSTAGES * TILE_ELEMS * 2 + MAX_KT * 4;

enum Layout { L_NT = 0, L_NN = 1, L_TN = 2 };
enum Skip { SKIP_NONE = 0, SKIP_OUT_TILE = 1, SKIP_K_BANK = 2, SKIP_K_TIME = 3 };

// C[b] = A[b] op B[b] (+ A2[b] op B2[b]) for one of up to three problems that
// share M, N, K and the layout.
//   L_NT: A [M][K], B [N][K]      (C = A B^T)
//   L_NN: A [M][K], B [K][N]      (C = A B)
//   L_TN: A [K][M], B [K][N]      (C = A^T B)
struct GemmProb {
  const bf16* A;
  const bf16* B;
  const bf16* A2;
  const bf16* B2;
  bf16* C;
  long long sA, sB, sC;  // per-batch strides in elements
  int lda, ldb, ldc;
};

struct GemmArgs {
  GemmProb p[3];
  int nprob;
  int M, N, K;
  int skip;
  const int* jmin32;  // [B][ldj] smallest admitted position per 32 bank entries
  int ldj;
  int T;              // query rows (causal bound)
};

template <int LAYOUT>
__global__ void __launch_bounds__(GTHREADS) read_gemm_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sA = (bf16*)smem_raw;
  bf16* sB = sA + GSTAGES * TILE_ELEMS;
  int* klist = (int*)(sB + GSTAGES * TILE_ELEMS);
  __shared__ int s_nlive;

  const int prob = blockIdx.z % a.nprob, b = blockIdx.z / a.nprob;
  const GemmProb P = a.p[prob];
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkt1 = (a.K + GBK - 1) / GBK;
  const int nkt = P.A2 ? 2 * nkt1 : nkt1;
  const int* jm = a.jmin32 ? a.jmin32 + (size_t)b * a.ldj : nullptr;
  const int t_last = min(m0 + GBM - 1, a.T - 1);

  if (a.skip == SKIP_OUT_TILE) {
    // rows are queries, columns bank entries: dead when every entry of the
    // column block sits after the block's last query.
    int mn = INT_MAX;
#pragma unroll
    for (int q = 0; q < GBN / 32; ++q) {
      const int c = n0 / 32 + q;
      if (c < a.ldj) mn = min(mn, jm[c]);
    }
    if (mn > t_last) return;
  }
  int jmin_rows = 0;
  if (a.skip == SKIP_K_TIME) {
    // rows are bank entries, k runs over queries t >= their positions
    jmin_rows = INT_MAX;
#pragma unroll
    for (int q = 0; q < GBM / 32; ++q) {
      const int c = m0 / 32 + q;
      if (c < a.ldj) jmin_rows = min(jmin_rows, jm[c]);
    }
  }
  if (warp == 0) {
    int cnt = 0;
    for (int base = 0; base < nkt; base += 32) {
      const int kt = base + lane;
      bool live = kt < nkt;
      if (live) {
        const int k1 = kt < nkt1 ? kt : kt - nkt1;
        if (a.skip == SKIP_K_BANK) live = jm[k1] <= t_last;
        else if (a.skip == SKIP_K_TIME) live = (long long)k1 * GBK + GBK - 1 >= (long long)jmin_rows;
      }
      const unsigned mask = __ballot_sync(0xffffffffu, live);
      if (live) klist[cnt + __popc(mask & ((1u << lane) - 1u))] = kt;
      cnt += __popc(mask);
    }
    if (lane == 0) s_nlive = cnt;
  }
  __syncthreads();
  const int nlive = s_nlive;

  auto load = [&](int stage, int kt) {
    const bool second = kt >= nkt1;
    const int k0 = (second ? kt - nkt1 : kt) * GBK;
    const bf16* A = (second ? P.A2 : P.A) + (size_t)b * P.sA;
    const bf16* B = (second ? P.B2 : P.B) + (size_t)b * P.sB;
    bf16* dA = sA + stage * TILE_ELEMS;
    bf16* dB = sB + stage * TILE_ELEMS;
#pragma unroll
    for (int c = tid; c < 512; c += GTHREADS) {
      if (LAYOUT == L_TN) {
        const int kr = c >> 4, cc = (c & 15) * 8;
        const int k = k0 + kr, m = m0 + cc;
        const bool ok = k < a.K;
        tc::cp16(dA + kr * COL_LD + cc, ok ? A + (size_t)k * P.lda + m : A, ok);
      } else {
        const int r = c >> 2, kc = (c & 3) * 8;
        const int m = m0 + r, k = k0 + kc;
        const bool ok = m < a.M && k < a.K;
        tc::cp16(dA + r * ROW_LD + kc, ok ? A + (size_t)m * P.lda + k : A, ok);
      }
      if (LAYOUT == L_NT) {
        const int r = c >> 2, kc = (c & 3) * 8;
        const int n = n0 + r, k = k0 + kc;
        const bool ok = n < a.N && k < a.K;
        tc::cp16(dB + r * ROW_LD + kc, ok ? B + (size_t)n * P.ldb + k : B, ok);
      } else {
        const int kr = c >> 4, cc = (c & 15) * 8;
        const int k = k0 + kr, n = n0 + cc;
        const bool ok = k < a.K && n < a.N;
        tc::cp16(dB + kr * COL_LD + cc, ok ? B + (size_t)k * P.ldb + n : B, ok);
      }
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;
  const int wm = warp >> 2, wn = warp & 3;

#pragma unroll
  for (int s = 0; s < GSTAGES - 1; ++s) {
    if (s < nlive) load(s, klist[s]);
    cp_async_commit();
  }
  for (int i = 0; i < nlive; ++i) {
    cp_async_wait<GSTAGES - 2>();
    __syncthreads();
    const int nx = i + GSTAGES - 1;
    if (nx < nlive) load(nx % GSTAGES, klist[nx]);
    cp_async_commit();
    const bf16* tA = sA + (i % GSTAGES) * TILE_ELEMS;
    const bf16* tB = sB + (i % GSTAGES) * TILE_ELEMS;
#pragma unroll
    for (int kk = 0; kk < GBK; kk += 16) {
      uint32_t af[4][4], bfr[2][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        if (LAYOUT == L_TN) {
          const bf16* p = tA + (kk + (lane & 7) + ((lane >> 4) << 3)) * COL_LD + wm * 64 + mt * 16 +
                          ((lane >> 3) & 1) * 8;
          tc::ldsm_x4_t(smem_u32(p), af[mt]);
        } else {
          const bf16* p = tA + (wm * 64 + mt * 16 + (lane & 15)) * ROW_LD + kk + (lane >> 4) * 8;
          tc::ldsm_x4(smem_u32(p), af[mt]);
        }
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        if (LAYOUT == L_NT) {
          const bf16* p = tB + (wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3)) * ROW_LD + kk +
                          ((lane >> 3) & 1) * 8;
          tc::ldsm_x4(smem_u32(p), bfr[np]);
        } else {
          const bf16* p = tB + (kk + (lane & 15)) * COL_LD + wn * 32 + np * 16 + (lane >> 4) * 8;
          tc::ldsm_x4_t(smem_u32(p), bfr[np]);
        }
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          tc::mma(acc[mt][nt], af[mt], bfr[nt >> 1][(nt & 1) * 2], bfr[nt >> 1][(nt & 1) * 2 + 1]);
    }
  }
  cp_async_wait<0>();

  bf16* C = P.C + (size_t)b * P.sC;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int c = n0 + wn * 32 + nt * 8 + (lane & 3) * 2;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = m0 + wm * 64 + mt * 16 + (lane >> 2) + h * 8;
        if (r >= a.M) continue;
        const float x = acc[mt][nt][2 * h], y = acc[mt][nt][2 * h + 1];
        bf16* dst = C + (size_t)r * P.ldc + c;
        if (c + 1 < a.N) {
          *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(x, y);
        } else if (c < a.N) {
          *dst = __float2bfloat16_rn(x);
        }
      }
    }
}

// ---------------------------------------------------------------------------
// Bank preparation: position (INT_MAX when not admitted), key bias + admission,
// BF16-rounded bank cocktail, and the smallest position per 32 entries.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int warp_min_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(256) read_wide_prep_kernel(int N, int Np, const int64_t* idx,
                                                             const uint8_t* valid, const float* kb,
                                                             const float* adm, const bf16* ck,
                                                             int* pos, float* kba, float4* ckf,
                                                             int* jmin32) {
  const int b = blockIdx.y, j = blockIdx.x * 256 + threadIdx.x;
  int p = INT_MAX;
  float s = 0.f;
  float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
  if (j < N) {
    const size_t o = (size_t)b * N + j;
    if (valid[o]) { const int64_t v = idx[o]; p = v < (int64_t)INT_MAX ? (int)v : INT_MAX - 1; }
    s = kb[o] + adm[o];
    c = make_float4(__bfloat162float(ck[o * 4 + 0]), __bfloat162float(ck[o * 4 + 1]),
                    __bfloat162float(ck[o * 4 + 2]), __bfloat162float(ck[o * 4 + 3]));
  }
  if (j < Np) {
    const size_t o = (size_t)b * Np + j;
    pos[o] = p;
    kba[o] = s;
    ckf[o] = c;
  }
  const int mn = warp_min_i(p);
  if ((threadIdx.x & 31) == 0 && j < Np) jmin32[(size_t)b * (Np / 32) + j / 32] = mn;
}

// ---------------------------------------------------------------------------
// Row kernels
// ---------------------------------------------------------------------------
struct RowArgs {
  int B, T, N, Np, mode, total_steps;
  const bf16* compat;   // [B,T,Np]
  const int* pos;       // [B,Np]
  const float* kba;     // [B,Np]
  const float4* ckf;    // [B,Np]
  const int* jmin32;    // [B,Np/32]
  const bf16* cq;       // [B,T,4]
  const float* scale;   // [1]
  const float* gains;   // [4] short, pad, induct, cocktail
  float* lse;           // [B,T,3]
  bf16* Pw;             // [B,T,Np] (backward: over G)
  bf16* Pi;             // [B,T,Np] (backward: over Gn)
  // backward
  bf16* dC;             // [B,T,Np]
  float* u3;            // [B,T,3]
  float* dcq;           // [B,T,4]
  float* rowpart;       // [B,T,2]: d scale, d cocktail_gain
  float* colpart;       // [B][nrb][Np][5]: d bias, d bank cocktail
  int nrb;
};

struct Online {
  float m = -INFINITY, l = 0.f;
  // adds a group of 8 values with maximum gm (entries at -inf are skipped)
  __device__ __forceinline__ void merge(float gm, const float (&x)[8]) {
    if (gm == -INFINITY) return;
    float gs = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) gs += __expf(x[e] - gm);
    if (gm > m) {
      l = l * __expf(m - gm) + gs;
      m = gm;
    } else {
      l += gs * __expf(gm - m);
    }
  }
  __device__ __forceinline__ void add(float x) {
    if (x > m) {
      l = l * __expf(m - x) + 1.f;
      m = x;
    } else {
      l += __expf(x - m);
    }
  }
  __device__ __forceinline__ float lse_warp() const {
    float M = warp_max(m);
    if (M == -INFINITY) return INFINITY;
    float L = warp_sum(m == -INFINITY ? 0.f : l * __expf(m - M));
    return M + __logf(L);
  }
};

__device__ __forceinline__ void row_masks(int mode, int p, int t, int total, bool& allow,
                                          bool& ind) {
  if (mode == 0) {
    allow = p <= t;
    ind = p < t;
  } else {
    allow = p != INT_MAX;
    ind = p < total - 1;
  }
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

struct Chunk8 {
  float c[8];
  int p[8];
  float kb[8];
  float4 ck[8];
};

__device__ __forceinline__ void load8_bf16(const bf16* src, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ void store8_bf16(bf16* dst, const float (&v)[8]) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
  *reinterpret_cast<uint4*>(dst) = raw;
}

__device__ __forceinline__ void load_chunk(const RowArgs& a, int b, const bf16* crow, int j0,
                                           Chunk8& ch) {
  load8_bf16(crow + j0, ch.c);
  const size_t o = (size_t)b * a.Np + j0;
  const int4 p0 = *reinterpret_cast<const int4*>(a.pos + o);
  const int4 p1 = *reinterpret_cast<const int4*>(a.pos + o + 4);
  const float4 k0 = *reinterpret_cast<const float4*>(a.kba + o);
  const float4 k1 = *reinterpret_cast<const float4*>(a.kba + o + 4);
  ch.p[0] = p0.x; ch.p[1] = p0.y; ch.p[2] = p0.z; ch.p[3] = p0.w;
  ch.p[4] = p1.x; ch.p[5] = p1.y; ch.p[6] = p1.z; ch.p[7] = p1.w;
  ch.kb[0] = k0.x; ch.kb[1] = k0.y; ch.kb[2] = k0.z; ch.kb[3] = k0.w;
  ch.kb[4] = k1.x; ch.kb[5] = k1.y; ch.kb[6] = k1.z; ch.kb[7] = k1.w;
#pragma unroll
  for (int e = 0; e < 8; ++e) ch.ck[e] = a.ckf[o + e];
}

__device__ __forceinline__ float4 load_cq(const bf16* cq) {
  return make_float4(__bfloat162float(cq[0]), __bfloat162float(cq[1]), __bfloat162float(cq[2]),
                     __bfloat162float(cq[3]));
}

__device__ __forceinline__ float cocktail_dot(const float4& a, const float4& b) {
  return bf16_round(a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w);
}

// Row kernels: a CTA owns RB = 64 query rows of one sequence (8 per warp) and
// sweeps the bank in 256-column chunks; lane l owns columns 8l .. 8l + 7 of a
// chunk for all of its warp's rows, so it loads those columns' bank data
// (position, bias, cocktail: 24 B each) once per chunk and reuses it for 8
// rows instead of once per row.  Chunks whose smallest bank position follows
// the block's last query are not computed (their outputs are written as
// zeros, which the consuming GEMMs of other row blocks may read).
constexpr int RB = 64;       // query rows per CTA
constexpr int RPW = RB / 8;  // rows per warp
constexpr int RCC = 256;     // bank columns per chunk (8 per lane)

struct Meta8 {
  int p[8];
  float kb[8];
  float4 ck[8];
};

__device__ __forceinline__ void load_meta(const RowArgs& a, int b, int j0, Meta8& m) {
  const size_t o = (size_t)b * a.Np + j0;
  const int4 p0 = *reinterpret_cast<const int4*>(a.pos + o);
  const int4 p1 = *reinterpret_cast<const int4*>(a.pos + o + 4);
  const float4 k0 = *reinterpret_cast<const float4*>(a.kba + o);
  const float4 k1 = *reinterpret_cast<const float4*>(a.kba + o + 4);
  m.p[0] = p0.x; m.p[1] = p0.y; m.p[2] = p0.z; m.p[3] = p0.w;
  m.p[4] = p1.x; m.p[5] = p1.y; m.p[6] = p1.z; m.p[7] = p1.w;
  m.kb[0] = k0.x; m.kb[1] = k0.y; m.kb[2] = k0.z; m.kb[3] = k0.w;
  m.kb[4] = k1.x; m.kb[5] = k1.y; m.kb[6] = k1.z; m.kb[7] = k1.w;
#pragma unroll
  for (int e = 0; e < 8; ++e) m.ck[e] = a.ckf[o + e];
}

// Whether any entry of columns [c0, c0 + RCC) can be allowed for a query row
// at or before t_last (seq geometry; the field geometry allows every chunk).
__device__ __forceinline__ bool chunk_live(const RowArgs& a, const int* jm, int c0, int t_last) {
  if (a.mode != 0) return true;
  return geom::groups_live(jm, a.Np >> 5, c0 >> 5, (c0 + RCC) >> 5, t_last);
}

// Last query row of the 128-row GEMM row tile holding this CTA's rows.  The
// GEMMs that read the row kernels' [B, T, Np] planes skip the K slices (and
// rows of bank tiles) that are dead for a whole 128-row tile, and a chunk
// dead for that tile holds only such slices, so the planes there are never
// read and are not written.
__device__ __forceinline__ int gemm_tile_last(const RowArgs& a) {
  return geom::row_tile_last((int)(blockIdx.x * RB), a.T, 128);
}

// Log-sum-exps of the three streams, then the BF16 value-product weights for
// the whole row (zeros where masked).
__global__ void __launch_bounds__(256, 2) read_wide_softmax_kernel(const RowArgs a) {
  __shared__ float4 s_cq[RB];  // per-row constants (warp-uniform reads)
  __shared__ float s_l[RB][3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, t0 = blockIdx.x * RB + warp * RPW;
  const int t_last_blk = min((int)(blockIdx.x * RB + RB - 1), a.T - 1);
  const float scale = a.scale[0];
  const float gs = a.gains[0], gp = a.gains[1], gi = a.gains[2], cg = a.gains[3];
  const int* jm = a.jmin32 + (size_t)b * (a.Np / 32);
  if (lane < RPW) {
    const int t = min(t0 + lane, a.T - 1);
    s_cq[warp * RPW + lane] = load_cq(a.cq + ((size_t)b * a.T + t) * 4);
  }
  __syncwarp();
  Online os[RPW], op[RPW], oi[RPW];
  for (int c0 = 0; c0 < a.Np; c0 += RCC) {
    if (!chunk_live(a, jm, c0, t_last_blk)) continue;
    const int j0 = c0 + lane * 8;
    if (j0 >= a.Np) continue;
    Meta8 m;
    load_meta(a, b, j0, m);
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int t = t0 + r;
      if (t >= a.T) continue;
      const float4 cqr = s_cq[warp * RPW + r];
      float c[8];
      load8_bf16(a.compat + ((size_t)b * a.T + t) * a.Np + j0, c);
      // the 8 entries' scores, then one merge per stream: the exponentials
      // of a group are independent of each other
      float S[8], P[8], I[8];
      float ms = -INFINITY, mp = -INFINITY, mi = -INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        bool allow, ind;
        row_masks(a.mode, m.p[e], t, a.total_steps, allow, ind);
        const float sv = c[e] * scale + m.kb[e];
        S[e] = allow ? sv : -INFINITY;
        P[e] = allow ? sv + cg * cocktail_dot(cqr, m.ck[e]) : -INFINITY;
        I[e] = (allow && ind) ? sv : -INFINITY;
        ms = fmaxf(ms, S[e]);
        mp = fmaxf(mp, P[e]);
        mi = fmaxf(mi, I[e]);
      }
      os[r].merge(ms, S);
      op[r].merge(mp, P);
      oi[r].merge(mi, I);
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float ls = os[r].lse_warp(), lp = op[r].lse_warp(), li = oi[r].lse_warp();
    const int t = t0 + r, lr = warp * RPW + r;
    if (lane == 0) {
      s_l[lr][0] = ls;
      s_l[lr][1] = lp;
      s_l[lr][2] = li;
      if (t < a.T) {
        const size_t row = (size_t)b * a.T + t;
        a.lse[row * 3 + 0] = ls;
        a.lse[row * 3 + 1] = lp;
        a.lse[row * 3 + 2] = li;
      }
    }
  }
  __syncwarp();
  const int t_last_tile = gemm_tile_last(a);
  for (int c0 = 0; c0 < a.Np; c0 += RCC) {
    const int j0 = c0 + lane * 8;
    if (j0 >= a.Np) continue;
    if (!chunk_live(a, jm, c0, t_last_tile)) continue;  // never read
    const bool live = chunk_live(a, jm, c0, t_last_blk);
    Meta8 m;
    if (live) load_meta(a, b, j0, m);
#pragma unroll 2
    for (int r = 0; r < RPW; ++r) {
      const int t = t0 + r;
      if (t >= a.T) continue;
      const size_t off = ((size_t)b * a.T + t) * a.Np + j0;
      float w[8], n[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = n[e] = 0.f;
      if (live) {
        const int lr = warp * RPW + r;
        const float4 cqr = s_cq[lr];
        const float ls = s_l[lr][0], lp = s_l[lr][1], li = s_l[lr][2];
        float c[8];
        load8_bf16(a.compat + off, c);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          bool allow, ind;
          row_masks(a.mode, m.p[e], t, a.total_steps, allow, ind);
          if (!allow) continue;
          const float S = c[e] * scale + m.kb[e];
          const float Pp = S + cg * cocktail_dot(cqr, m.ck[e]);
          w[e] = gs * __expf(S - ls) + gp * __expf(Pp - lp);
          if (ind) n[e] = gi * __expf(S - li);
        }
      }
      store8_bf16(a.Pw + off, w);
      store8_bf16(a.Pi + off, n);
    }
  }
}

constexpr int BWD_RB = RB;  // query rows per CTA

// Backward, first sweep: u_s, u_p, u_i per row (sum_j p_stream(j) G(j)),
// the row statistics every entry's dS needs.
__global__ void __launch_bounds__(256, 2) read_wide_softmax_bwd_u_kernel(const RowArgs a) {
  __shared__ float4 s_cq[RB];
  __shared__ float s_l[RB][3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, t0 = blockIdx.x * RB + warp * RPW;
  const int t_last_blk = min((int)(blockIdx.x * RB + RB - 1), a.T - 1);
  const float scale = a.scale[0];
  const float cg = a.gains[3];
  const int* jm = a.jmin32 + (size_t)b * (a.Np / 32);
  if (lane < RPW) {
    const int lr = warp * RPW + lane;
    const int t = min(t0 + lane, a.T - 1);
    const size_t row = (size_t)b * a.T + t;
    s_cq[lr] = load_cq(a.cq + row * 4);
    s_l[lr][0] = a.lse[row * 3 + 0];
    s_l[lr][1] = a.lse[row * 3 + 1];
    s_l[lr][2] = a.lse[row * 3 + 2];
  }
  __syncwarp();
  float us[RPW], up[RPW], ui[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) us[r] = up[r] = ui[r] = 0.f;
  for (int c0 = 0; c0 < a.Np; c0 += RCC) {
    if (!chunk_live(a, jm, c0, t_last_blk)) continue;
    const int j0 = c0 + lane * 8;
    if (j0 >= a.Np) continue;
    Meta8 m;
    load_meta(a, b, j0, m);
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int t = t0 + r;
      if (t >= a.T) continue;
      const size_t off = ((size_t)b * a.T + t) * a.Np + j0;
      float c[8], g[8], gn[8];
      load8_bf16(a.compat + off, c);
      load8_bf16(a.Pw + off, g);
      load8_bf16(a.Pi + off, gn);
      const int lr = warp * RPW + r;
      const float4 cqr = s_cq[lr];
      const float lsr = s_l[lr][0], lpr = s_l[lr][1], lir = s_l[lr][2];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        bool allow, ind;
        row_masks(a.mode, m.p[e], t, a.total_steps, allow, ind);
        if (!allow) continue;
        const float S = c[e] * scale + m.kb[e];
        const float Pp = S + cg * cocktail_dot(cqr, m.ck[e]);
        us[r] += __expf(S - lsr) * g[e];
        up[r] += __expf(Pp - lpr) * g[e];
        if (ind) ui[r] += __expf(S - lir) * gn[e];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float vs = warp_sum(us[r]), vp = warp_sum(up[r]), vi = warp_sum(ui[r]);
    const int t = t0 + r;
    if (lane == 0 && t < a.T) {
      const size_t row = (size_t)b * a.T + t;
      a.u3[row * 3 + 0] = vs;
      a.u3[row * 3 + 1] = vp;
      a.u3[row * 3 + 2] = vi;
    }
  }
}

// Backward, second sweep, for 64 query rows of one sequence: dS per entry,
// dC, and the weights Pw / Pi, written over G / Gn (= gout W^T, gout Wnext^T,
// BF16) in place for the weight-gradient GEMMs.  Per-column partials (d bias,
// d bank cocktail) are summed over a warp's rows in registers and over the
// CTA's warps through shared memory in a fixed order (no atomics:
// deterministic); per-row partials stay in registers.
__global__ void __launch_bounds__(256, 2) read_wide_softmax_bwd_kernel(const RowArgs a) {
  // per-warp column partials of one chunk: [8][RCC * 5] FP32, dynamic shared
  // memory (the static part holds the per-row and per-chunk constants)
  extern __shared__ float colbuf_raw[];
  float (*colbuf)[RCC * 5] = reinterpret_cast<float (*)[RCC * 5]>(colbuf_raw);
  __shared__ float4 s_cq[RB];           // per-row constants (warp-uniform reads)
  __shared__ float s_l[RB][3], s_u[RB][3];
  __shared__ float s_racc[RB][6];       // per-row partials: d scale, d cocktail_gain, dcq4
  // the chunk's bank data, [entry e][lane] for lane l's columns 8l + e
  // (conflict-free reads), staged once per chunk for the CTA's 64 rows
  __shared__ int m_pos[8][32];
  __shared__ float m_kb[8][32];
  __shared__ float4 m_ck[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, t0 = blockIdx.x * RB + warp * RPW;
  const int t_last_blk = min((int)(blockIdx.x * RB + RB - 1), a.T - 1);
  const float scale = a.scale[0];
  const float gs = a.gains[0], gp = a.gains[1], gi = a.gains[2], cg = a.gains[3];
  const int* jm = a.jmin32 + (size_t)b * (a.Np / 32);
  bf16* Gw = a.Pw;  // G on entry, Pw on exit
  bf16* Gi = a.Pi;  // Gn on entry, Pi on exit
  if (lane < RPW) {
    const int lr = warp * RPW + lane;
    const int t = min(t0 + lane, a.T - 1);
    const size_t row = (size_t)b * a.T + t;
    s_cq[lr] = load_cq(a.cq + row * 4);
    s_l[lr][0] = a.lse[row * 3 + 0];
    s_l[lr][1] = a.lse[row * 3 + 1];
    s_l[lr][2] = a.lse[row * 3 + 2];
    s_u[lr][0] = a.u3[row * 3 + 0];
    s_u[lr][1] = a.u3[row * 3 + 1];
    s_u[lr][2] = a.u3[row * 3 + 2];
#pragma unroll
    for (int k = 0; k < 6; ++k) s_racc[lr][k] = 0.f;
  }
  __syncwarp();
  // dS per entry, dC, weights, row and column partials
  const int t_last_tile = gemm_tile_last(a);
  for (int c0 = 0; c0 < a.Np; c0 += RCC) {
    const int j0 = c0 + lane * 8;
    const bool live = chunk_live(a, jm, c0, t_last_blk);
    const bool read_later = chunk_live(a, jm, c0, t_last_tile);  // planes read by the GEMMs
    if (live) {
      const int cc = threadIdx.x, j = c0 + cc;  // one column per thread
      if (j < a.Np) {
        const size_t o = (size_t)b * a.Np + j;
        m_pos[cc & 7][cc >> 3] = a.pos[o];
        m_kb[cc & 7][cc >> 3] = a.kba[o];
        m_ck[cc & 7][cc >> 3] = a.ckf[o];
      }
    }
    __syncthreads();
    float col[8][5];
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int k = 0; k < 5; ++k) col[e][k] = 0.f;
    // lanes past the last column take part in the warp reductions with zeros
    const bool colok = j0 < a.Np;
    {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int t = t0 + r;
        if (t >= a.T) continue;  // uniform over the warp
        const size_t off = ((size_t)b * a.T + t) * a.Np + j0;
        float dc[8], w[8], n[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) dc[e] = w[e] = n[e] = 0.f;
        float racc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live && colok) {
          float c[8], g[8], gn[8];
          load8_bf16(a.compat + off, c);
          load8_bf16(Gw + off, g);
          load8_bf16(Gi + off, gn);
          const int lr = warp * RPW + r;
          const float4 cqr = s_cq[lr];
          const float lsr = s_l[lr][0], lpr = s_l[lr][1], lir = s_l[lr][2];
          const float usr = s_u[lr][0], upr = s_u[lr][1], uir = s_u[lr][2];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            bool allow, ind;
            row_masks(a.mode, m_pos[e][lane], t, a.total_steps, allow, ind);
            if (!allow) continue;
            const float S = c[e] * scale + m_kb[e][lane];
            const float4 cke = m_ck[e][lane];
            const float cc = cocktail_dot(cqr, cke);
            const float Pp = S + cg * cc;
            const float ps = __expf(S - lsr), pp = __expf(Pp - lpr);
            const float pi = ind ? __expf(S - lir) : 0.f;
            const float dSs = gs * ps * (g[e] - usr);
            const float dSp = gp * pp * (g[e] - upr);
            const float dSi = ind ? gi * pi * (gn[e] - uir) : 0.f;
            const float dS = dSs + dSp + dSi;
            dc[e] = dS * scale;
            w[e] = gs * ps + gp * pp;
            n[e] = gi * pi;
            racc[0] += dS * c[e];
            racc[1] += dSp * cc;
            const float dpc = dSp * cg;
            racc[2] += dpc * cke.x;
            racc[3] += dpc * cke.y;
            racc[4] += dpc * cke.z;
            racc[5] += dpc * cke.w;
            col[e][0] += dS;
            col[e][1] += dpc * cqr.x;
            col[e][2] += dpc * cqr.y;
            col[e][3] += dpc * cqr.z;
            col[e][4] += dpc * cqr.w;
          }
        }
        if (colok && read_later) {
          store8_bf16(a.dC + off, dc);
          store8_bf16(Gw + off, w);
          store8_bf16(Gi + off, n);
        }
        if (live) {  // uniform over the warp: every lane reaches the reductions
          // the row's partials of this chunk, summed over the warp (its
          // lanes cover the chunk's columns); one lane owns the row's sums
#pragma unroll
          for (int k = 0; k < 6; ++k) racc[k] = warp_sum(racc[k]);
          if (lane == 0) {
            const int lr = warp * RPW + r;
#pragma unroll
            for (int k = 0; k < 6; ++k) s_racc[lr][k] += racc[k];
          }
        }
      }
    }
    // column partials of this chunk: the warps' sums in shared memory, then
    // one fixed-order sum per column
    float* mine = colbuf[warp] + lane * 8 * 5;
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int k = 0; k < 5; ++k) mine[e * 5 + k] = col[e][k];
    __syncthreads();
    const int cend = min(c0 + RCC, a.Np);
    float* dst = a.colpart + (((size_t)b * a.nrb + blockIdx.x) * a.Np + c0) * 5;
    for (int i = threadIdx.x; i < (cend - c0) * 5; i += blockDim.x) {
      float v = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) v += colbuf[w8][i];
      dst[i] = v;
    }
    __syncthreads();
  }
  // per-row outputs
  __syncwarp();
  if (lane < RPW) {
    const int t = t0 + lane, lr = warp * RPW + lane;
    if (t < a.T) {
      const size_t row = (size_t)b * a.T + t;
      a.rowpart[row * 2 + 0] = s_racc[lr][0];
      a.rowpart[row * 2 + 1] = s_racc[lr][1];
      a.dcq[row * 4 + 0] = s_racc[lr][2];
      a.dcq[row * 4 + 1] = s_racc[lr][3];
      a.dcq[row * 4 + 2] = s_racc[lr][4];
      a.dcq[row * 4 + 3] = s_racc[lr][5];
    }
  }
}

__global__ void __launch_bounds__(256) read_wide_colsum_kernel(int N, int Np, int nrb,
                                                               const float* colpart, float* dbias,
                                                               float* dck) {
  const int b = blockIdx.y, j = blockIdx.x * 256 + threadIdx.x;
  if (j >= N) return;
  float s[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < nrb; ++r) {
    const float* src = colpart + (((size_t)b * nrb + r) * Np + j) * 5;
#pragma unroll
    for (int k = 0; k < 5; ++k) s[k] += src[k];
  }
  dbias[(size_t)b * N + j] = s[0];
#pragma unroll
  for (int k = 0; k < 4; ++k) dck[((size_t)b * N + j) * 4 + k] = s[1 + k];
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct BankWs {
  int* pos;
  float* kba;
  float4* ckf;
  int* jmin32;
};

size_t bank_ws_bytes(int64_t B, int64_t Np) {
  return align256(B * Np * 4) * 2 + align256(B * Np * 16) + align256(B * (Np / 32) * 4);
}

char* carve_bank(char* p, int64_t B, int64_t Np, BankWs* w) {
  w->pos = (int*)p;
  p += align256(B * Np * 4);
  w->kba = (float*)p;
  p += align256(B * Np * 4);
  w->ckf = (float4*)p;
  p += align256(B * Np * 16);
  w->jmin32 = (int*)p;
  p += align256(B * (Np / 32) * 4);
  return p;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int check_sizes(const char* what, int64_t B, int64_t T, int64_t N, int64_t H) {
  if (B <= 0 || T <= 0 || N <= 0 || H <= 0 || H % 8 != 0) {
    set_error("%s: unsupported sizes B=%lld T=%lld N=%lld H=%lld (H a multiple of 8)", what,
              (long long)B, (long long)T, (long long)N, (long long)H);
    return DABSN_ERR_SHAPE;
  }
  const int64_t Np = (N + 127) / 128 * 128;
  if (2 * (Np / GBK) > MAX_KT || (T + GBK - 1) / GBK > MAX_KT || H / GBK > MAX_KT ||
      B * 3 > 65535 || (T + GBM - 1) / GBM > 65535 || T * Np > ((int64_t)1 << 40)) {
    set_error("%s: sizes beyond the tiling limits (N <= 16384, T <= 32768, H <= 32768)", what);
    return DABSN_ERR_UNSUPPORTED;
  }
  return DABSN_OK;
}

template <int LAYOUT>
int launch_gemm(const GemmArgs& g, int B, cudaStream_t st, const char* what) {
  auto kern = read_gemm_kernel<LAYOUT>;
  if (!kernel_prepared((const void*)kern, (int)GEMM_SMEM)) return DABSN_ERR_LAUNCH;
  dim3 grid((g.N + GBN - 1) / GBN, (g.M + GBM - 1) / GBM, B * g.nprob);
  kern<<<grid, GTHREADS, GEMM_SMEM, st>>>(g);
  return launch_status(what);
}

// The read's GEMMs run on the tcgen05 tensor cores (tc_gemm.cuh);
// DABSN_B200_TCGEN05=0 selects the mma.sync kernels above instead.
bool use_tcgen05() {
  const char* e = getenv("DABSN_B200_TCGEN05");
  return !(e && e[0] == '0');
}

// Output tile width of the read's tcgen05 GEMMs: 256, or 128 with
// DABSN_B200_READ_BN=128.
int read_bn() {
  const char* e = getenv("DABSN_B200_READ_BN");  // read per launch, like the other switches
  return (e && atoi(e) == 128) ? 128 : 256;
}

template <int LAYOUT, int BN>
int launch_tc_bn(tcg::Args t, int B, cudaStream_t st, const char* what) {
  using TL = tcg::Tile<BN>;
  auto kern = tcg::gemm_kernel<LAYOUT, BN>;
  if (!kernel_prepared((const void*)kern, (int)TL::SMEM)) return DABSN_ERR_LAUNCH;
  t.batch = B;
  kern<<<tcg::grid_size(t, TL::BN), tcg::THREADS, TL::SMEM, st>>>(t);
  return launch_status(what);
}

template <int LAYOUT>
int launch_tc(const tcg::Args& t, int B, cudaStream_t st, const char* what) {
  return read_bn() == 256 ? launch_tc_bn<LAYOUT, 256>(t, B, st, what)
                          : launch_tc_bn<LAYOUT, 128>(t, B, st, what);
}

tcg::Args tc_args(int nprob, int M, int N, int K, int skip, const int* jmin32, int Np, int T) {
  tcg::Args t;
  memset(&t, 0, sizeof(t));
  t.nprob = nprob;
  t.M = M;
  t.N = N;
  t.K = K;
  t.skip = skip;
  t.jmin32 = jmin32;
  t.ldj = Np / 32;
  t.T = T;
  t.status = device_status();
  return t;
}

// C[i] = A B[i]^T (scores, value gradients): A [B][T][H], B[i] [B][N][H].
int launch_nt(int B, int T, int N, int Np, int H, const bf16* A, const bf16* const* Bs,
              bf16* const* Cs, int nprob, int mode, const int* jmin32, cudaStream_t st,
              const char* what) {
  if (use_tcgen05()) {
    tcg::Args t = tc_args(nprob, T, N, H, mode == 0 ? tcg::SKIP_OUT_TILE : tcg::SKIP_NONE,
                          jmin32, Np, T);
    for (int i = 0; i < nprob; ++i) {
      if (!tcg::make_map_k(&t.p[i].ta, A, H, T, B, H, (long long)T * H) ||
          !tcg::make_map_k(&t.p[i].tb, Bs[i], H, N, B, H, (long long)N * H, read_bn())) {
        set_error("%s: tensor map encoding failed", what);
        return DABSN_ERR_LAUNCH;
      }
      t.p[i].C = Cs[i];
      t.p[i].sC = (long long)T * Np;
      t.p[i].ldc = Np;
    }
    return launch_tc<tcg::LNT>(t, B, st, what);
  }
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  g.nprob = nprob;
  g.jmin32 = jmin32;
  g.ldj = Np / 32;
  g.T = T;
  g.M = T;
  g.N = N;
  g.K = H;
  g.skip = mode == 0 ? SKIP_OUT_TILE : SKIP_NONE;
  for (int i = 0; i < nprob; ++i)
    g.p[i] = GemmProb{A, Bs[i], nullptr, nullptr, Cs[i], (long long)T * H, (long long)N * H,
                      (long long)T * Np, H, H, Np};
  return launch_gemm<L_NT>(g, B, st, what);
}

// C = A1 B1 (+ A2 B2): A [B][T][Np] (K = N bank entries), B [B][N][H].
int launch_nn(int B, int T, int N, int Np, int H, const bf16* A1, const bf16* B1, const bf16* A2,
              const bf16* B2, bf16* C, int mode, const int* jmin32, cudaStream_t st,
              const char* what) {
  if (use_tcgen05()) {
    tcg::Args t = tc_args(1, T, H, N, mode == 0 ? tcg::SKIP_K_BANK : tcg::SKIP_NONE, jmin32, Np,
                          T);
    t.dual = A2 != nullptr;
    bool ok = tcg::make_map_k(&t.p[0].ta, A1, N, T, B, Np, (long long)T * Np) &&
              tcg::make_map_mn(&t.p[0].tb, B1, H, N, B, H, (long long)N * H);
    if (t.dual)
      ok = ok && tcg::make_map_k(&t.p[0].ta2, A2, N, T, B, Np, (long long)T * Np) &&
           tcg::make_map_mn(&t.p[0].tb2, B2, H, N, B, H, (long long)N * H);
    if (!ok) {
      set_error("%s: tensor map encoding failed", what);
      return DABSN_ERR_LAUNCH;
    }
    t.p[0].C = C;
    t.p[0].sC = (long long)T * H;
    t.p[0].ldc = H;
    return launch_tc<tcg::LNN>(t, B, st, what);
  }
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  g.nprob = 1;
  g.jmin32 = jmin32;
  g.ldj = Np / 32;
  g.T = T;
  g.M = T;
  g.N = H;
  g.K = N;
  g.skip = mode == 0 ? SKIP_K_BANK : SKIP_NONE;
  g.p[0] = GemmProb{A1, B1, A2, B2, C, (long long)T * Np, (long long)N * H, (long long)T * H,
                    Np, H, H};
  return launch_gemm<L_NN>(g, B, st, what);
}

// C[i] = A[i]^T B[i] (bank gradients): A [B][T][Np], B [B][T][H], C [B][N][H].
int launch_tn(int B, int T, int N, int Np, int H, const bf16* const* As, const bf16* const* Bs,
              bf16* const* Cs, int nprob, int mode, const int* jmin32, cudaStream_t st,
              const char* what) {
  if (use_tcgen05()) {
    tcg::Args t = tc_args(nprob, N, H, T, mode == 0 ? tcg::SKIP_K_TIME : tcg::SKIP_NONE, jmin32,
                          Np, T);
    for (int i = 0; i < nprob; ++i) {
      if (!tcg::make_map_mn(&t.p[i].ta, As[i], N, T, B, Np, (long long)T * Np) ||
          !tcg::make_map_mn(&t.p[i].tb, Bs[i], H, T, B, H, (long long)T * H)) {
        set_error("%s: tensor map encoding failed", what);
        return DABSN_ERR_LAUNCH;
      }
      t.p[i].C = Cs[i];
      t.p[i].sC = (long long)N * H;
      t.p[i].ldc = H;
    }
    return launch_tc<tcg::LTN>(t, B, st, what);
  }
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  g.nprob = nprob;
  g.jmin32 = jmin32;
  g.ldj = Np / 32;
  g.T = T;
  g.M = N;
  g.N = H;
  g.K = T;
  g.skip = mode == 0 ? SKIP_K_TIME : SKIP_NONE;
  for (int i = 0; i < nprob; ++i)
    g.p[i] = GemmProb{As[i], Bs[i], nullptr, nullptr, Cs[i], (long long)T * Np, (long long)T * H,
                      (long long)N * H, Np, H, H};
  return launch_gemm<L_TN>(g, B, st, what);
}

int launch_prep(int64_t B, int64_t N, int64_t Np, const int64_t* idx, const uint8_t* valid,
                const float* kb, const float* adm, const bf16* ck, const BankWs& w,
                cudaStream_t st) {
  dim3 grid((unsigned)((Np + 255) / 256), (unsigned)B);
  read_wide_prep_kernel<<<grid, 256, 0, st>>>((int)N, (int)Np, idx, valid, kb, adm, ck, w.pos,
                                              w.kba, w.ckf, w.jmin32);
  return launch_status("read_wide_prep");
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int64_t dabsn_read_wide_ld(int64_t N) { return (N + 127) / 128 * 128; }

extern "C" size_t dabsn_read_wide_fwd_workspace(int64_t B, int64_t T, int64_t N) {
  const int64_t Np = dabsn_read_wide_ld(N);
  return bank_ws_bytes(B, Np) + 2 * align256((size_t)B * T * Np * 2);
}

extern "C" size_t dabsn_read_wide_bwd_workspace(int64_t B, int64_t T, int64_t N) {
  const int64_t Np = dabsn_read_wide_ld(N);
  const int64_t nrb = (T + BWD_RB - 1) / BWD_RB;
  return bank_ws_bytes(B, Np) + 3 * align256((size_t)B * T * Np * 2) +
         align256((size_t)B * nrb * Np * 5 * 4);
}

extern "C" int dabsn_read_wide_fwd(int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                                   int64_t total_steps, const void* q, const void* k,
                                   const void* w, const void* wn, const void* cq, const void* ck,
                                   const float* kb, const float* adm, const float* scale,
                                   const int64_t* idx, const uint8_t* valid, const float* gains,
                                   void* out, void* compat, float* lse, void* ws, size_t ws_bytes,
                                   void* stream) {
  int st0 = check_sizes("read_wide_fwd", B, T, N, H);
  if (st0) return st0;
  if (mode != 0 && mode != 1) {
    set_error("read_wide_fwd: mode must be 0 (seq) or 1 (field)");
    return DABSN_ERR_SHAPE;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(w) || !aligned16(wn) || !aligned16(out) ||
      !aligned16(compat) || !aligned16(ws)) {
    set_error("read_wide_fwd: BF16 operands must be 16-byte aligned");
    return DABSN_ERR_SHAPE;
  }
  if (ws_bytes < dabsn_read_wide_fwd_workspace(B, T, N)) {
    set_error("read_wide_fwd: workspace of %zu bytes < %zu", ws_bytes,
              dabsn_read_wide_fwd_workspace(B, T, N));
    return DABSN_ERR_SHAPE;
  }
  const int64_t Np = dabsn_read_wide_ld(N);
  cudaStream_t st = (cudaStream_t)stream;
  BankWs bw;
  char* p = carve_bank((char*)ws, B, Np, &bw);
  bf16* Pw = (bf16*)p;
  bf16* Pi = (bf16*)(p + align256((size_t)B * T * Np * 2));
  int rc = launch_prep(B, N, Np, idx, valid, kb, adm, (const bf16*)ck, bw, st);
  if (rc) return rc;

  // C = Q K^T
  {
    const bf16* bs[1] = {(const bf16*)k};
    bf16* cs[1] = {(bf16*)compat};
    rc = launch_nt((int)B, (int)T, (int)N, (int)Np, (int)H, (const bf16*)q, bs, cs, 1, mode,
                   bw.jmin32, st, "read_wide_scores");
  }
  if (rc) return rc;

  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.B = (int)B; r.T = (int)T; r.N = (int)N; r.Np = (int)Np; r.mode = mode;
  r.total_steps = (int)total_steps;
  r.compat = (const bf16*)compat;
  r.pos = bw.pos; r.kba = bw.kba; r.ckf = bw.ckf; r.jmin32 = bw.jmin32;
  r.cq = (const bf16*)cq; r.scale = scale; r.gains = gains;
  r.lse = lse; r.Pw = Pw; r.Pi = Pi;
  read_wide_softmax_kernel<<<dim3((unsigned)((T + RB - 1) / RB), (unsigned)B), 256, 0, st>>>(r);
  rc = launch_status("read_wide_softmax");
  if (rc) return rc;

  // out = Pw W + Pi Wnext
  return launch_nn((int)B, (int)T, (int)N, (int)Np, (int)H, Pw, (const bf16*)w, Pi,
                   (const bf16*)wn, (bf16*)out, mode, bw.jmin32, st, "read_wide_values");
}

extern "C" int dabsn_read_wide_bwd(int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                                   int64_t total_steps, const void* q, const void* k,
                                   const void* w, const void* wn, const void* cq, const void* ck,
                                   const float* kb, const float* adm, const float* scale,
                                   const int64_t* idx, const uint8_t* valid, const float* gains,
                                   const void* compat, const float* lse, const void* gout,
                                   float* u3, void* dq, float* dcq, void* dk, void* dw, void* dwn,
                                   float* dbias, float* dck, float* rowpart, void* ws,
                                   size_t ws_bytes, void* stream) {
  int st0 = check_sizes("read_wide_bwd", B, T, N, H);
  if (st0) return st0;
  if (mode != 0 && mode != 1) {
    set_error("read_wide_bwd: mode must be 0 (seq) or 1 (field)");
    return DABSN_ERR_SHAPE;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(w) || !aligned16(wn) || !aligned16(gout) ||
      !aligned16(compat) || !aligned16(dq) || !aligned16(dk) || !aligned16(dw) ||
      !aligned16(dwn) || !aligned16(ws)) {
    set_error("read_wide_bwd: BF16 operands must be 16-byte aligned");
    return DABSN_ERR_SHAPE;
  }
  if (ws_bytes < dabsn_read_wide_bwd_workspace(B, T, N)) {
    set_error("read_wide_bwd: workspace of %zu bytes < %zu", ws_bytes,
              dabsn_read_wide_bwd_workspace(B, T, N));
    return DABSN_ERR_SHAPE;
  }
  const int64_t Np = dabsn_read_wide_ld(N);
  const int64_t nrb = (T + BWD_RB - 1) / BWD_RB;
  const size_t plane = align256((size_t)B * T * Np * 2);
  cudaStream_t st = (cudaStream_t)stream;
  BankWs bw;
  char* p = carve_bank((char*)ws, B, Np, &bw);
  bf16* G = (bf16*)p;
  bf16* Gn = (bf16*)(p + plane);
  bf16* dC = (bf16*)(p + 2 * plane);
  float* colpart = (float*)(p + 3 * plane);
  int rc = launch_prep(B, N, Np, idx, valid, kb, adm, (const bf16*)ck, bw, st);
  if (rc) return rc;

  // G = gout W^T, Gn = gout Wnext^T
  {
    const bf16* bs[2] = {(const bf16*)w, (const bf16*)wn};
    bf16* cs[2] = {G, Gn};
    rc = launch_nt((int)B, (int)T, (int)N, (int)Np, (int)H, (const bf16*)gout, bs, cs, 2, mode,
                   bw.jmin32, st, "read_wide_value_grads");
  }
  if (rc) return rc;

  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.B = (int)B; r.T = (int)T; r.N = (int)N; r.Np = (int)Np; r.mode = mode;
  r.total_steps = (int)total_steps;
  r.compat = (const bf16*)compat;
  r.pos = bw.pos; r.kba = bw.kba; r.ckf = bw.ckf; r.jmin32 = bw.jmin32;
  r.cq = (const bf16*)cq; r.scale = scale; r.gains = gains;
  r.lse = (float*)lse; r.Pw = G; r.Pi = Gn;
  r.dC = dC; r.u3 = u3; r.dcq = dcq; r.rowpart = rowpart; r.colpart = colpart;
  r.nrb = (int)nrb;
  read_wide_softmax_bwd_u_kernel<<<dim3((unsigned)nrb, (unsigned)B), 256, 0, st>>>(r);
  rc = launch_status("read_wide_softmax_bwd_u");
  if (rc) return rc;
  constexpr int kColBuf = 8 * RCC * 5 * sizeof(float);  // + static part: above 48 KB
  if (!kernel_prepared((const void*)read_wide_softmax_bwd_kernel, kColBuf)) return DABSN_ERR_LAUNCH;
  read_wide_softmax_bwd_kernel<<<dim3((unsigned)nrb, (unsigned)B), 256, kColBuf, st>>>(r);
  rc = launch_status("read_wide_softmax_bwd");
  if (rc) return rc;
  read_wide_colsum_kernel<<<dim3((unsigned)((N + 255) / 256), (unsigned)B), 256, 0, st>>>(
      (int)N, (int)Np, (int)nrb, colpart, dbias, dck);
  rc = launch_status("read_wide_colsum");
  if (rc) return rc;

  // dQ = dC K
  rc = launch_nn((int)B, (int)T, (int)N, (int)Np, (int)H, dC, (const bf16*)k, nullptr, nullptr,
                 (bf16*)dq, mode, bw.jmin32, st, "read_wide_query_grad");
  if (rc) return rc;

  // dK = dC^T Q, dW = Pw^T gout, dWnext = Pi^T gout
  const bf16* as[3] = {dC, G, Gn};
  const bf16* bs[3] = {(const bf16*)q, (const bf16*)gout, (const bf16*)gout};
  bf16* cs[3] = {(bf16*)dk, (bf16*)dw, (bf16*)dwn};
  return launch_tn((int)B, (int)T, (int)N, (int)Np, (int)H, as, bs, cs, 3, mode, bw.jmin32, st,
                   "read_wide_bank_grads");
}
