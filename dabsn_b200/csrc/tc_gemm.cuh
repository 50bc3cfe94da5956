// Batched BF16 GEMMs on the 5th-generation tensor cores (tcgen05): FP32
// accumulation in tensor memory, operands staged by TMA, BF16 output.
//
//   LNT: C = A B^T   A [M][K], B [N][K]   (both K-major)
//   LNN: C = A B     A [M][K], B [K][N]   (A K-major, B MN-major)
//   LTN: C = A^T B   A [K][M], B [K][N]   (both MN-major)
// optionally plus up to two more pairs A2 op B2 (+ A3 op B3) over K ranges
// of the same length, accumulated into the same output (the read's
// Pw W + Pi Wnext; the read's output projection over [y, b, retrieved]), for
// up to three problems that share shapes.
//
// Persistent and warp-specialised: one CTA per SM walks the output tiles
// (128 x BN) round-robin.
//   * warp 0 (one thread) issues TMA loads (cp.async.bulk.tensor, 128-byte
//     swizzle) of the live 64-wide K slices of its tiles into a ring of
//     shared-memory stages, across tile boundaries;
//   * warp 1 allocates TMEM and (one thread) issues tcgen05.mma (M=128, N=BN,
//     K=16, four per slice) into one of two accumulator buffers, releasing
//     each stage with tcgen05.commit on its "empty" mbarrier and each finished
//     accumulator on its "full" mbarrier;
//   * warps 2-9 read the accumulator rows of their TMEM lane quarter
//     (tcgen05.ld 32x32b; two warps per quarter, one per half of the
//     columns), run the epilogue and hand the buffer back, so a tile's
//     epilogue overlaps the next tile's main loop.
// Live slices follow the read's causal structure (bank slices after the
// tile's last query, or query slices before the tile's first bank position,
// contribute nothing); every role evaluates the same predicates, and a tile
// with no live slice stores zeros.  Every mbarrier wait is bounded; a timeout
// records status code 6, raises a CTA-wide abort flag and every role leaves
// its loop (TMEM is always released).
//
// Shared-memory operand layouts (what TMA writes with SWIZZLE_128B and what
// the UMMA descriptors describe):
//   K-major : rows of 64 BF16 along K (128 B), 8-row groups 1024 B apart; one
//             box of 64 x rows; a K16 step advances the start by 32 B.
//   MN-major: rows of 64 BF16 along M/N (128 B) for consecutive k, 8-row
//             groups 1024 B apart, 64-wide M/N blocks 8 KB apart (one
//             64 x 64 box each); a K16 step advances the start by 2048 B.
// In both, the 16-byte chunks of a 128-byte row r are XOR-permuted by r mod 8.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <climits>

#include "common.cuh"
#include "geometry.cuh"

namespace dabsn {
namespace tcg {

typedef __nv_bfloat16 bf16;

enum Layout { LNT = 0, LNN = 1, LTN = 2 };
enum Skip { SKIP_NONE = 0, SKIP_OUT_TILE = 1, SKIP_K_BANK = 2, SKIP_K_TIME = 3 };

constexpr int BM = 128, BK = 64;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, each half of the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // producer warp, MMA warp, epilogue warps
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr int STATUS_CODE = 6;
constexpr int GROUP_M = 16;  // row tiles per raster group
constexpr uint32_t WAIT_LIMIT = 1u << 26;

// Output tile 128 x BN_ (64 <= BN_ <= 256, a multiple of 64); stages fill
// ~192 KB of shared memory; TMEM holds two accumulators of BN_ columns.
// Shared memory: 1 KB of alignment slack, the stages, 256 B of mbarriers,
// 2 KB for the mode-1 merge of the column halves, 2 KB of store staging per
// epilogue warp.
template <int BN_>
struct Tile {
  static constexpr int BN = BN_;
  static constexpr uint32_t B_BYTES = BN_ * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN_;
  static constexpr size_t SMEM =
      1024 + (size_t)STAGES * STAGE_BYTES + 256 + 4 * BM * 4 + EPI_WARPS * 2048;
};

// UMMA instruction descriptor: FP32 accumulator, BF16 A and B, M = 128,
// N = bn, A / B MN-major flags.
__host__ __device__ constexpr uint32_t idesc(bool a_mn, bool b_mn, int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct Prob {
  CUtensorMap ta, tb;    // pair 0
  CUtensorMap ta2, tb2;  // pair 1 (dual >= 1)
  CUtensorMap ta3, tb3;  // pair 2 (dual == 2)
  bf16* C;
  long long sC;
  int ldc;
  const float* bias;     // mode 3: [N] added to each row (rounded to BF16), or null
};

// Epilogue of the output tile.  Mode 0 stores C; mode 3 stores C + bias (the
// problem's FP32 bias rounded to BF16 first, as autocast casts a Linear's
// bias before the GEMM; no bias: mode 0); mode 4 stores, in FP32,
// bf16(C + bias) + (*add_scale) * addend (a BF16 Linear's output added to an
// FP32 term, as type promotion evaluates it); mode 5 stores C in FP32 (C32,
// row stride ld32) and mode 6 adds it to C32 (an FP32 accumulation over
// several launches: a product split along K into row chunks).  Modes 1 and 2 treat the
// rows of C as logits (plus an optional bias, rounded to BF16 when the
// caller's logits would be BF16) against one target class per row:
//   1: writes, per row and per BN-column tile, the tile's maximum and
//      sum of exp(logit - maximum), and the target's logit (nothing stored);
//   2: stores BF16 scale * (exp(logit - lse[row]) - onehot(target)), zero for
//      rows whose target is ignore_index.
// Two epilogue warps share a row range, one per half of the columns; in mode
// 1 the second half's (maximum, sum) per row reaches the first through shared
// memory and a bounded mbarrier, so no atomics are needed.
struct Epi {
  int mode;
  const float* bias;       // [N] or null
  const int64_t* targets;  // [M]
  int ignore_index;
  int round_bf16;
  float* part_m;           // mode 1: [M][ldp]
  float* part_s;
  int ldp;
  float* tgt_logit;        // mode 1: [M]
  const float* lse;        // mode 2: [M]
  const float* scale;      // mode 2: one device value
  float* C32;              // modes 4-6: FP32 output [M][ld32]
  const float* addend;     // mode 4: FP32 [M][ld32] added times *add_scale
  const float* add_scale;  // mode 4: one device value
  long long ld32;
};

struct Args {
  Epi epi;
  Prob p[3];
  int nprob;
  int batch;          // batch items per problem (tiles of each)
  int dual;           // extra operand pairs accumulated into the output (0-2)
  int M, N, K;
  int skip;
  const int* jmin32;  // [batch][ldj]
  int ldj;
  int T;
  int* status;
};

// Shared-memory matrix descriptor, SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo_bytes) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;  // leading byte offset
  d |= (uint64_t)(1024u >> 4) << 32;                  // stride byte offset: 8-row groups
  d |= (uint64_t)1 << 46;                             // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;                             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t id,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(id), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                             int* status) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    if (mbar_try_wait_cta(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *abort) return false;
  }
  *abort = 1;
  if (status) atomicExch(status, STATUS_CODE);
  return false;
}

#define DABSN_TMEM_LD32(addr, r)                                                                 \
  asm volatile(                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),            \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),            \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])             \
      : "r"(addr))

// Loads of one K slice of one operand (`rows` M/N rows) into its stage slot:
// one box of 64 x rows (K-major) or rows/64 boxes of 64 x 64 (MN-major).
template <bool MN, int ROWS>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap* map, int k0,
                                             int mn0, int b, uint32_t bar) {
  if (MN) {
#pragma unroll
    for (int j = 0; j < ROWS / 64; ++j) tma_load_3d(dst + j * 8192, map, mn0 + 64 * j, k0, b, bar);
  } else {
    tma_load_3d(dst, map, k0, mn0, b, bar);
  }
}

// One output tile: coordinates and causal structure, evaluated identically by
// every role of the CTA.
struct TileInfo {
  int prob, b, m0, n0, nx;
  bool dead;       // never computed nor stored (the read's dead score tiles)
  int t_last;      // last query row of the tile (causal bound)
  int jmin_rows;   // smallest bank position among the tile's rows (SKIP_K_TIME)
};

template <int BN>
__device__ __forceinline__ TileInfo tile_info(const Args& a, int id, int ntm, int ntn) {
  TileInfo ti;
  // Grouped order (geometry.cuh): the CTAs resident at one time share a band
  // of A rows and a few B column tiles, both L2-resident, so DRAM sees A once
  // and B once per group of GROUP_M row tiles instead of once per row tile.
  const geom::TileCoord c = geom::gemm_tile(id, ntm, ntn, a.nprob, GROUP_M);
  ti.nx = c.nx;
  ti.prob = c.prob;
  ti.b = c.b;
  ti.m0 = c.my * BM;
  ti.n0 = ti.nx * BN;
  ti.t_last = min(ti.m0 + BM - 1, a.T - 1);
  ti.dead = false;
  ti.jmin_rows = 0;
  const int* jm = a.jmin32 ? a.jmin32 + (size_t)ti.b * a.ldj : nullptr;
  if (a.skip == SKIP_OUT_TILE) {
    int mn = INT_MAX;
    for (int q = 0; q < BN / 32; ++q) {
      const int c = ti.n0 / 32 + q;
      if (c < a.ldj) mn = min(mn, jm[c]);
    }
    ti.dead = mn > ti.t_last;
  } else if (a.skip == SKIP_K_TIME) {
    ti.jmin_rows = INT_MAX;
    for (int q = 0; q < BM / 32; ++q) {
      const int c = ti.m0 / 32 + q;
      if (c < a.ldj) ti.jmin_rows = min(ti.jmin_rows, jm[c]);
    }
  }
  return ti;
}

__device__ __forceinline__ bool slice_live(const Args& a, const TileInfo& ti, int kt, int nkt1) {
  const int k1 = kt % nkt1;
  if (a.skip == SKIP_K_BANK) {  // a BK = 64 slice: two 32-entry groups
    const int* jm = a.jmin32 + (size_t)ti.b * a.ldj;
    return geom::groups_live(jm, a.ldj, 2 * k1, 2 * k1 + 2, ti.t_last);
  }
  if (a.skip == SKIP_K_TIME) return (long long)k1 * BK + BK - 1 >= (long long)ti.jmin_rows;
  return true;
}

__device__ __forceinline__ const Prob* prob_of(const Args& a, int prob) {
  // tensor maps are read by TMA from the kernel's parameter space
  return prob == 0 ? &a.p[0] : (prob == 1 ? &a.p[1] : &a.p[2]);
}

// Stores one 32 x 32 BF16 chunk (this warp's 32 rows, columns col0 ..
// col0 + 31) held as four 16-byte packs per lane (lane = row): the packs go
// through the warp's 2 KB of shared memory (16-byte units XOR-permuted by
// row so both phases are free of bank conflicts) and leave as 64-byte row
// segments, eight rows per instruction.
__device__ __forceinline__ void store_chunk(const uint4 (&pk)[4], unsigned char* stage,
                                            bf16* C0, int ldc, int row0, int M, int col0, int N) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(stage + geom::stage_unit_offset(lane, q)) = pk[q];
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), q = lane & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + geom::stage_unit_offset(r, q));
    const int row = row0 + r, col = col0 + q * 8;
    if (row >= M) continue;
    bf16* dst = C0 + (size_t)row * ldc + col;
    if (col + 8 <= N) {
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
      const bf16* e = reinterpret_cast<const bf16*>(&v);
      for (int k = 0; k < 8 && col + k < N; ++k) dst[k] = e[k];
    }
  }
}

// Epilogue of one row of one tile over accumulator columns [cb, ce), in
// 32-column chunks.  Mode 1 returns the row's running maximum and sum of
// exponentials over those columns (and writes the target's logit if it lies
// there); the caller merges the halves.  All lanes of the warp take part
// (the stores are cooperative); rows at or beyond M only skip their work.
template <int BN>
__device__ __forceinline__ float2 epilogue_row(const Args& a, const TileInfo& ti, int row0,
                                              uint32_t tacc, bool zero, int cb, int ce,
                                              unsigned char* stage) {
  const int row = row0 + (threadIdx.x & 31);
  const bool live = row < a.M;
  const Prob* P = prob_of(a, ti.prob);
  bf16* C0 = P->C + (size_t)ti.b * P->sC;
  const Epi& E = a.epi;
  const long long tgt = ((E.mode == 1 || E.mode == 2) && live) ? E.targets[row] : -1;
  const float lse = (E.mode == 2 && live) ? E.lse[row] : 0.f;
  const float sc = (E.mode == 2 && !(tgt == E.ignore_index || tgt < 0)) ? *E.scale : 0.f;
  float run_m = -INFINITY, run_s = 0.f, tgt_val = 0.f;
#pragma unroll 1
  for (int c0 = cb; c0 < ce; c0 += 32) {
    uint32_t r[32];
    if (!zero) {
      DABSN_TMEM_LD32(tacc + (uint32_t)c0, r);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) r[e] = 0u;
    }
    const int col0 = ti.n0 + c0;
    if (col0 >= a.N) continue;  // uniform over the warp
    uint4 pk[4];
    if (E.mode == 5 || E.mode == 6) {
      if (live) {
        float* out = E.C32 + (size_t)row * E.ld32 + col0;
        const bool vec = col0 + 32 <= a.N && (E.ld32 & 3) == 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = __uint_as_float(r[q * 4 + e]);
          if (vec) {
            float4* o4 = reinterpret_cast<float4*>(out + q * 4);
            if (E.mode == 6) {
              const float4 pv = *o4;
              v[0] += pv.x; v[1] += pv.y; v[2] += pv.z; v[3] += pv.w;
            }
            *o4 = make_float4(v[0], v[1], v[2], v[3]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col0 + q * 4 + e < a.N)
                out[q * 4 + e] = v[e] + (E.mode == 6 ? out[q * 4 + e] : 0.f);
          }
        }
      }
      continue;
    }
    if (E.mode == 4) {
      if (live) {
        const float as = *E.add_scale;
        const float* ad = E.addend + (size_t)row * E.ld32 + col0;
        float* out = E.C32 + (size_t)row * E.ld32 + col0;
        const bool vec = col0 + 32 <= a.N && (E.ld32 & 3) == 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = col0 + q * 4 + e;
            const float bv = (P->bias && col < a.N)
                                 ? __bfloat162float(__float2bfloat16_rn(P->bias[col])) : 0.f;
            v[e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[q * 4 + e]) + bv));
          }
          if (vec) {
            const float4 av = *reinterpret_cast<const float4*>(ad + q * 4);
            *reinterpret_cast<float4*>(out + q * 4) =
                make_float4(v[0] + as * av.x, v[1] + as * av.y, v[2] + as * av.z, v[3] + as * av.w);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col0 + q * 4 + e < a.N) out[q * 4 + e] = v[e] + as * ad[q * 4 + e];
          }
        }
      }
      continue;
    }
    if (E.mode == 0 || E.mode == 3) {
      if (E.mode == 3 && P->bias) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = col0 + e;
          const float bv = col < a.N ? __bfloat162float(__float2bfloat16_rn(P->bias[col])) : 0.f;
          r[e] = __float_as_uint(__uint_as_float(r[e]) + bv);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          h[e] = __floats2bfloat162_rn(__uint_as_float(r[q * 8 + 2 * e]),
                                       __uint_as_float(r[q * 8 + 2 * e + 1]));
      }
      store_chunk(pk, stage, C0, P->ldc, row0, a.M, col0, a.N);
      continue;
    }
    float x[32];
    float cmax = -INFINITY;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int col = col0 + e;
      float v = __uint_as_float(r[e]);
      if (E.bias && col < a.N) v += E.bias[col];
      if (E.round_bf16) v = __bfloat162float(__float2bfloat16_rn(v));
      x[e] = col < a.N ? v : -INFINITY;
      cmax = fmaxf(cmax, x[e]);
      if (col == tgt) tgt_val = v;
    }
    if (E.mode == 1) {
      if (live && cmax > -INFINITY) {
        const float m_new = fmaxf(run_m, cmax);
        float sacc = run_s * __expf(run_m - m_new);
#pragma unroll
        for (int e = 0; e < 32; ++e) sacc += __expf(x[e] - m_new);
        run_m = m_new;
        run_s = sacc;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = q * 8 + 2 * e;
          const float g0 = sc * (__expf(x[c] - lse) - (col0 + c == tgt ? 1.f : 0.f));
          const float g1 = sc * (__expf(x[c + 1] - lse) - (col0 + c + 1 == tgt ? 1.f : 0.f));
          h[e] = __floats2bfloat162_rn(g0, g1);
        }
      }
      store_chunk(pk, stage, C0, P->ldc, row0, a.M, col0, a.N);
    }
  }
  if (E.mode == 1 && live && tgt >= ti.n0 + cb && tgt < ti.n0 + ce) E.tgt_logit[row] = tgt_val;
  return make_float2(run_m, run_s);
}

template <int LAYOUT, int BN_>
__global__ void __launch_bounds__(THREADS, 1) gemm_kernel(const __grid_constant__ Args a) {
  using TL = Tile<BN_>;
  constexpr int BN = TL::BN, STAGES = TL::STAGES;
  constexpr uint32_t STAGE_BYTES = TL::STAGE_BYTES, TMEM_COLS = TL::TMEM_COLS;
  constexpr bool A_MN = LAYOUT == LTN;
  constexpr bool B_MN = LAYOUT != LNT;
  constexpr uint32_t ID = idesc(A_MN, B_MN, BN);
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_abort;
  __shared__ uint32_t s_tmem;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + (size_t)STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* pair = acc_empty + 2;        // [2][4]: second column half posted

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntm = (a.M + BM - 1) / BM, ntn = (a.N + BN - 1) / BN;
  const int ntiles = ntm * ntn * a.nprob * a.batch;
  const int nkt1 = (a.K + BK - 1) / BK;
  const int nkt = (1 + a.dual) * nkt1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], EPI_WARPS);  // one arrival per epilogue warp
      for (int q = 0; q < 4; ++q) mbar_init(&pair[i * 4 + q], 32);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  volatile int* abort = &s_abort;

  if (warp == 0) {
    if (lane == 0) {
      // TMA producer
      uint32_t it = 0;
      for (int id = blockIdx.x; id < ntiles && !*abort; id += gridDim.x) {
        const TileInfo ti = tile_info<BN>(a, id, ntm, ntn);
        if (ti.dead) continue;
        const Prob* P = prob_of(a, ti.prob);
        for (int kt = 0; kt < nkt; ++kt) {
          if (!slice_live(a, ti, kt, nkt1)) continue;
          const int s = it % STAGES;
          if (it >= (uint32_t)STAGES &&
              !wait_bounded(&empty[s], ((it / STAGES) & 1) ^ 1, abort, a.status))
            break;
          const int pair = kt / nkt1;
          const int k0 = (kt - pair * nkt1) * BK;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          const uint32_t dst = base + (uint32_t)s * STAGE_BYTES;
          const uint32_t bar = smem_u32(&full[s]);
          const CUtensorMap* ma = pair == 0 ? &P->ta : (pair == 1 ? &P->ta2 : &P->ta3);
          const CUtensorMap* mb = pair == 0 ? &P->tb : (pair == 1 ? &P->tb2 : &P->tb3);
          load_operand<A_MN, BM>(dst, ma, k0, ti.m0, ti.b, bar);
          load_operand<B_MN, BN>(dst + A_BYTES, mb, k0, ti.n0, ti.b, bar);
          ++it;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer
      uint32_t it = 0, acc = 0;
      for (int id = blockIdx.x; id < ntiles && !*abort; id += gridDim.x) {
        const TileInfo ti = tile_info<BN>(a, id, ntm, ntn);
        if (ti.dead) continue;
        const int buf = acc & 1;
        if (acc >= 2 && !wait_bounded(&acc_empty[buf], ((acc / 2) & 1) ^ 1, abort, a.status))
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tacc = tmem + (uint32_t)(buf * BN);
        int n = 0;
        bool ok = true;
        for (int kt = 0; kt < nkt && ok; ++kt) {
          if (!slice_live(a, ti, kt, nkt1)) continue;
          const int s = it % STAGES;
          if (!wait_bounded(&full[s], (it / STAGES) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = base + (uint32_t)s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(sa + k * 2048, 8192) : sw128_desc(sa + k * 32, 16);
            const uint64_t bd = B_MN ? sw128_desc(sb + k * 2048, 8192) : sw128_desc(sb + k * 32, 16);
            umma(tacc, ad, bd, ID, (n > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          ++it;
          ++n;
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);  // arrives once this tile's MMAs are done
        ++acc;
      }
    }
  } else {
    // Epilogue warps 2-9: TMEM lane quarter = warp % 4, column half by warp.
    const int quarter = warp & 3, half = (warp - 2) / 4;
    const int row_in = quarter * 32 + lane;
    float* xm = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(full) + 256);  // [2][128]
    float* xs = xm + 2 * BM;
    unsigned char* stage = reinterpret_cast<unsigned char*>(xs + 2 * BM) + (warp - 2) * 2048;
    uint32_t acc = 0;
    for (int id = blockIdx.x; id < ntiles && !*abort; id += gridDim.x) {
      const TileInfo ti = tile_info<BN>(a, id, ntm, ntn);
      if (ti.dead) continue;
      int n = 0;
      for (int kt = 0; kt < nkt; ++kt) n += slice_live(a, ti, kt, nkt1) ? 1 : 0;
      const int buf = acc & 1;
      const bool have = __all_sync(0xffffffffu,
                                   wait_bounded(&acc_full[buf], (acc / 2) & 1, abort, a.status));
      if (!have) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t tacc = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN);
      const int row = ti.m0 + row_in;
      const float2 ms = epilogue_row<BN>(a, ti, ti.m0 + quarter * 32, tacc, n == 0,
                                         half * (BN / 2), (half + 1) * (BN / 2), stage);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      if (a.epi.mode == 1) {
        // merge the column halves of each row: the second half posts its
        // statistics and arrives on the pair's mbarrier; the first waits
        // (bounded) and combines.  The buffer is rewritten only after both
        // halves released the accumulator, so one slot per buffer suffices.
        bool merged = true;
        if (half == 1) {
          xm[buf * BM + row_in] = ms.x;
          xs[buf * BM + row_in] = ms.y;
          mbar_arrive(&pair[buf * 4 + quarter]);
        } else {
          merged = wait_bounded(&pair[buf * 4 + quarter], (acc / 2) & 1, abort, a.status);
        }
        if (half == 0 && merged && row < a.M) {
          const float m2 = xm[buf * BM + row_in], s2 = xs[buf * BM + row_in];
          const float m = fmaxf(ms.x, m2);
          float sum = 0.f;
          if (m > -INFINITY) sum = ms.y * __expf(ms.x - m) + s2 * __expf(m2 - m);
          a.epi.part_m[(size_t)row * a.epi.ldp + ti.nx] = m;
          a.epi.part_s[(size_t)row * a.epi.ldp + ti.nx] = sum;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++acc;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

#undef DABSN_TMEM_LD32

// Grid of the persistent kernel: one CTA per SM, at most one per tile.
inline unsigned grid_size(const Args& a, int bn) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
  const long long ntiles = (long long)((a.M + BM - 1) / BM) * ((a.N + bn - 1) / bn) * a.nprob *
                           a.batch;
  return (unsigned)std::max<long long>(1, std::min<long long>(ntiles, sms));
}

// ---------------------------------------------------------------------------
// Host: tensor maps through the driver entry point (no link to libcuda).
// ---------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [batch][rows][K] BF16 (K-major operand), row stride `ld` elements, batch
// stride `sb` elements: box 64 (K) x box_rows, 128-byte swizzle, zero fill.
inline bool make_map_k(CUtensorMap* m, const void* ptr, long long K, long long rows,
                       long long batch, long long ld, long long sb, int box_rows = BM) {
  auto enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [batch][K][cols] BF16 (MN-major operand), row stride `ld` elements, batch
// stride `sb` elements: box 64 (cols) x 64 (K), 128-byte swizzle, zero fill.
inline bool make_map_mn(CUtensorMap* m, const void* ptr, long long cols, long long K,
                        long long batch, long long ld, long long sb) {
  auto enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)K, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)BK, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tcg
}  // namespace dabsn
