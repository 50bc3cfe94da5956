// Batched BF16 GEMMs on the 5th-generation tensor cores (tcgen05): FP32
// accumulation in tensor memory, operands staged by TMA, BF16 output.
//
//   LNT: C = A B^T   A [M][K], B [N][K]   (both K-major)
//   LNN: C = A B     A [M][K], B [K][N]   (A K-major, B MN-major)
//   LTN: C = A^T B   A [K][M], B [K][N]   (both MN-major)
// optionally plus a second pair A2 op B2 over its own K range (the read's
// Pw W + Pi Wnext), for up to three problems that share shapes.
//
// One CTA computes a 128 x 128 tile of C with 4 warps:
//   * warp 0 first lists the live 64-wide K slices (causal structure of the
//     read: bank slices after the tile's last query, or query slices before
//     the tile's first bank position, contribute nothing);
//   * thread 0 issues TMA loads (cp.async.bulk.tensor, 128-byte swizzle) of
//     the live slices into a 3-stage shared-memory ring (two CTAs share an
//     SM, so one CTA's epilogue overlaps the other's main loop);
//   * thread 32 issues tcgen05.mma (M=128, N=128, K=16, four per slice) into
//     a 128-column FP32 accumulator in TMEM and releases each stage with
//     tcgen05.commit on its "empty" mbarrier;
//   * all four warps read their 32 accumulator rows (tcgen05.ld 32x32b) and
//     store BF16 rows of C.
// Every mbarrier wait is bounded; a timeout records status code 6 and the
// CTA skips the rest of its work (TMEM is always released).  A tile with no
// live slice stores zeros.
//
// Shared-memory operand layouts (what TMA writes with SWIZZLE_128B and what
// the UMMA descriptors describe):
//   K-major : rows of 64 BF16 along K (128 B), 8-row groups 1024 B apart; one
//             16 KB box of 128 rows; a K16 step advances the start by 32 B.
//   MN-major: rows of 64 BF16 along M/N (128 B) for consecutive k, 8-row
//             groups 1024 B apart, the two 64-wide M/N halves 8 KB apart
//             (two 8 KB boxes); a K16 step advances the start by 2048 B.
// In both, the 16-byte chunks of a 128-byte row r are XOR-permuted by r mod 8.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <climits>

#include "common.cuh"

namespace dabsn {
namespace tcg {

typedef __nv_bfloat16 bf16;

enum Layout { LNT = 0, LNN = 1, LTN = 2 };
enum Skip { SKIP_NONE = 0, SKIP_OUT_TILE = 1, SKIP_K_BANK = 2, SKIP_K_TIME = 3 };

constexpr int BM = 128, BK = 64, THREADS = 128;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr int MAX_KT = 1024;

// Output tile 128 x BN_ (a multiple of 64, <= 256).  With BN_ = 128: 3
// stages, two CTAs per SM, so one CTA's epilogue overlaps the other's main
// loop.  (128 x 256 tiles, with 4 stages on one CTA per SM or 2 stages on two,
// measured slower on the readout GEMMs of config 5.)
template <int BN_>
struct Tile {
  static constexpr int BN = BN_;
  static constexpr int STAGES = BN_ <= 128 ? 3 : 2;
  static constexpr int MIN_BLOCKS = 2;
  static constexpr uint32_t B_BYTES = BN_ * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = BN_;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256 + MAX_KT * 4;
};
constexpr int STATUS_CODE = 6;
constexpr uint32_t WAIT_LIMIT = 1u << 26;

// UMMA instruction descriptor: FP32 accumulator, BF16 A and B, N = M = 128,
// A / B MN-major flags.
__host__ __device__ constexpr uint32_t idesc(bool a_mn, bool b_mn, int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct Prob {
  CUtensorMap ta, tb;    // pair 0
  CUtensorMap ta2, tb2;  // pair 1 (dual)
  bf16* C;
  long long sC;
  int ldc;
};

// Epilogue of the output tile.  Mode 0 stores C.  Modes 1 and 2 treat the
// rows of C as logits (plus an optional bias, rounded to BF16 when the
// caller's logits would be BF16) against one target class per row:
//   1: writes, per row and per 128-column tile, the tile's maximum and
//      sum of exp(logit - maximum), and the target's logit (nothing stored);
//   2: stores BF16 scale * (exp(logit - lse[row]) - onehot(target)), zero for
//      rows whose target is ignore_index.
// Each epilogue thread owns one row, so no cross-thread reduction is needed.
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
};

struct Args {
  Epi epi;
  Prob p[3];
  int nprob;
  int dual;
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

template <int LAYOUT, int BN_>
__global__ void __launch_bounds__(THREADS, Tile<BN_>::MIN_BLOCKS)
    gemm_kernel(const __grid_constant__ Args a) {
  using TL = Tile<BN_>;
  constexpr int BN = TL::BN, STAGES = TL::STAGES;
  constexpr uint32_t STAGE_BYTES = TL::STAGE_BYTES, TMEM_COLS = TL::TMEM_COLS;
  constexpr bool A_MN = LAYOUT == LTN;
  constexpr bool B_MN = LAYOUT != LNT;
  constexpr uint32_t ID = idesc(A_MN, B_MN, BN);
  extern __shared__ unsigned char smem_raw[];
  __shared__ int s_abort;
  __shared__ uint32_t s_tmem;
  __shared__ int s_nlive;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + (size_t)STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  int* klist = reinterpret_cast<int*>(gbase + (size_t)STAGES * STAGE_BYTES + 256);

  const int prob = blockIdx.z % a.nprob, b = blockIdx.z / a.nprob;
  // tensor maps are read by TMA from the kernel's parameter space
  const Prob* P = prob == 0 ? &a.p[0] : (prob == 1 ? &a.p[1] : &a.p[2]);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int* jm = a.jmin32 ? a.jmin32 + (size_t)b * a.ldj : nullptr;
  const int t_last = min(m0 + BM - 1, a.T - 1);

  if (a.skip == SKIP_OUT_TILE) {
    int mn = INT_MAX;
#pragma unroll
    for (int q = 0; q < BN / 32; ++q) {
      const int c = n0 / 32 + q;
      if (c < a.ldj) mn = min(mn, jm[c]);
    }
    if (mn > t_last) return;  // uniform over the CTA; the tile is never read
  }
  int jmin_rows = 0;
  if (a.skip == SKIP_K_TIME) {
    jmin_rows = INT_MAX;
#pragma unroll
    for (int q = 0; q < BM / 32; ++q) {
      const int c = m0 / 32 + q;
      if (c < a.ldj) jmin_rows = min(jmin_rows, jm[c]);
    }
  }
  const int nkt1 = (a.K + BK - 1) / BK;
  const int nkt = a.dual ? 2 * nkt1 : nkt1;
  // Without causal skipping slice i is slice i (no list, any K); with it the
  // live slices are listed (callers keep K / 64 <= MAX_KT).
  if (warp == 0 && a.skip != SKIP_NONE) {
    int cnt = 0;
    for (int base_kt = 0; base_kt < nkt; base_kt += 32) {
      const int kt = base_kt + lane;
      bool live = kt < nkt;
      if (live) {
        const int k1 = kt < nkt1 ? kt : kt - nkt1;
        if (a.skip == SKIP_K_BANK) {
          const int c0 = 2 * k1, c1 = 2 * k1 + 1;
          int mn = c0 < a.ldj ? jm[c0] : INT_MAX;
          if (c1 < a.ldj) mn = min(mn, jm[c1]);
          live = mn <= t_last;
        } else if (a.skip == SKIP_K_TIME) {
          live = (long long)k1 * BK + BK - 1 >= (long long)jmin_rows;
        }
      }
      const unsigned mask = __ballot_sync(0xffffffffu, live);
      if (live) klist[cnt + __popc(mask & ((1u << lane) - 1u))] = kt;
      cnt += __popc(mask);
    }
    if (lane == 0) s_nlive = cnt;
  } else if (threadIdx.x == 0) {
    s_nlive = nkt;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
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
  const int nlive = s_nlive;
  volatile int* abort = &s_abort;

  if (threadIdx.x == 0) {
    // TMA producer
    for (int i = 0; i < nlive; ++i) {
      const int s = i % STAGES;
      if (i >= STAGES && !wait_bounded(&empty[s], ((i / STAGES) & 1) ^ 1, abort, a.status)) break;
      const int kt = a.skip == SKIP_NONE ? i : klist[i];
      const bool second = kt >= nkt1;
      const int k0 = (second ? kt - nkt1 : kt) * BK;
      const CUtensorMap* ma = second ? &P->ta2 : &P->ta;
      const CUtensorMap* mb = second ? &P->tb2 : &P->tb;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      const uint32_t dst = base + (uint32_t)s * STAGE_BYTES;
      const uint32_t bar = smem_u32(&full[s]);
      load_operand<A_MN, BM>(dst, ma, k0, m0, b, bar);
      load_operand<B_MN, BN>(dst + A_BYTES, mb, k0, n0, b, bar);
    }
  } else if (threadIdx.x == 32) {
    // MMA issuer
    bool ok = nlive > 0;
    for (int i = 0; i < nlive; ++i) {
      const int s = i % STAGES;
      if (!wait_bounded(&full[s], (i / STAGES) & 1, abort, a.status)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = base + (uint32_t)s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        const uint64_t ad = A_MN ? sw128_desc(sa + k * 2048, 8192) : sw128_desc(sa + k * 32, 16);
        const uint64_t bd = B_MN ? sw128_desc(sb + k * 2048, 8192) : sw128_desc(sb + k * 32, 16);
        umma(tmem, ad, bd, ID, (i > 0 || k > 0) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    if (ok) umma_commit(done);
  }
  __syncwarp();

  // Epilogue: warp w owns accumulator rows 32w .. 32w+31 (TMEM lanes).
  const bool have =
      nlive > 0 && __all_sync(0xffffffffu, wait_bounded(done, 0, abort, a.status));
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const int row = m0 + warp * 32 + lane;
  bf16* C = P->C + (size_t)b * P->sC + (size_t)row * P->ldc;
  const Epi& E = a.epi;
  const long long tgt = (E.mode != 0 && row < a.M) ? E.targets[row] : -1;
  float run_m = -INFINITY, run_s = 0.f, tgt_val = 0.f;
  if (nlive == 0 || have) {
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      if (have) {
        const uint32_t addr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
        DABSN_TMEM_LD32(addr, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
      if (row >= a.M) continue;
      const int col0 = n0 + c0;
      if (E.mode == 0) {
        if (col0 + 32 <= a.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 pk;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              h[e] = __floats2bfloat162_rn(__uint_as_float(r[q * 8 + 2 * e]),
                                           __uint_as_float(r[q * 8 + 2 * e + 1]));
            *reinterpret_cast<uint4*>(C + col0 + q * 8) = pk;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (col0 + e < a.N) C[col0 + e] = __float2bfloat16_rn(__uint_as_float(r[e]));
        }
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
        if (cmax > -INFINITY) {
          const float m_new = fmaxf(run_m, cmax);
          float s = run_s * __expf(run_m - m_new);
#pragma unroll
          for (int e = 0; e < 32; ++e) s += __expf(x[e] - m_new);
          run_m = m_new;
          run_s = s;
        }
      } else {
        const bool ignored = tgt == E.ignore_index || tgt < 0;
        const float sc = ignored ? 0.f : *E.scale;
        const float l = E.lse[row];
        float gv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = col0 + e;
          gv[e] = col < a.N ? sc * (__expf(x[e] - l) - (col == tgt ? 1.f : 0.f)) : 0.f;
        }
        if (col0 + 32 <= a.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 pk;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(gv[q * 8 + 2 * e], gv[q * 8 + 2 * e + 1]);
            *reinterpret_cast<uint4*>(C + col0 + q * 8) = pk;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (col0 + e < a.N) C[col0 + e] = __float2bfloat16_rn(gv[e]);
        }
      }
    }
    if (E.mode == 1 && row < a.M) {
      E.part_m[(size_t)row * E.ldp + blockIdx.x] = run_m;
      E.part_s[(size_t)row * E.ldp + blockIdx.x] = run_s;
      if (tgt >= n0 && tgt < n0 + BN) E.tgt_logit[row] = tgt_val;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

#undef DABSN_TMEM_LD32

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
