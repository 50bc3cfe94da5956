// Grid-wide persistent scan of the DABSN core for wide states (BF16, H up to
// 2368): the recurrent matrix [Ug;A] (8 MB at H = 2048) is spread over the
// whole GPU instead of one cluster.
//
// Mathematics: src/dabsn/kernels/batched_runtime.py:38-158 (forward step) and
// :299-466 (reverse step) of the reference, shared with the narrow scan
// through core_math.cuh.
//
// Decomposition.  One cooperative grid of G = H / Hs CTAs (G <= the SM count,
// all co-resident) runs all T steps for up to 32 sequences.  CTA c owns units
// [c*Hs, (c+1)*Hs): their state lives in registers (two elements per thread)
// and their 2*Hs rows of [Ug;A] (forward) or Hs columns (reverse) stay in
// shared memory for the whole scan (~128 KB).  A step:
//   1. stages the previous step's recurrent vector (y, or [dgate;dexpr];
//      BF16 [32 x K], L2-resident, written by every CTA) in K-chunks with
//      cp.async.cg, double buffered;
//   2. forms the CTA's slice of the product on tensor cores
//      (mma.sync m16n8k16, BF16 in, FP32 accumulate), warps splitting K,
//      partial sums combined with shared-memory reductions;
//   3. runs the per-element step and writes this CTA's slice of the next
//      vector to the exchange buffer;
//   4. crosses a grid barrier (one release-add and acquire-polled counter;
//      bounded, a timeout records code 3/4 in the status word).
// The exchange buffer is double buffered, so one barrier per step suffices.
// The caller provides the exchange buffer and the zeroed counter (scratch).
//
// Cluster split (single GPU; the reverse scan by default): CTAs form
// clusters of 2-8 that share their units' rows of the matrix, each CTA
// holding all of them for 1/CL of the contraction, so a step stages 1/CL of
// the vector and the partial sums travel between the cluster's CTAs through
// distributed shared memory (see ClusterLayout below).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/dabsn_b200.h"
#include "common.cuh"
#include "core_math.cuh"
#include "geometry.cuh"

namespace dabsn {
namespace {

constexpr int WThreads = 256;
constexpr int WWarps = WThreads / 32;
constexpr int MB = 32;         // sequences per launch (two m16 tiles)
static_assert(MB == geom::kSeq && WWarps == geom::kWarps, "geometry.cuh constants");
#ifndef DABSN_WIDE_KC
#define DABSN_WIDE_KC 512
#endif
#ifndef DABSN_WIDE_NBUF
#define DABSN_WIDE_NBUF 2
#endif
constexpr int KC = DABSN_WIDE_KC;      // contraction chunk staged per copy
constexpr int KCP = KC + 8;            // padded chunk row (breaks ldmatrix bank conflicts)
constexpr int NBUF = DABSN_WIDE_NBUF;  // staging buffers (chunks in flight + 1)

constexpr int EPT = 2;         // state elements per thread (MB * 16 / WThreads)

typedef __nv_bfloat16 bf16;

struct WideGeom {
  int B, T, H;
  int Hs;     // units per CTA (8 or 16)
  int G;      // CTAs on this GPU
  int P;      // GPUs sharing the state (tensor parallel); 1 otherwise
  int Hl;     // units owned by this GPU (= H when P = 1)
  int ubase;  // global index of this GPU's first unit
};

// Tensor parallel over units: the exchange buffer and barrier counter of every
// GPU of the group (peer pointers, CUDA IPC), this GPU's rank, and the
// barrier count all counters held when this launch began (identical on every
// rank: launches are collective and counters are never reset).
constexpr int TP_MAX = 8;
struct Peers {
  bf16* x[TP_MAX];
  unsigned* cnt[TP_MAX];
  int rank;
  unsigned base;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16_cg(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

// Grid barrier: all CTAs of the cooperative grid have arrived `target` times.
__device__ __forceinline__ void grid_sync(unsigned* counter, unsigned target, int* status,
                                          int code) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    unsigned v = 0;
    uint32_t it = 0;
    do {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
    } while (v < target && ++it < (1u << 26));
    if (v < target && status) atomicExch(status, code);
  }
  __syncthreads();
}

// Layout of the exchanged vector in global memory: chunk-major, one block of
// MB rows x KC columns per KC-wide column chunk (element (b, k) at
// xoff(b, k) within a parity buffer of xstride(H) elements).  A CTA stages a
// chunk as one contiguous run; with rows of the whole width instead, a chunk
// is MB segments 2*K bytes apart and every CTA meets the same few L2 slices
// at once (measured 4.0 -> 3.1 us per step for barrier + staging at B = 32,
// H = 2048).
__host__ __device__ __forceinline__ size_t xoff(int b, int k) {
  return (size_t)(k / KC) * (MB * KC) + (size_t)b * KC + (k % KC);
}
__host__ __device__ __forceinline__ size_t xstride(int H) {
  return (size_t)MB * ((2 * H + KC - 1) / KC) * KC;  // the reverse pass's 2H columns
}

// Stage rows [0, rows) x global columns [k0, min(k0 + KC, kend)) of the
// chunk-major vector into a [MB x KCP] shared tile (rows >= `rows` stay zero).
__device__ __forceinline__ void stage_chunk(bf16* dst, const bf16* xbase, int rows, int k0,
                                            int kend) {
  const int per_row = KC / 8;  // 16-byte pieces per row
  for (int p = threadIdx.x; p < rows * per_row; p += WThreads) {
    const int r = p / per_row, c = (p % per_row) * 8;
    if (k0 + c < kend) cp_async16_cg(dst + r * KCP + c, xbase + xoff(r, k0 + c));
  }
  cp_async_commit();
}

// Waits until the chunk about to be used has landed: the copy groups
// committed after it (at most NBUF - 1, and no more than the `later` chunks
// left in this step) may still be pending.
__device__ __forceinline__ void wait_chunk(int later, int nbuf = NBUF) {
  const int pend = min(nbuf - 1, later);
  if (pend <= 0) cp_async_wait<0>();
  else if (pend == 1) cp_async_wait<1>();
  else if (pend == 2) cp_async_wait<2>();
  else cp_async_wait<3>();
}

// out[b][o] += sum_{k in chunk} X[b][k] * W[o][k] for o < NO (NO = 8 * NT),
// on tensor cores.  Warp w takes k16 steps w, w+8, ... of the chunk and
// accumulates all (2 m-tiles x NT n-tiles) fragments in `acc`.
template <int NT>
__device__ __forceinline__ void chunk_mma(float (&acc)[2][NT][4], const bf16* X, const bf16* Wrow0,
                                          int ldw, int kw0, int K, int nm = 2) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nks = min(KC, K - kw0) / 16;  // K is a multiple of 16
  for (int ks = warp; ks < nks; ks += WWarps) {
    const int k = ks * 16;
    uint32_t a[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (m >= nm) break;
      const bf16* pa = X + (m * 16 + (lane & 15)) * KCP + k + (lane >> 4) * 8;
      ldsm_x4(smem_u32(pa), a[m][0], a[m][1], a[m][2], a[m][3]);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      uint32_t b0, b1;
      const bf16* pb = Wrow0 + (size_t)(n * 8 + (lane & 7)) * ldw + kw0 + k + ((lane >> 3) & 1) * 8;
      ldsm_x2(smem_u32(pb), b0, b1);
#pragma unroll
      for (int m = 0; m < 2; ++m)
        if (m < nm) mma_bf16(acc[m][n], a[m][0], a[m][1], a[m][2], a[m][3], b0, b1);
    }
  }
}

// Cross-GPU barrier: every CTA arrives on every GPU's counter (system-scope
// release after a system fence, so its peer stores are visible first) and
// waits on its own GPU's counter.  Counts are compared modulo 2^32; the wait
// is bounded and records `code` on timeout.
__device__ __forceinline__ void tp_arrive(const Peers& p, int P) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < P; ++r)
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p.cnt[r]) : "memory");
  }
}

__device__ __forceinline__ void tp_wait(unsigned* cnt, unsigned target, int* status, int code) {
  // after one wait of this launch gave up (a lost peer), later ones return at
  // once: one timeout per launch, not one per step
  if (threadIdx.x == 0 && !(status && *reinterpret_cast<const volatile int*>(status) != 0)) {
    unsigned v = 0;
    uint32_t it = 0;
    do {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
    } while ((int)(v - target) < 0 && ++it < (1u << 26));
    if ((int)(v - target) < 0 && status) atomicExch(status, code);
  }
  __syncthreads();
}

// One exchange-buffer element: this GPU's buffer, or every GPU's (TP).
template <bool TP>
__device__ __forceinline__ void publish(const Peers& p, int P, bf16* local, size_t off, float v) {
  const bf16 h = __float2bfloat16_rn(v);
  if (TP) {
    for (int r = 0; r < P; ++r) p.x[r][off] = h;
  } else {
    local[off] = h;
  }
}

// Bytes of the staging region: the NBUF chunk tiles, which after the product
// also hold the warps' partial sums [WWarps][MB][part_ld(no)] (FP32).
__host__ __device__ constexpr int part_ld(int no);
__host__ __device__ inline size_t stage_bytes(int no) {
  const size_t tiles = (size_t)NBUF * MB * KCP * 2;
  const size_t parts = (size_t)WWarps * MB * part_ld(no) * 4;
  return ((tiles > parts ? tiles : parts) + 15) / 16 * 16;
}

// Row stride (floats) of one warp's [MB][NO] partial-sum slice: float2
// stores of a fragment hit distinct banks.
__host__ __device__ constexpr int part_ld(int no) { return (no + 8) % 16 == 8 ? no + 8 : no + 16; }

// Each warp writes its fragment partial sums to its own slice
// part[warp][MB][S]; readers add the WWarps slices (no atomics).
template <int NT>
__device__ __forceinline__ void store_frags(const float (&acc)[2][NT][4], float* part, int S,
                                            int nm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* p = part + (size_t)warp * MB * S;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    if (m >= nm) break;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int r = m * 16 + (lane >> 2), c = n * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2*>(p + r * S + c) = make_float2(acc[m][n][0], acc[m][n][1]);
      *reinterpret_cast<float2*>(p + (r + 8) * S + c) = make_float2(acc[m][n][2], acc[m][n][3]);
    }
  }
}

__device__ __forceinline__ float part_sum(const float* part, int S, int idx) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < WWarps; ++w) s += part[w * MB * S + idx];
  return s;
}

// ---------------------------------------------------------------------------
// Cluster split of the contraction (single GPU, CL > 1 CTAs per cluster).
// Cluster q owns units [q*CL*Hs, (q+1)*CL*Hs); its CTA of rank r keeps the
// cluster's NOc rows of the (forward: [Ug;A], reverse: [Ug;A]^T) matrix for
// contraction slice r (K / CL columns), so each step stages only that slice
// of the recurrent vector.  Warps split the rows into NG groups of 32 (four
// n8 tiles) and the slice's k16 steps into KG = 8 / NG groups; each warp
// sends its fragment sums for the rows a cluster CTA owns straight into that
// CTA's receive slot [r * KG + kg][MB][RW] with st.async, which completes
// transaction bytes on the receiver's mbarrier (bounded wait, one phase per
// step).  The receiver adds its CL * KG slots.
// ---------------------------------------------------------------------------
using geom::ClusterLayout;

__host__ __device__ inline ClusterLayout cluster_layout(int H, int Hs, int CL, bool reverse) {
  return geom::cluster_layout(H, Hs, CL, reverse, KC, KCP, NBUF);
}
using geom::cluster_tx;

__device__ __forceinline__ void st_async_v2(uint32_t remote_addr, float a, float b,
                                            uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          remote_addr),
      "f"(a), "f"(b), "r"(remote_bar)
      : "memory");
}

// out[b][o] += sum_k X[b][k] * W[o][k] for the 32 rows of this warp's n-group
// (Wrow0 = its first row) over the chunk's k16 steps kg, kg + KG, ...
__device__ __forceinline__ void chunk_mma_group(float (&acc)[2][4][4], const bf16* X,
                                                const bf16* Wrow0, int ldw, int kw0, int K,
                                                int nm, int kg, int KG) {
  const int lane = threadIdx.x & 31;
  const int nks = min(KC, K - kw0) / 16;
  for (int ks = kg; ks < nks; ks += KG) {
    const int k = ks * 16;
    uint32_t a[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (m >= nm) break;
      const bf16* pa = X + (m * 16 + (lane & 15)) * KCP + k + (lane >> 4) * 8;
      ldsm_x4(smem_u32(pa), a[m][0], a[m][1], a[m][2], a[m][3]);
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      uint32_t b0, b1;
      const bf16* pb = Wrow0 + (size_t)(n * 8 + (lane & 7)) * ldw + kw0 + k + ((lane >> 3) & 1) * 8;
      ldsm_x2(smem_u32(pb), b0, b1);
#pragma unroll
      for (int m = 0; m < 2; ++m)
        if (m < nm) mma_bf16(acc[m][n], a[m][0], a[m][1], a[m][2], a[m][3], b0, b1);
    }
  }
}

// Sends this warp's fragment sums to the CTAs owning their rows.  Forward
// rows: [0, CL*Hs) are Ug rows and [CL*Hs, 2*CL*Hs) A rows of the cluster's
// units (owner = unit / Hs, receive column = unit % Hs, + Hs for A); reverse
// rows are the cluster's units.
__device__ __forceinline__ void scatter_frags(const float (&acc)[2][4][4], bool reverse, int ng,
                                              int slot, int CL, int Hs, int RW, int nm,
                                              const uint32_t* peer_recv,
                                              const uint32_t* peer_bar) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int o = ng * 32 + n * 8 + (lane & 3) * 2;
    int d, lr;
    geom::cluster_row_owner(o, reverse, CL, Hs, d, lr);
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (m >= nm) break;
      const int b = m * 16 + (lane >> 2);
      const uint32_t off0 = geom::cluster_recv_offset(slot, b, lr, RW);
      const uint32_t off1 = geom::cluster_recv_offset(slot, b + 8, lr, RW);
      st_async_v2(peer_recv[d] + off0, acc[m][n][0], acc[m][n][1], peer_bar[d]);
      st_async_v2(peer_recv[d] + off1, acc[m][n][2], acc[m][n][3], peer_bar[d]);
    }
  }
}

__device__ __forceinline__ float recv_sum(const float* recv, int nslot, int RW, int idx) {
  float s = 0.f;
  for (int q = 0; q < nslot; ++q) s += recv[q * MB * RW + idx];
  return s;
}

// Split grid barrier: arrive publishes this CTA's writes (after a CTA-wide
// barrier), wait blocks until `target` arrivals; work that no other CTA needs
// runs in between.  The wait is bounded; a timeout records `code`.  The CTA
// barrier orders every thread's stores before thread 0's release reduction,
// which is cumulative, so no separate fence is needed.
__device__ __forceinline__ void grid_arrive(unsigned* counter) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
  }
}

// True once a bounded wait of this launch has given up: its later waits
// return at once, so a lost signal ends a long scan in one timeout, not one
// per step.  The word is per launch (cleared before it), so one timeout does
// not disable the waits of later launches.
__device__ __forceinline__ bool wait_failed(const int* status) {
  return status && *reinterpret_cast<const volatile int*>(status) != 0;
}

// At the end of a launch, copy its wait status into the device's sticky
// status word, which the host reads (dabsn_device_status) to raise.
__device__ __forceinline__ void publish_status(const int* status, int* gstatus) {
  if (threadIdx.x == 0 && gstatus && wait_failed(status))
    atomicMax(gstatus, *reinterpret_cast<const volatile int*>(status));
}

__device__ __forceinline__ void grid_wait(unsigned* counter, unsigned target, int* status,
                                          int code) {
  if (threadIdx.x == 0 && !wait_failed(status)) {
    unsigned v = 0;
    uint32_t it = 0;
    do {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
    } while (v < target && ++it < (1u << 26));
    if (v < target && status) atomicExch(status, code);
  }
  __syncthreads();
}

#ifdef DABSN_SCAN_TRACE
// Diagnostic build only: SM clock of thread 0 of CTA 0 at the phase
// boundaries of steps 100-163 of a scan (forward: dir 0, reverse: dir 1).
__device__ unsigned long long g_trace[2][64][8];
__device__ __forceinline__ void trace(int dir, int t, int T, int ph) {
  const int s = dir ? (T - 1 - t) - 100 : t - 100;
  if (blockIdx.x == 0 && threadIdx.x == 0 && s >= 0 && s < 64) g_trace[dir][s][ph] = clock64();
}
#define TRACE(d, t, T, ph) trace(d, t, T, ph)
#else
#define TRACE(d, t, T, ph)
#endif

struct WideFwdArgs {
  const bf16* Wx;   // [B,T,H]
  const bf16* Wgx;  // [B,T,H]
  const bf16* rec;  // [2H,H]
  CoreParams p;
  const float* init_b;
  const float* init_e;
  const float* init_c;
  bf16* U;
  bf16* nov;
  bf16* plast;
  bf16* expr;
  bf16* write;
  bf16* energy;
  bf16* sat;
  bf16* gate;
  bf16* fin_b;
  bf16* fin_e;
  bf16* fin_c;
  bf16* xbuf;         // [2][MB][H] exchange buffer for y
  unsigned* counter;  // grid barrier counter, zero at launch
  int* status;        // this launch's wait status, zero at launch (fail-fast)
  int* gstatus;       // the device's sticky status word (the host's record)
  WideGeom g;
  Peers peers;        // tensor parallel only
};

// TP: the state's units are split over g.P GPUs; this grid owns g.Hl of them
// (its inputs, parameters, tapes and rows of [Ug;A] are local slices) and
// the exchange buffer column of unit u is its global index.
template <int NT, bool TP, int CL = 1>  // NT = 2*Hs/8 output tiles; CL: cluster split (no TP)
__global__ void __launch_bounds__(WThreads, 1) core_scan_wide_fwd_kernel(const WideFwdArgs a) {
  static_assert(CL == 1 || !TP, "the cluster split is single-GPU only");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const WideGeom g = a.g;
  const int H = g.H, Hs = g.Hs, NO = 2 * Hs, Hl = g.Hl;
  const int ul0 = blockIdx.x * Hs;   // first local unit of this CTA
  const int u0 = g.ubase + ul0;      // its global index
  const int nm = g.B > 16 ? 2 : 1;   // m16 tiles holding live sequences
  const ClusterLayout CLY = cluster_layout(H, Hs, CL, false);
  const int rank = CL > 1 ? (int)(blockIdx.x % CL) : 0;
  const int kbase = CL > 1 ? rank * CLY.Kc : 0;
  const int ldw = CL > 1 ? CLY.Kc + 8 : H + 8;
  bf16* Wsm = reinterpret_cast<bf16*>(smem_raw);  // [NO][H+8], or [NOc][Kc+8] (CL > 1)
  bf16* xs = CL > 1 ? reinterpret_cast<bf16*>(smem_raw + CLY.w_bytes)
                    : Wsm + (size_t)NO * ldw;      // [NBUF][MB][KCP]
  float* recv = reinterpret_cast<float*>(smem_raw + CLY.w_bytes + CLY.xs_bytes);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(smem_raw + CLY.w_bytes + CLY.xs_bytes +
                                               CLY.recv_bytes);
  uint32_t* peer_tab = reinterpret_cast<uint32_t*>(rbar + 1);  // [8] receive slots, [8] mbarriers

  if constexpr (CL == 1) {
    for (int i = threadIdx.x; i < NO * H; i += WThreads) {
      const int o = i / H, k = i % H;
      const int src = o < Hs ? ul0 + o : Hl + ul0 + o - Hs;
      Wsm[(size_t)o * ldw + k] = a.rec[(size_t)src * H + k];
    }
    for (int i = threadIdx.x; i < NBUF * MB * KCP; i += WThreads) xs[i] = __float2bfloat16_rn(0.f);
  } else {
    const int uq0 = (blockIdx.x / CL) * CL * Hs;  // the cluster's first unit (Hl == H)
    for (int i = threadIdx.x; i < CLY.NOc * CLY.Kc; i += WThreads) {
      const int o = i / CLY.Kc, k = i % CLY.Kc;
      const int src = o < CL * Hs ? uq0 + o : H + uq0 + o - CL * Hs;
      Wsm[(size_t)o * ldw + k] = a.rec[(size_t)src * H + kbase + k];
    }
    for (int i = threadIdx.x; i < CLY.nbuf * MB * KCP; i += WThreads)
      xs[i] = __float2bfloat16_rn(0.f);
    if (threadIdx.x == 0) {
      mbar_init(rbar, 1);
      mbar_fence_init();
      mbar_arrive_expect_tx(rbar, cluster_tx(CLY, CL, nm));  // step 0
    }
    if (threadIdx.x < CL) {
      peer_tab[threadIdx.x] = map_shared_rank(recv, threadIdx.x);
      peer_tab[8 + threadIdx.x] = map_shared_rank(rbar, threadIdx.x);
    }
    // every CTA's barrier and table exist before anyone stores remotely
    cluster_sync_all();
  }
  const float alpha = sigmoidf_(a.p.logit_alpha[0]);
  const float lam = softplusf_(a.p.log_lambda[0]);
  const float suppress = sigmoidf_(a.p.logit_c_suppress[0]);

  // Elements: e = threadIdx.x + k * WThreads -> (b = e / Hs, i = e % Hs).
  bool live[EPT];
  int eb[EPT], ei[EPT];
  UnitConsts uc[EPT];
  float sb[EPT], se[EPT], sc[EPT], sy[EPT];
  bf16 wgx[EPT], wxn[EPT];  // next inputs, raw until used (the loads do not stall)
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int e = threadIdx.x + k * WThreads;
    eb[k] = e / Hs;
    ei[k] = e % Hs;
    live[k] = eb[k] < g.B;
    sb[k] = se[k] = sc[k] = sy[k] = 0.f;
    wgx[k] = wxn[k] = __float2bfloat16_rn(0.f);
    if (live[k]) {
      const int ul = ul0 + ei[k], u = u0 + ei[k];
      uc[k] = load_unit(a.p, ul);
      const size_t bs = (size_t)eb[k] * Hl + ul;
      sb[k] = a.init_b[bs];
      se[k] = a.init_e[bs];
      sc[k] = a.init_c[bs];
      const size_t x0 = (size_t)eb[k] * g.T * Hl + ul;
      sy[k] = tanh_fast(__bfloat162float(a.Wx[x0]) + sb[k]);
      publish<TP>(a.peers, g.P, a.xbuf, xoff(eb[k], u), sy[k]);
      wgx[k] = a.Wgx[x0];
      wxn[k] = g.T > 1 ? a.Wx[x0 + Hl] : __float2bfloat16_rn(0.f);
    }
  }
  const unsigned round = TP ? (unsigned)(g.P * g.G) : (unsigned)g.G;
  unsigned target = TP ? a.peers.base + round : round;
  if (TP) {
    tp_arrive(a.peers, g.P);
    tp_wait(a.peers.cnt[a.peers.rank], target, a.status, 3);
  } else {
    grid_sync(a.counter, g.G, a.status, 3);
  }

  const int S = part_ld(NO);
  float* part = reinterpret_cast<float*>(xs);  // [WWarps][MB][S], reuses the staging tiles
  const int warp = threadIdx.x >> 5;
  for (int t = 0; t < g.T; ++t) {
    TRACE(0, t, g.T, 0);
    const bf16* x = a.xbuf + (size_t)(t & 1) * xstride(H);
    if constexpr (CL == 1) {
      const int nchunk = (H + KC - 1) / KC;
      float acc[2][NT][4];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.f;
      for (int c = 0; c < NBUF - 1 && c < nchunk; ++c)
        stage_chunk(xs + c * MB * KCP, x, g.B, c * KC, H);
      for (int c = 0; c < nchunk; ++c) {
        if (c + NBUF - 1 < nchunk)
          stage_chunk(xs + ((c + NBUF - 1) % NBUF) * MB * KCP, x, g.B, (c + NBUF - 1) * KC, H);
        wait_chunk(nchunk - 1 - c);
        __syncthreads();
        chunk_mma<NT>(acc, xs + (c % NBUF) * MB * KCP, Wsm, ldw, c * KC, H, nm);
        __syncthreads();
        if (c == 0) TRACE(0, t, g.T, 1);
      }
      TRACE(0, t, g.T, 2);
      store_frags<NT>(acc, part, S, nm);
      __syncthreads();
    } else {
      // this CTA's contraction slice of y_t, then its sums for every
      // cluster CTA's rows, then the sums for its own rows
      const int nchunk = (CLY.Kc + KC - 1) / KC, nbuf = CLY.nbuf;
      const int ng = warp % CLY.NG, kg = warp / CLY.NG;
      float acc[2][4][4];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.f;
      for (int c = 0; c < nbuf - 1 && c < nchunk; ++c)
        stage_chunk(xs + c * MB * KCP, x, g.B, kbase + c * KC, kbase + CLY.Kc);
      for (int c = 0; c < nchunk; ++c) {
        if (c + nbuf - 1 < nchunk)
          stage_chunk(xs + ((c + nbuf - 1) % nbuf) * MB * KCP, x, g.B,
                      kbase + (c + nbuf - 1) * KC, kbase + CLY.Kc);
        wait_chunk(nchunk - 1 - c, nbuf);
        __syncthreads();
        chunk_mma_group(acc, xs + (c % nbuf) * MB * KCP, Wsm + (size_t)ng * 32 * ldw, ldw, c * KC,
                        CLY.Kc, nm, kg, CLY.KG);
        __syncthreads();
        if (c == 0) TRACE(0, t, g.T, 1);
      }
      TRACE(0, t, g.T, 2);
      scatter_frags(acc, false, ng, rank * CLY.KG + kg, CL, Hs, CLY.RW, nm, peer_tab, peer_tab + 8);
      if (!wait_failed(a.status)) mbar_wait_bounded(rbar, (uint32_t)(t & 1), a.status, 3);
      if (threadIdx.x == 0 && t + 1 < g.T) mbar_arrive_expect_tx(rbar, cluster_tx(CLY, CL, nm));
    }
    TRACE(0, t, g.T, 3);
    // 1) what the next recurrent vector needs, then publish it
    FwdPoint fp[EPT];
    float av[EPT], yn[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k]) continue;
      const int b = eb[k], i = ei[k];
      float gsum, asum;
      if constexpr (CL == 1) {
        gsum = part_sum(part, S, b * S + i);
        asum = part_sum(part, S, b * S + Hs + i);
      } else {
        gsum = recv_sum(recv, CL * CLY.KG, CLY.RW, b * CLY.RW + i);
        asum = recv_sum(recv, CL * CLY.KG, CLY.RW, b * CLY.RW + Hs + i);
      }
      const float gr = __bfloat162float(__float2bfloat16_rn(gsum));
      av[k] = __bfloat162float(__float2bfloat16_rn(asum));
      fwd_gate(sb[k], se[k], __bfloat162float(wgx[k]), gr, av[k], uc[k], alpha, lam, fp[k]);
      if (t + 1 < g.T) {
        yn[k] = tanh_fast(__bfloat162float(wxn[k]) + fp[k].bn);
        publish<TP>(a.peers, g.P, a.xbuf, (size_t)((t + 1) & 1) * xstride(H) + xoff(b, u0 + i),
                    yn[k]);
      }
    }
    if (t + 1 < g.T) {
      if (TP) tp_arrive(a.peers, g.P);
      else grid_arrive(a.counter);
    }
    TRACE(0, t, g.T, 4);
    // 2) the rest of the step and the tapes, while the other CTAs catch up
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k]) continue;
      const int b = eb[k], ul = ul0 + ei[k];
      fwd_rest(sy[k], sb[k], se[k], sc[k], av[k], uc[k], suppress, fp[k]);
      const size_t bt = (size_t)b * g.T + t;
      const size_t row = bt * Hl + ul;
      a.U[bt * 2 * Hl + ul] = __float2bfloat16_rn(sy[k]);
      a.U[bt * 2 * Hl + Hl + ul] = __float2bfloat16_rn(fp[k].bn);
      a.nov[row] = __float2bfloat16_rn(fp[k].n);
      a.plast[row] = __float2bfloat16_rn(fp[k].pl);
      a.expr[row] = __float2bfloat16_rn(av[k]);
      a.write[row] = __float2bfloat16_rn(fp[k].w);
      a.energy[row] = __float2bfloat16_rn(se[k]);
      a.sat[row] = __float2bfloat16_rn(fp[k].c);
      a.gate[row] = __float2bfloat16_rn(fp[k].s);
      if (t + 1 < g.T) sy[k] = yn[k];
      sb[k] = fp[k].bn;
      se[k] = fp[k].enew;
      sc[k] = fp[k].c;
    }
    TRACE(0, t, g.T, 7);
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k] || t + 1 >= g.T) continue;
      const size_t row = ((size_t)eb[k] * g.T + t) * Hl + ul0 + ei[k];
      wgx[k] = a.Wgx[row + Hl];
      wxn[k] = t + 2 < g.T ? a.Wx[row + 2 * Hl] : __float2bfloat16_rn(0.f);
    }
    TRACE(0, t, g.T, 5);
    if (t + 1 < g.T) {
      target += round;
      if (TP) tp_wait(a.peers.cnt[a.peers.rank], target, a.status, 3);
      else grid_wait(a.counter, target, a.status, 3);
    }
    TRACE(0, t, g.T, 6);
  }
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    if (!live[k]) continue;
    const size_t bs = (size_t)eb[k] * Hl + ul0 + ei[k];
    a.fin_b[bs] = __float2bfloat16_rn(sb[k]);
    a.fin_e[bs] = __float2bfloat16_rn(se[k]);
    a.fin_c[bs] = __float2bfloat16_rn(sc[k]);
  }
  if (TP) {
    // closing round: no GPU starts its next launch (which rewrites the
    // exchange buffers) before every GPU has finished reading this one's
    tp_arrive(a.peers, g.P);
    tp_wait(a.peers.cnt[a.peers.rank], target + round, a.status, 3);
  }
  publish_status(a.status, a.gstatus);
  // no CTA leaves while a cluster peer might still address its shared memory
  if constexpr (CL > 1) cluster_sync_all();
}

struct WideBwdArgs {
  const bf16* U;
  const bf16* energy;
  const bf16* sat;
  const bf16* gate;
  const bf16* plast;
  const bf16* expr;
  const bf16* rec;
  CoreParams p;
  const float* init_b;
  const float* init_c;
  // gradients of the tapes: FP32, or BF16 when grad_bf16 (the tapes' own
  // dtype under autocast, read as they arrive instead of widened first)
  const void* gU;
  const void* gnov;
  const void* gp;
  const void* gay;
  const void* gwrite;
  const void* ge;
  const void* gc;
  int grad_bf16;
  // bit i (0 gnov, 1 gp, 2 gay, 3 gwrite, 4 ge, 5 gc): that gradient is one
  // value per (sequence, step), [B, T], the same for every unit (a per-token
  // mean's gradient spread over the units), read without the [B, T, H] copy
  unsigned row_bcast;
  const float* gfin_b;
  const float* gfin_e;
  const float* gfin_c;
  bf16* gWx;
  bf16* gWgx;
  bf16* day;
  float* g_init_b;
  float* g_init_e;
  float* g_init_c;
  float* partial;     // [B,19,H]
  bf16* xbuf;         // [2][MB][2H] exchange buffer for [dgate; dexpr]
  unsigned* counter;  // zero at launch
  int* status;        // this launch's wait status, zero at launch (fail-fast)
  int* gstatus;       // the device's sticky status word (the host's record)
  WideGeom g;
  Peers peers;        // tensor parallel only
};

// One tape gradient (0 when the tape has none).
__device__ __forceinline__ float load_grad(const void* g, size_t i, bool bf16_grads) {
  if (g == nullptr) return 0.f;
  return bf16_grads ? __bfloat162float(static_cast<const bf16*>(g)[i])
                    : static_cast<const float*>(g)[i];
}

// Saved tapes of step t for local unit u (tape row stride: this GPU's units),
// as loaded: BF16 values stay raw until the step that uses them (a step
// later), so the loads do not stall the thread that issues them.
template <bool GB>
struct StepRaw {
  typedef typename std::conditional<GB, bf16, float>::type G;
  bf16 y, b_prev, e_prev, c_prev, gate, p, ay, c_t;  // b_prev, c_prev: unset at t = 0
  G gy0, gb, gc, gnov, gp, gay, gw, ge;
};

template <typename G>
__device__ __forceinline__ G raw_grad(const void* g, size_t i) {
  if (g == nullptr) return G(0.f);
  return static_cast<const G*>(g)[i];
}

template <typename G>
__device__ __forceinline__ float gval(G v) {
  if constexpr (std::is_same<G, float>::value) return v;
  else return __bfloat162float(v);
}

template <bool GB>
__device__ __forceinline__ StepRaw<GB> wide_load_step(const WideBwdArgs& a, int b, int u, int t) {
  typedef typename StepRaw<GB>::G G;
  const int H = a.g.Hl;
  const size_t bt = (size_t)b * a.g.T + t;
  const size_t row = bt * H + u;
  StepRaw<GB> s;
  s.y = a.U[bt * 2 * H + u];
  s.b_prev = t > 0 ? a.U[(bt - 1) * 2 * H + H + u] : __float2bfloat16_rn(0.f);
  s.e_prev = a.energy[row];
  s.c_prev = t > 0 ? a.sat[row - H] : __float2bfloat16_rn(0.f);
  s.gate = a.gate[row];
  s.p = a.plast[row];
  s.ay = a.expr[row];
  s.c_t = a.sat[row];
  s.gy0 = raw_grad<G>(a.gU, bt * 2 * H + u);
  s.gb = raw_grad<G>(a.gU, bt * 2 * H + H + u);
  const unsigned rb = a.row_bcast;
  s.gc = raw_grad<G>(a.gc, (rb & 32u) ? bt : row);
  s.gnov = raw_grad<G>(a.gnov, (rb & 1u) ? bt : row);
  s.gp = raw_grad<G>(a.gp, (rb & 2u) ? bt : row);
  s.gay = raw_grad<G>(a.gay, (rb & 4u) ? bt : row);
  s.gw = raw_grad<G>(a.gwrite, (rb & 8u) ? bt : row);
  s.ge = raw_grad<G>(a.ge, (rb & 16u) ? bt : row);
  return s;
}

// The step's values as floats; at t = 0 the previous b and c are the initial
// state (read here: once per scan).
template <bool GB>
__device__ __forceinline__ StepIn unpack_step(const StepRaw<GB>& r, const WideBwdArgs& a, int b,
                                              int u, int t) {
  StepIn s;
  s.y = __bfloat162float(r.y);
  s.b_prev = t > 0 ? __bfloat162float(r.b_prev) : a.init_b[(size_t)b * a.g.Hl + u];
  s.e_prev = __bfloat162float(r.e_prev);
  s.c_prev = t > 0 ? __bfloat162float(r.c_prev) : a.init_c[(size_t)b * a.g.Hl + u];
  s.gate = __bfloat162float(r.gate);
  s.p = __bfloat162float(r.p);
  s.ay = __bfloat162float(r.ay);
  s.c_t = __bfloat162float(r.c_t);
  s.gy0 = gval(r.gy0);
  s.gb = gval(r.gb);
  s.gc = gval(r.gc);
  s.gnov = gval(r.gnov);
  s.gp = gval(r.gp);
  s.gay = gval(r.gay);
  s.gw = gval(r.gw);
  s.ge = gval(r.ge);
  return s;
}

// TP: this grid owns g.Hl units (local tapes, parameters and gradients) and
// reads the full [Ug;A] (gathered once per call); [dgate; dexpr] columns are
// global unit indices, published to every GPU.
template <int NT, bool TP, int CL = 1, bool GB = false>  // NT = Hs/8 output tiles; GB: BF16 tape grads
__global__ void __launch_bounds__(WThreads, 1) core_scan_wide_bwd_kernel(const WideBwdArgs a) {
  static_assert(CL == 1 || !TP, "the cluster split is single-GPU only");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const WideGeom g = a.g;
  const int H = g.H, Hs = g.Hs, K = 2 * H, Hl = g.Hl;
  const int ul0 = blockIdx.x * Hs;   // first local unit of this CTA
  const int u0 = g.ubase + ul0;      // its global index
  const int nm = g.B > 16 ? 2 : 1;
  const ClusterLayout CLY = cluster_layout(H, Hs, CL, true);
  const int rank = CL > 1 ? (int)(blockIdx.x % CL) : 0;
  const int kbase = CL > 1 ? rank * CLY.Kc : 0;
  const int ldw = CL > 1 ? CLY.Kc + 8 : K + 8;
  bf16* Wsm = reinterpret_cast<bf16*>(smem_raw);  // [Hs][2H+8] or [NOc][Kc+8]: columns of [Ug;A]
  bf16* xs = CL > 1 ? reinterpret_cast<bf16*>(smem_raw + CLY.w_bytes)
                    : Wsm + (size_t)Hs * ldw;      // [NBUF][MB][KCP]
  float* recv = reinterpret_cast<float*>(smem_raw + CLY.w_bytes + CLY.xs_bytes);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(smem_raw + CLY.w_bytes + CLY.xs_bytes +
                                               CLY.recv_bytes);
  uint32_t* peer_tab = reinterpret_cast<uint32_t*>(rbar + 1);

  if constexpr (CL == 1) {
    for (int i = threadIdx.x; i < Hs * K; i += WThreads) {
      const int o = i / K, k = i % K;
      Wsm[(size_t)o * ldw + k] = a.rec[(size_t)k * H + u0 + o];
    }
    for (int i = threadIdx.x; i < NBUF * MB * KCP; i += WThreads) xs[i] = __float2bfloat16_rn(0.f);
  } else {
    const int uq0 = (blockIdx.x / CL) * CL * Hs;
    for (int i = threadIdx.x; i < CLY.NOc * CLY.Kc; i += WThreads) {
      const int o = i / CLY.Kc, k = i % CLY.Kc;
      Wsm[(size_t)o * ldw + k] = a.rec[(size_t)(kbase + k) * H + uq0 + o];
    }
    for (int i = threadIdx.x; i < CLY.nbuf * MB * KCP; i += WThreads)
      xs[i] = __float2bfloat16_rn(0.f);
    if (threadIdx.x == 0) {
      mbar_init(rbar, 1);
      mbar_fence_init();
      mbar_arrive_expect_tx(rbar, cluster_tx(CLY, CL, nm));  // step T-1
    }
    if (threadIdx.x < CL) {
      peer_tab[threadIdx.x] = map_shared_rank(recv, threadIdx.x);
      peer_tab[8 + threadIdx.x] = map_shared_rank(rbar, threadIdx.x);
    }
    cluster_sync_all();
  }
  const float alpha = sigmoidf_(a.p.logit_alpha[0]);
  const float lam = softplusf_(a.p.log_lambda[0]);
  const float sig_lam = sigmoidf_(a.p.log_lambda[0]);
  const float suppress = sigmoidf_(a.p.logit_c_suppress[0]);

  bool live[EPT];
  int eb[EPT], ei[EPT];
  UnitConsts uc[EPT];
  float gbn[EPT], gen[EPT], gcn[EPT], gyr[EPT], gbr[EPT], ky[EPT];
  float pacc[EPT][19];
  StepRaw<GB> nxt[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int e = threadIdx.x + k * WThreads;
    eb[k] = e / Hs;
    ei[k] = e % Hs;
    live[k] = eb[k] < g.B;
    gbn[k] = gen[k] = gcn[k] = gyr[k] = gbr[k] = ky[k] = 0.f;
#pragma unroll
    for (int j = 0; j < 19; ++j) pacc[k][j] = 0.f;
    if (live[k]) {
      const int ul = ul0 + ei[k];
      uc[k] = load_unit(a.p, ul);
      const size_t bs = (size_t)eb[k] * Hl + ul;
      if (a.gfin_b) gbn[k] = a.gfin_b[bs];
      if (a.gfin_e) gen[k] = a.gfin_e[bs];
      if (a.gfin_c) gcn[k] = a.gfin_c[bs];
      nxt[k] = wide_load_step<GB>(a, eb[k], ul, g.T - 1);
    }
  }
  __syncthreads();

  const int nchunk = (K + KC - 1) / KC;
  const int S = part_ld(Hs);
  float* part = reinterpret_cast<float*>(xs);  // [WWarps][MB][S], reuses the staging tiles
  StepPre pre[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    if (!live[k]) continue;
    pre[k] = pre_step(unpack_step(nxt[k], a, eb[k], ul0 + ei[k], g.T - 1), uc[k], suppress);
    if (g.T >= 2) nxt[k] = wide_load_step<GB>(a, eb[k], ul0 + ei[k], g.T - 2);
  }
  const unsigned round = TP ? (unsigned)(g.P * g.G) : (unsigned)g.G;
  unsigned target = TP ? a.peers.base : 0u;
  for (int t = g.T - 1; t >= 0; --t) {
    TRACE(1, t, g.T, 0);
    const bf16* xw = a.xbuf + (size_t)(t & 1) * xstride(H);
    // 1) the carried adjoints -> [dgate; dexpr], published at once
    float dg[EPT], de[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k]) continue;
      const int b = eb[k], u = u0 + ei[k];
      BwdCarry o;
      bwd_carry(pre[k], uc[k], gbn[k], gen[k], gcn[k], alpha, lam, sig_lam, suppress, o);
      dg[k] = o.dgate_pre;
      de[k] = o.d_expr;
      const size_t xo = (size_t)(t & 1) * xstride(H);
      publish<TP>(a.peers, g.P, a.xbuf, xo + xoff(b, u), o.dgate_pre);
      publish<TP>(a.peers, g.P, a.xbuf, xo + xoff(b, H + u), o.d_expr);
#pragma unroll
      for (int j = 0; j < 16; ++j) pacc[k][j] += o.p[j];
      pacc[k][16] += o.s0;
      pacc[k][17] += o.s1;
      pacc[k][18] += o.s2;
      gyr[k] = o.gy_rest;
      gbr[k] = o.gb_rest;
      ky[k] = pre[k].in.y;
      gen[k] = o.ge_next;
      gcn[k] = o.gc_next;
    }
    if (TP) tp_arrive(a.peers, g.P);
    else grid_arrive(a.counter);
    TRACE(1, t, g.T, 1);
    // 2) tapes of this step and the carry-independent part of the next one
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k]) continue;
      const int b = eb[k], ul = ul0 + ei[k];
      const size_t row = ((size_t)b * g.T + t) * Hl + ul;
      a.gWgx[row] = __float2bfloat16_rn(dg[k]);
      a.day[row] = __float2bfloat16_rn(de[k]);
      if (t > 0) pre[k] = pre_step(unpack_step(nxt[k], a, b, ul, t - 1), uc[k], suppress);
    }
    TRACE(1, t, g.T, 7);
#pragma unroll
    for (int k = 0; k < EPT; ++k)
      if (live[k] && t >= 2) nxt[k] = wide_load_step<GB>(a, eb[k], ul0 + ei[k], t - 2);
    TRACE(1, t, g.T, 2);
    target += round;
    if (TP) tp_wait(a.peers.cnt[a.peers.rank], target, a.status, 4);
    else grid_wait(a.counter, target, a.status, 4);
    TRACE(1, t, g.T, 3);
    if constexpr (CL == 1) {
      float acc[2][NT][4];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.f;
      for (int c = 0; c < NBUF - 1 && c < nchunk; ++c)
        stage_chunk(xs + c * MB * KCP, xw, g.B, c * KC, K);
      for (int c = 0; c < nchunk; ++c) {
        if (c + NBUF - 1 < nchunk)
          stage_chunk(xs + ((c + NBUF - 1) % NBUF) * MB * KCP, xw, g.B, (c + NBUF - 1) * KC, K);
        wait_chunk(nchunk - 1 - c);
        __syncthreads();
        chunk_mma<NT>(acc, xs + (c % NBUF) * MB * KCP, Wsm, ldw, c * KC, K, nm);
        __syncthreads();
        if (c == 0) TRACE(1, t, g.T, 4);
      }
      TRACE(1, t, g.T, 5);
      store_frags<NT>(acc, part, S, nm);
      __syncthreads();
    } else {
      const int ncl = (CLY.Kc + KC - 1) / KC, nbuf = CLY.nbuf;
      const int warp = threadIdx.x >> 5;
      const int ng = warp % CLY.NG, kg = warp / CLY.NG;
      float acc[2][4][4];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.f;
      for (int c = 0; c < nbuf - 1 && c < ncl; ++c)
        stage_chunk(xs + c * MB * KCP, xw, g.B, kbase + c * KC, kbase + CLY.Kc);
      for (int c = 0; c < ncl; ++c) {
        if (c + nbuf - 1 < ncl)
          stage_chunk(xs + ((c + nbuf - 1) % nbuf) * MB * KCP, xw, g.B,
                      kbase + (c + nbuf - 1) * KC, kbase + CLY.Kc);
        wait_chunk(ncl - 1 - c, nbuf);
        __syncthreads();
        chunk_mma_group(acc, xs + (c % nbuf) * MB * KCP, Wsm + (size_t)ng * 32 * ldw, ldw, c * KC,
                        CLY.Kc, nm, kg, CLY.KG);
        __syncthreads();
        if (c == 0) TRACE(1, t, g.T, 4);
      }
      TRACE(1, t, g.T, 5);
      scatter_frags(acc, true, ng, rank * CLY.KG + kg, CL, Hs, CLY.RW, nm, peer_tab, peer_tab + 8);
      if (!wait_failed(a.status)) mbar_wait_bounded(rbar, (uint32_t)((g.T - 1 - t) & 1), a.status, 4);
      if (threadIdx.x == 0 && t > 0) mbar_arrive_expect_tx(rbar, cluster_tx(CLY, CL, nm));
    }
    TRACE(1, t, g.T, 6);
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if (!live[k]) continue;
      const int b = eb[k], i = ei[k], ul = ul0 + i;
      const float rsum = CL == 1 ? part_sum(part, S, b * S + i)
                                 : recv_sum(recv, CL * CLY.KG, CLY.RW, b * CLY.RW + i);
      const float radj = __bfloat162float(__float2bfloat16_rn(rsum));
      const float gpre = (gyr[k] + radj) * (1.0f - ky[k] * ky[k]);
      gbn[k] = gbr[k] + gpre;
      a.gWx[((size_t)b * g.T + t) * Hl + ul] = __float2bfloat16_rn(gpre);
    }
    // the next step's writes into the staging tiles (its stage_chunk) come
    // after its grid barrier, which orders them after these reads.
  }
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    if (!live[k]) continue;
    const int b = eb[k], ul = ul0 + ei[k];
    const size_t bs = (size_t)b * Hl + ul;
    a.g_init_b[bs] = gbn[k];
    a.g_init_e[bs] = gen[k];
    a.g_init_c[bs] = gcn[k];
    float* dst = a.partial + (size_t)b * 19 * Hl + ul;
#pragma unroll
    for (int j = 0; j < 19; ++j) dst[(size_t)j * Hl] = pacc[k][j];
  }
  if (TP) {
    // closing round (see the forward kernel)
    tp_arrive(a.peers, g.P);
    tp_wait(a.peers.cnt[a.peers.rank], target + round, a.status, 4);
  }
  publish_status(a.status, a.gstatus);
  if constexpr (CL > 1) cluster_sync_all();
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool wide_geom(int64_t B, int64_t T, int64_t H, WideGeom* g) {
  if (B < 1 || B > MB || T < 1 || H < 64) return false;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
  for (int Hs : {8, 16}) {
    if (H % Hs || H % 16) continue;
    if (H / Hs > sms) continue;
    *g = WideGeom{(int)B, (int)T, (int)H, Hs, (int)(H / Hs), 1, (int)H, 0};
    return true;
  }
  return false;
}

size_t fwd_smem(const WideGeom& g) {
  return (size_t)2 * g.Hs * (g.H + 8) * 2 + stage_bytes(2 * g.Hs);
}
size_t bwd_smem(const WideGeom& g) {
  return (size_t)g.Hs * (2 * g.H + 8) * 2 + stage_bytes(g.Hs);
}

template <typename Kern, typename Args>
int launch_coop(Kern kernel, const Args& a, size_t smem, cudaStream_t stream, const char* what,
                int cl = 1) {
  if (smem > 227 * 1024) {
    set_error("%s: H=%d needs %zu bytes of shared memory", what, a.g.H, smem);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (!kernel_prepared((const void*)kernel, (int)smem)) return DABSN_ERR_LAUNCH;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, WThreads, smem);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
  if (per_sm * sms < a.g.G) {
    set_error("%s: %d CTAs cannot be co-resident (%d per SM)", what, a.g.G, per_sm);
    return DABSN_ERR_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.g.G, 1, 1);
  cfg.blockDim = dim3(WThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cl;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cl > 1 ? 2 : 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) {
    set_error("%s launch: %s (G=%d Hs=%d cluster=%d smem=%zu)", what, cudaGetErrorString(err),
              a.g.G, a.g.Hs, cl, smem);
    return DABSN_ERR_LAUNCH;
  }
  return DABSN_OK;
}

// Largest cluster split (8, 4 or 2 CTAs) the geometry admits: whole clusters,
// contraction slices of whole k16 steps, the cluster's rows in whole 32-row
// warp groups (at most eight), the layout within 227 KB of shared memory and
// every cluster co-resident.  By default only the reverse scan splits: at
// H = 2048, B = 32 its step went from 12.8 to 11.3 us, while the forward step
// (a quarter of the staging to save, the scatter and cluster wait to add) went
// from 7.2 to 8.4 us.  DABSN_B200_WIDE_CLUSTER forces a size (1: none).
template <typename KernelFor>
int pick_cluster(const WideGeom& g, bool reverse, KernelFor kernel_for) {
  const char* e = getenv("DABSN_B200_WIDE_CLUSTER");
  const int forced = e ? atoi(e) : 0;
  if (forced == 1 || (!forced && !reverse)) return 1;
  const int K = reverse ? 2 * g.H : g.H;
  for (int cl : {8, 4, 2}) {
    if (forced && cl != forced) continue;
    if (g.G % cl || K % (16 * cl)) continue;
    const ClusterLayout L = cluster_layout(g.H, g.Hs, cl, reverse);
    if (L.NOc % 32 || L.NG < 1 || L.NG > WWarps || L.total > 227 * 1024) continue;
    const void* kern = kernel_for(cl);
    if (!kern || !kernel_prepared(kern, (int)L.total)) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g.G, 1, 1);
    cfg.blockDim = dim3(WThreads, 1, 1);
    cfg.dynamicSmemBytes = L.total;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (n * cl >= g.G) return cl;
  }
  return 1;
}

inline CoreParams params_of(const dabsn_core_params* p) {
  CoreParams q;
  static_assert(sizeof(CoreParams) == sizeof(dabsn_core_params), "parameter layout");
  memcpy(&q, p, sizeof(q));
  return q;
}

template <bool GB>
int launch_wide_bwd(const WideBwdArgs& a, const WideGeom& g, cudaStream_t st) {
  const int cl = pick_cluster(g, true, [](int c) -> const void* {
    return c == 8 ? (const void*)core_scan_wide_bwd_kernel<2, false, 8, GB>
         : c == 4 ? (const void*)core_scan_wide_bwd_kernel<2, false, 4, GB>
         : c == 2 ? (const void*)core_scan_wide_bwd_kernel<2, false, 2, GB> : nullptr;
  });
  if (cl > 1) {
    const size_t smem = cluster_layout(g.H, g.Hs, cl, true).total;
    int rc = cl == 8 ? launch_coop(core_scan_wide_bwd_kernel<2, false, 8, GB>, a, smem, st,
                                   "core_scan_wide_bwd", 8)
           : cl == 4 ? launch_coop(core_scan_wide_bwd_kernel<2, false, 4, GB>, a, smem, st,
                                   "core_scan_wide_bwd", 4)
                     : launch_coop(core_scan_wide_bwd_kernel<2, false, 2, GB>, a, smem, st,
                                   "core_scan_wide_bwd", 2);
    if (rc == DABSN_OK) return rc;
    cudaGetLastError();
  }
  if (g.Hs == 8)
    return launch_coop(core_scan_wide_bwd_kernel<1, false, 1, GB>, a, bwd_smem(g), st,
                       "core_scan_wide_bwd");
  return launch_coop(core_scan_wide_bwd_kernel<2, false, 1, GB>, a, bwd_smem(g), st,
                     "core_scan_wide_bwd");
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

// Scratch of the grid-wide kernels: two parity buffers of the chunk-major
// exchanged vector (xstride) plus a 256-byte counter and status slot.
static size_t smem_scan_scratch_bytes(int64_t H) {
  return (size_t)2 * xstride((int)H) * sizeof(bf16) + 256;
}

extern "C" size_t dabsn_core_scan_wide_scratch_bytes(int64_t H) {
  return smem_scan_scratch_bytes(H);
}

extern "C" int dabsn_core_scan_wide_fwd(int64_t B, int64_t T, int64_t H, const void* Wx,
                                        const void* Wgx, const void* rec,
                                        const dabsn_core_params* params, const float* init_b,
                                        const float* init_e, const float* init_c, void* U,
                                        void* nov, void* plast, void* expr, void* write,
                                        void* energy, void* sat, void* gate, void* fin_b,
                                        void* fin_e, void* fin_c, void* scratch,
                                        size_t scratch_bytes, void* stream) {
  WideGeom g;
  if (!wide_geom(B, T, H, &g)) {
    set_error("core_scan_wide_fwd: unsupported sizes B=%lld T=%lld H=%lld (B <= 32, H a "
              "multiple of 8, H/8 or H/16 <= SM count)",
              (long long)B, (long long)T, (long long)H);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (scratch_bytes < smem_scan_scratch_bytes(H)) {
    set_error("core_scan_wide_fwd: scratch of %zu bytes < %zu", scratch_bytes,
              dabsn_core_scan_wide_scratch_bytes(H));
    return DABSN_ERR_SHAPE;
  }
  WideFwdArgs a;
  memset(&a, 0, sizeof(a));
  a.Wx = (const bf16*)Wx;
  a.Wgx = (const bf16*)Wgx;
  a.rec = (const bf16*)rec;
  a.p = params_of(params);
  a.init_b = init_b;
  a.init_e = init_e;
  a.init_c = init_c;
  a.U = (bf16*)U;
  a.nov = (bf16*)nov;
  a.plast = (bf16*)plast;
  a.expr = (bf16*)expr;
  a.write = (bf16*)write;
  a.energy = (bf16*)energy;
  a.sat = (bf16*)sat;
  a.gate = (bf16*)gate;
  a.fin_b = (bf16*)fin_b;
  a.fin_e = (bf16*)fin_e;
  a.fin_c = (bf16*)fin_c;
  a.counter = (unsigned*)scratch;
  a.status = (int*)((char*)scratch + 4);  // cleared with the counter below
  a.xbuf = (bf16*)((char*)scratch + 256);
  a.gstatus = device_status();
  a.g = g;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(scratch, 0, 256, st) != cudaSuccess) {
    set_error("core_scan_wide_fwd: counter reset failed");
    return DABSN_ERR_LAUNCH;
  }
  const int cl = pick_cluster(g, false, [](int c) -> const void* {
    return c == 8 ? (const void*)core_scan_wide_fwd_kernel<4, false, 8>
         : c == 4 ? (const void*)core_scan_wide_fwd_kernel<4, false, 4>
         : c == 2 ? (const void*)core_scan_wide_fwd_kernel<4, false, 2> : nullptr;
  });
  if (cl > 1) {
    const size_t smem = cluster_layout(g.H, g.Hs, cl, false).total;
    int rc = cl == 8 ? launch_coop(core_scan_wide_fwd_kernel<4, false, 8>, a, smem, st,
                                   "core_scan_wide_fwd", 8)
           : cl == 4 ? launch_coop(core_scan_wide_fwd_kernel<4, false, 4>, a, smem, st,
                                   "core_scan_wide_fwd", 4)
                     : launch_coop(core_scan_wide_fwd_kernel<4, false, 2>, a, smem, st,
                                   "core_scan_wide_fwd", 2);
    if (rc == DABSN_OK) return rc;
    cudaGetLastError();  // refused cluster launch: the unsplit kernel below
  }
  if (g.Hs == 8)
    return launch_coop(core_scan_wide_fwd_kernel<2, false>, a, fwd_smem(g), st, "core_scan_wide_fwd");
  return launch_coop(core_scan_wide_fwd_kernel<4, false>, a, fwd_smem(g), st, "core_scan_wide_fwd");
}

extern "C" int dabsn_core_scan_wide_bwd(
    int64_t B, int64_t T, int64_t H, const void* U, const void* energy, const void* sat,
    const void* gate, const void* plast, const void* expr, const void* rec,
    const dabsn_core_params* params, const float* init_b, const float* init_c, int grad_dtype,
    unsigned row_bcast,
    const void* gU, const void* gnov, const void* gp, const void* gay, const void* gwrite,
    const void* ge, const void* gc, const float* gfin_b, const float* gfin_e, const float* gfin_c, void* gWx,
    void* gWgx, void* day, float* g_init_b, float* g_init_e, float* g_init_c, float* partial,
    void* scratch, size_t scratch_bytes, void* stream) {
  WideGeom g;
  if (!wide_geom(B, T, H, &g)) {
    set_error("core_scan_wide_bwd: unsupported sizes B=%lld T=%lld H=%lld", (long long)B,
              (long long)T, (long long)H);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (scratch_bytes < smem_scan_scratch_bytes(H)) {
    set_error("core_scan_wide_bwd: scratch too small");
    return DABSN_ERR_SHAPE;
  }
  WideBwdArgs a;
  memset(&a, 0, sizeof(a));
  a.U = (const bf16*)U;
  a.energy = (const bf16*)energy;
  a.sat = (const bf16*)sat;
  a.gate = (const bf16*)gate;
  a.plast = (const bf16*)plast;
  a.expr = (const bf16*)expr;
  a.rec = (const bf16*)rec;
  a.p = params_of(params);
  a.init_b = init_b;
  a.init_c = init_c;
  a.gU = gU;
  a.gnov = gnov;
  a.gp = gp;
  a.gay = gay;
  a.gwrite = gwrite;
  a.ge = ge;
  a.gc = gc;
  a.grad_bf16 = grad_dtype == DABSN_BF16;
  a.row_bcast = row_bcast;
  if (grad_dtype != DABSN_BF16 && grad_dtype != DABSN_F32) {
    set_error("core_scan_wide_bwd: tape gradients must be FP32 or BF16");
    return DABSN_ERR_DTYPE;
  }
  a.gfin_b = gfin_b;
  a.gfin_e = gfin_e;
  a.gfin_c = gfin_c;
  a.gWx = (bf16*)gWx;
  a.gWgx = (bf16*)gWgx;
  a.day = (bf16*)day;
  a.g_init_b = g_init_b;
  a.g_init_e = g_init_e;
  a.g_init_c = g_init_c;
  a.partial = partial;
  a.counter = (unsigned*)scratch;
  a.status = (int*)((char*)scratch + 4);  // cleared with the counter below
  a.xbuf = (bf16*)((char*)scratch + 256);
  a.gstatus = device_status();
  a.g = g;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(scratch, 0, 256, st) != cudaSuccess) {
    set_error("core_scan_wide_bwd: counter reset failed");
    return DABSN_ERR_LAUNCH;
  }
  if (a.grad_bf16) return launch_wide_bwd<true>(a, g, st);
  return launch_wide_bwd<false>(a, g, st);
}

// ---------------------------------------------------------------------------
// Forward scan without caller-provided scratch.
//
// Some callers cannot allocate device memory at the point where they run the
// scan: code inside a custom allocator or memory-pool callback, plugins whose
// host framework owns every allocation and hands out only the tensors of the
// operation, and runtimes that forbid cudaMalloc after start-up.  For them the
// exchange buffer and the barrier counter live in one static device array that
// the library image brings with it; every GPU that loads the library keeps
// DABSN_WIDE_NOALLOC_SCRATCH_BYTES bytes of it until the process exits.
//
// Host code may not use the array's name as a device pointer (on the host it
// names a stand-in object), so the device address is looked up with
// cudaGetSymbolAddress, with that device current, on the first call made on
// it, and cached per device together with the identity of its context (a
// cudaDeviceReset makes a new context, whose first call looks it up again).
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char
    g_wide_noalloc_scratch[DABSN_WIDE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
const void* g_noalloc_ctx[kNoAllocMaxDevices] = {};

// Device address of g_wide_noalloc_scratch on the current device, or nullptr
// with the error message set.
void* noalloc_scratch_address() {
  int dev = current_device();
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("core_scan_wide_fwd_noalloc: device ordinal %d out of range", dev);
    return nullptr;
  }
  const void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_wide_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      set_error("core_scan_wide_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(err));
      return nullptr;
    }
    g_noalloc_addr[dev] = ptr;
    g_noalloc_ctx[dev] = ctx;
  }
  return g_noalloc_addr[dev];
}

}  // namespace

extern "C" int dabsn_core_scan_wide_fwd_noalloc(int64_t B, int64_t T, int64_t H, const void* Wx,
                                                const void* Wgx, const void* rec,
                                                const dabsn_core_params* params,
                                                const float* init_b, const float* init_e,
                                                const float* init_c, void* U, void* nov,
                                                void* plast, void* expr, void* write,
                                                void* energy, void* sat, void* gate, void* fin_b,
                                                void* fin_e, void* fin_c, void* stream) {
  if (H <= 0 || H > DABSN_WIDE_NOALLOC_MAX_H) {
    set_error("core_scan_wide_fwd_noalloc: H=%lld outside 1..%d (the static scratch holds %d "
              "bytes; use dabsn_core_scan_wide_fwd with caller scratch for wider states)",
              (long long)H, DABSN_WIDE_NOALLOC_MAX_H, DABSN_WIDE_NOALLOC_SCRATCH_BYTES);
    return DABSN_ERR_UNSUPPORTED;
  }
  size_t need = smem_scan_scratch_bytes(H);
  if (need > (size_t)DABSN_WIDE_NOALLOC_SCRATCH_BYTES) {
    set_error("core_scan_wide_fwd_noalloc: H=%lld needs %zu scratch bytes > %d", (long long)H,
              need, DABSN_WIDE_NOALLOC_SCRATCH_BYTES);
    return DABSN_ERR_UNSUPPORTED;
  }
  void* scratch = noalloc_scratch_address();
  if (scratch == nullptr) return DABSN_ERR_LAUNCH;
  // The counter is cleared on `stream` before the launch (no allocation); the
  // exchange buffer is fully written before it is read in every step.
  return dabsn_core_scan_wide_fwd(B, T, H, Wx, Wgx, rec, params, init_b, init_e, init_c, U, nov,
                                  plast, expr, write, energy, sat, gate, fin_b, fin_e, fin_c,
                                  scratch, (size_t)DABSN_WIDE_NOALLOC_SCRATCH_BYTES, stream);
}

// ---------------------------------------------------------------------------
// Tensor parallel over units (TensorParallelDABSNCore, core.py:609-874): the
// grid-wide scan spread over the GPUs of a group.  Each GPU runs H/P units;
// every step its CTAs store their slice of the recurrent vector into every
// GPU's exchange buffer (peer pointers) and meet at a cross-GPU barrier.
// ---------------------------------------------------------------------------
namespace dabsn {
namespace {

bool tp_geom(int64_t B, int64_t T, int64_t H, int64_t Hl, int64_t ubase, int P, WideGeom* g) {
  if (B < 1 || B > MB || T < 1 || H < 64 || H % 16 || P < 1 || P > TP_MAX || Hl < 8 ||
      ubase < 0 || ubase + Hl > H)
    return false;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
  for (int Hs : {8, 16}) {
    if (Hl % Hs) continue;
    if (Hl / Hs > sms) continue;
    *g = WideGeom{(int)B, (int)T, (int)H, Hs, (int)(Hl / Hs), P, (int)Hl, (int)ubase};
    return true;
  }
  return false;
}

constexpr size_t TP_COUNTER_BYTES = 256;

bool tp_peers(void* const* bufs, int P, int rank, uint32_t base, Peers* p) {
  memset(p, 0, sizeof(*p));
  for (int r = 0; r < P; ++r) {
    if (!bufs[r]) return false;
    p->cnt[r] = reinterpret_cast<unsigned*>(bufs[r]);
    p->x[r] = reinterpret_cast<bf16*>(reinterpret_cast<char*>(bufs[r]) + TP_COUNTER_BYTES);
  }
  p->rank = rank;
  p->base = base;
  return true;
}

}  // namespace
}  // namespace dabsn

extern "C" size_t dabsn_tp_buffer_bytes(int64_t H) {
  // barrier counter + two parity buffers of the chunk-major exchanged vector
  // (the reverse pass's 2H columns, rounded up to whole chunks)
  return TP_COUNTER_BYTES + (size_t)2 * xstride((int)H) * sizeof(bf16);
}

extern "C" int dabsn_tp_alloc(size_t bytes, void** ptr) {
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) {
    set_error("tp_alloc: %s", cudaGetErrorString(e));
    return DABSN_ERR_LAUNCH;
  }
  return DABSN_OK;
}

extern "C" int dabsn_tp_free(void* ptr) {
  return cudaFree(ptr) == cudaSuccess ? DABSN_OK : DABSN_ERR_LAUNCH;
}

extern "C" int dabsn_tp_ipc_handle(void* ptr, void* handle) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    set_error("tp_ipc_handle: %s", cudaGetErrorString(e));
    return DABSN_ERR_LAUNCH;
  }
  memcpy(handle, &h, sizeof(h));
  return DABSN_OK;
}

extern "C" int dabsn_tp_ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("tp_ipc_open: %s", cudaGetErrorString(e));
    return DABSN_ERR_LAUNCH;
  }
  return DABSN_OK;
}

extern "C" int dabsn_tp_ipc_close(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DABSN_OK : DABSN_ERR_LAUNCH;
}

extern "C" int dabsn_core_scan_tp_fwd(
    int64_t B, int64_t T, int64_t H, int64_t Hl, int64_t ubase, int P, int rank,
    void* const* peer_bufs, uint32_t base, uint32_t* next_base, const void* Wx, const void* Wgx,
    const void* rec, const dabsn_core_params* params, const float* init_b, const float* init_e,
    const float* init_c, void* U, void* nov, void* plast, void* expr, void* write, void* energy,
    void* sat, void* gate, void* fin_b, void* fin_e, void* fin_c, void* stream) {
  WideGeom g;
  if (!tp_geom(B, T, H, Hl, ubase, P, &g) || rank < 0 || rank >= P) {
    set_error("core_scan_tp_fwd: unsupported sizes B=%lld T=%lld H=%lld Hl=%lld ubase=%lld P=%d",
              (long long)B, (long long)T, (long long)H, (long long)Hl, (long long)ubase, P);
    return DABSN_ERR_UNSUPPORTED;
  }
  WideFwdArgs a;
  memset(&a, 0, sizeof(a));
  if (!tp_peers(peer_bufs, P, rank, base, &a.peers)) {
    set_error("core_scan_tp_fwd: missing peer buffer");
    return DABSN_ERR_SHAPE;
  }
  a.Wx = (const bf16*)Wx;
  a.Wgx = (const bf16*)Wgx;
  a.rec = (const bf16*)rec;
  a.p = params_of(params);
  a.init_b = init_b;
  a.init_e = init_e;
  a.init_c = init_c;
  a.U = (bf16*)U;
  a.nov = (bf16*)nov;
  a.plast = (bf16*)plast;
  a.expr = (bf16*)expr;
  a.write = (bf16*)write;
  a.energy = (bf16*)energy;
  a.sat = (bf16*)sat;
  a.gate = (bf16*)gate;
  a.fin_b = (bf16*)fin_b;
  a.fin_e = (bf16*)fin_e;
  a.fin_c = (bf16*)fin_c;
  a.xbuf = a.peers.x[rank];
  a.counter = a.peers.cnt[rank];
  // this launch's status word sits after the counter in the local buffer;
  // peers only ever add to the counter itself
  a.status = reinterpret_cast<int*>(a.peers.cnt[rank] + 1);
  a.gstatus = device_status();
  a.g = g;
  *next_base = base + (uint32_t)(T + 1) * (uint32_t)(P * g.G);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(a.status, 0, sizeof(int), st) != cudaSuccess) {
    set_error("core_scan_tp: status reset failed");
    return DABSN_ERR_LAUNCH;
  }
  if (g.Hs == 8)
    return launch_coop(core_scan_wide_fwd_kernel<2, true>, a, fwd_smem(g), st, "core_scan_tp_fwd");
  return launch_coop(core_scan_wide_fwd_kernel<4, true>, a, fwd_smem(g), st, "core_scan_tp_fwd");
}

extern "C" int dabsn_core_scan_tp_bwd(
    int64_t B, int64_t T, int64_t H, int64_t Hl, int64_t ubase, int P, int rank,
    void* const* peer_bufs, uint32_t base, uint32_t* next_base, const void* U, const void* energy,
    const void* sat, const void* gate, const void* plast, const void* expr, const void* rec_full,
    const dabsn_core_params* params, const float* init_b, const float* init_c, int grad_dtype,
    const void* gU, const void* gnov, const void* gp, const void* gay, const void* gwrite,
    const void* ge, const void* gc, const float* gfin_b, const float* gfin_e, const float* gfin_c, void* gWx,
    void* gWgx, void* day, float* g_init_b, float* g_init_e, float* g_init_c, float* partial,
    void* stream) {
  WideGeom g;
  if (!tp_geom(B, T, H, Hl, ubase, P, &g) || rank < 0 || rank >= P) {
    set_error("core_scan_tp_bwd: unsupported sizes B=%lld T=%lld H=%lld Hl=%lld P=%d",
              (long long)B, (long long)T, (long long)H, (long long)Hl, P);
    return DABSN_ERR_UNSUPPORTED;
  }
  WideBwdArgs a;
  memset(&a, 0, sizeof(a));
  if (!tp_peers(peer_bufs, P, rank, base, &a.peers)) {
    set_error("core_scan_tp_bwd: missing peer buffer");
    return DABSN_ERR_SHAPE;
  }
  a.U = (const bf16*)U;
  a.energy = (const bf16*)energy;
  a.sat = (const bf16*)sat;
  a.gate = (const bf16*)gate;
  a.plast = (const bf16*)plast;
  a.expr = (const bf16*)expr;
  a.rec = (const bf16*)rec_full;
  a.p = params_of(params);
  a.init_b = init_b;
  a.init_c = init_c;
  a.gU = gU;
  a.gnov = gnov;
  a.gp = gp;
  a.gay = gay;
  a.gwrite = gwrite;
  a.ge = ge;
  a.gc = gc;
  a.grad_bf16 = grad_dtype == DABSN_BF16;
  a.row_bcast = 0;
  if (grad_dtype != DABSN_BF16 && grad_dtype != DABSN_F32) {
    set_error("core_scan_wide_bwd: tape gradients must be FP32 or BF16");
    return DABSN_ERR_DTYPE;
  }
  a.gfin_b = gfin_b;
  a.gfin_e = gfin_e;
  a.gfin_c = gfin_c;
  a.gWx = (bf16*)gWx;
  a.gWgx = (bf16*)gWgx;
  a.day = (bf16*)day;
  a.g_init_b = g_init_b;
  a.g_init_e = g_init_e;
  a.g_init_c = g_init_c;
  a.partial = partial;
  a.xbuf = a.peers.x[rank];
  a.counter = a.peers.cnt[rank];
  // this launch's status word sits after the counter in the local buffer;
  // peers only ever add to the counter itself
  a.status = reinterpret_cast<int*>(a.peers.cnt[rank] + 1);
  a.gstatus = device_status();
  a.g = g;
  *next_base = base + (uint32_t)(T + 1) * (uint32_t)(P * g.G);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(a.status, 0, sizeof(int), st) != cudaSuccess) {
    set_error("core_scan_tp: status reset failed");
    return DABSN_ERR_LAUNCH;
  }
  if (g.Hs == 8)
    return launch_coop(core_scan_wide_bwd_kernel<1, true>, a, bwd_smem(g), st, "core_scan_tp_bwd");
  return launch_coop(core_scan_wide_bwd_kernel<2, true>, a, bwd_smem(g), st, "core_scan_tp_bwd");
}

#ifdef DABSN_SCAN_TRACE
extern "C" int dabsn_scan_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, dabsn::g_trace, sizeof(dabsn::g_trace));
}
#endif
