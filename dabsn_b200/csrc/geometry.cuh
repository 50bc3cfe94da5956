// Index arithmetic shared by kernels and host code: pure functions of sizes
// and indices, compiled for both sides so that a host program can check the
// coverage and bounds properties the kernels rely on (tests/geometry_check.cpp).
#pragma once

#if !defined(__CUDACC__) && !defined(__host__)
#define __host__
#define __device__
#endif

#include <cstddef>
#include <cstdint>

namespace dabsn {
namespace geom {

__host__ __device__ inline int imin(int a, int b) { return a < b ? a : b; }

// ---------------------------------------------------------------------------
// Persistent GEMM tile order (tc_gemm.cuh).  Tile ids run over
// [0, ntm * ntn * nprob * batch); within one (problem, batch item) the row
// tiles come in groups of `group_m`, and inside a group the row tile varies
// fastest, so the CTAs resident at one time share a band of A rows and a few
// B column tiles.
// ---------------------------------------------------------------------------
struct TileCoord {
  int prob, b, my, nx;
};

__host__ __device__ inline TileCoord gemm_tile(int id, int ntm, int ntn, int nprob,
                                               int group_m) {
  TileCoord c;
  const int per_z = ntn * ntm;
  const int z = id / per_z, local = id % per_z;
  const int first_m = (local / (group_m * ntn)) * group_m;
  const int gsize = imin(group_m, ntm - first_m);
  const int in_group = local % (group_m * ntn);
  c.my = first_m + in_group % gsize;
  c.nx = in_group / gsize;
  c.prob = z % nprob;
  c.b = z / nprob;
  return c;
}

// Epilogue store staging (tc_gemm.cuh, store_chunk): a warp's 32 rows x 32
// BF16 columns as 16-byte units, row r's unit q at byte r * 64 +
// 16 * (q ^ ((r >> 1) & 3)); written one row per lane, read back as eight
// 64-byte rows per instruction.
__host__ __device__ inline int stage_unit_offset(int r, int q) {
  return r * 64 + ((q ^ ((r >> 1) & 3)) * 16);
}

// ---------------------------------------------------------------------------
// Cluster split of the grid-wide scan's contraction (core_scan_wide.cu).
// A cluster of CL CTAs owns CL * Hs units; its CTA of rank r keeps the
// cluster's NOc rows (forward: Ug rows then A rows of those units; reverse:
// the units' columns of [Ug;A]) for contraction slice r (Kc columns).  Eight
// warps split the rows into NG groups of 32 and the slice's k16 steps into
// KG = 8 / NG groups.  Each CTA receives, per step, CL * KG slots of
// [32 sequences][RW] FP32 sums, RW = the rows it owns.
// ---------------------------------------------------------------------------
constexpr int kWarps = 8;
constexpr int kSeq = 32;  // sequences per launch

struct ClusterLayout {
  int NOc, Kc, RW, NG, KG, nbuf;
  size_t w_bytes, xs_bytes, recv_bytes, total;
};

// kc: staged chunk width (columns); kcp: its padded row length; nbuf_max:
// staging buffers.
__host__ __device__ inline ClusterLayout cluster_layout(int H, int Hs, int CL, bool reverse,
                                                        int kc, int kcp, int nbuf_max) {
  ClusterLayout L;
  const int K = reverse ? 2 * H : H;
  L.NOc = reverse ? CL * Hs : 2 * CL * Hs;
  L.Kc = K / CL;
  L.RW = reverse ? Hs : 2 * Hs;
  L.NG = L.NOc / 32;
  L.KG = L.NG > 0 ? kWarps / L.NG : 0;
  const int nchunk = (L.Kc + kc - 1) / kc;
  L.nbuf = nchunk < nbuf_max ? nchunk : nbuf_max;
  L.w_bytes = ((size_t)L.NOc * (L.Kc + 8) * 2 + 127) / 128 * 128;
  L.xs_bytes = ((size_t)L.nbuf * kSeq * kcp * 2 + 127) / 128 * 128;
  L.recv_bytes = (size_t)CL * L.KG * kSeq * L.RW * 4;
  L.total = L.w_bytes + L.xs_bytes + L.recv_bytes + 256;  // + mbarrier and peer table
  return L;
}

// Transaction bytes one CTA receives per step: CL * KG slots of nm * 16 rows.
__host__ __device__ inline uint32_t cluster_tx(const ClusterLayout& L, int CL, int nm) {
  return (uint32_t)(CL * L.KG * nm * 16 * L.RW * 4);
}

// Owner CTA `d` and receive column `lr` of cluster row `o`.
__host__ __device__ inline void cluster_row_owner(int o, bool reverse, int CL, int Hs, int& d,
                                                  int& lr) {
  if (reverse) {
    d = o / Hs;
    lr = o % Hs;
  } else {
    const int oo = o % (CL * Hs);
    d = oo / Hs;
    lr = (o >= CL * Hs ? Hs : 0) + oo % Hs;
  }
}

// Byte offset in the receiver's slots of sequence b, column lr, slot `slot`.
__host__ __device__ inline uint32_t cluster_recv_offset(int slot, int b, int lr, int RW) {
  return (uint32_t)(((slot * kSeq + b) * RW + lr) * 4);
}

// ---------------------------------------------------------------------------
// Causal structure of the tensor-core read (seq geometry).  jm[g] is the
// smallest bank position among the 32 bank entries of group g (ldj groups).
// A query row t can read an entry only if the entry's position is <= t.
// ---------------------------------------------------------------------------

// Whether any group of [g0, g1) (clipped to ldj) holds an entry that a query
// row at or before t_last can read.
__host__ __device__ inline bool groups_live(const int* jm, int ldj, int g0, int g1, int t_last) {
  bool live = false;
  for (int g = g0; g < imin(g1, ldj); ++g) live = live || jm[g] <= t_last;
  return live;
}

// Last row of the `tile`-row tile holding row r (rows clipped to T).
__host__ __device__ inline int row_tile_last(int r, int T, int tile) {
  return imin(r / tile * tile + tile - 1, T - 1);
}

}  // namespace geom
}  // namespace dabsn
