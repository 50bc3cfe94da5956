// Host check of the index arithmetic in dabsn_b200/csrc/geometry.cuh that
// the kernels rely on (built with g++ by tests/test_geometry_cpu.py):
//   * the persistent GEMM's grouped tile order visits every tile of every
//     (problem, batch item) exactly once, and its epilogue's store staging
//     is a bank-conflict-free bijection in both phases;
//   * the grid-wide scan's cluster split: for every geometry the launcher
//     accepts, the warps' scattered fragment sums write every receive slot
//     element of every cluster CTA exactly once, inside the slot area, in
//     8-byte aligned pairs that stay with one owner, the bytes arriving at a
//     CTA equal the transaction count its mbarrier expects, each row reaches
//     the CTA owning its unit, and the layout fits in 227 KB.
// Prints "ok" and exits 0, or lists the failures and exits 1.
#include <algorithm>
#include <climits>
#include <cstdio>
#include <vector>

#include "geometry.cuh"

using namespace dabsn::geom;

static int failures = 0;
#define CHECK(cond, ...)                  \
  do {                                    \
    if (!(cond)) {                        \
      if (failures < 20) {                \
        std::printf("FAIL: " __VA_ARGS__); \
        std::printf("\n");                \
      }                                   \
      ++failures;                         \
    }                                     \
  } while (0)

static void check_gemm_order(int M, int N, int BM, int BN, int nprob, int batch, int group_m) {
  const int ntm = (M + BM - 1) / BM, ntn = (N + BN - 1) / BN;
  const long total = (long)ntm * ntn * nprob * batch;
  std::vector<int> seen(total, 0);
  for (long id = 0; id < total; ++id) {
    const TileCoord c = gemm_tile((int)id, ntm, ntn, nprob, group_m);
    const bool in = c.prob >= 0 && c.prob < nprob && c.b >= 0 && c.b < batch && c.my >= 0 &&
                    c.my < ntm && c.nx >= 0 && c.nx < ntn;
    CHECK(in, "gemm tile %ld of M=%d N=%d out of range", id, M, N);
    if (!in) continue;
    seen[(((long)c.b * nprob + c.prob) * ntm + c.my) * ntn + c.nx] += 1;
    // a group's row tiles stay inside its band
    const long local = id % ((long)ntm * ntn);
    const int first = (int)(local / ((long)group_m * ntn)) * group_m;
    CHECK(c.my >= first && c.my < first + group_m, "gemm tile %ld leaves its group", id);
  }
  for (long i = 0; i < total; ++i)
    CHECK(seen[i] == 1, "gemm tile %ld of M=%d N=%d BN=%d seen %d times", i, M, N, BN, seen[i]);
}

// Mirrors the launcher's acceptance test for a cluster size.
static bool accepted(int H, int Hs, int CL, bool reverse, const ClusterLayout& L) {
  const int G = H / Hs, K = reverse ? 2 * H : H;
  if (G % CL || K % (16 * CL)) return false;
  if (L.NOc % 32 || L.NG < 1 || L.NG > kWarps) return false;
  return L.total <= 227 * 1024;
}

static void check_cluster(int H, int Hs, int CL, bool reverse, int nm) {
  const ClusterLayout L = cluster_layout(H, Hs, CL, reverse, 512, 520, 2);
  if (!accepted(H, Hs, CL, reverse, L)) return;
  CHECK(L.KG * L.NG == kWarps, "H=%d CL=%d: warp split %d x %d", H, CL, L.NG, L.KG);
  CHECK(L.Kc % 16 == 0, "H=%d CL=%d: slice %d not whole k16 steps", H, CL, L.Kc);
  const int nfloat = (int)(L.recv_bytes / 4);
  std::vector<std::vector<int>> hits(CL, std::vector<int>(nfloat, 0));
  std::vector<long> bytes(CL, 0);
  for (int r = 0; r < CL; ++r)
    for (int w = 0; w < kWarps; ++w) {
      const int ng = w % L.NG, kg = w / L.NG, slot = r * L.KG + kg;
      for (int lane = 0; lane < 32; ++lane)
        for (int n = 0; n < 4; ++n) {
          const int o = ng * 32 + n * 8 + (lane & 3) * 2;
          int d, lr, d1, lr1;
          cluster_row_owner(o, reverse, CL, Hs, d, lr);
          cluster_row_owner(o + 1, reverse, CL, Hs, d1, lr1);
          CHECK(d >= 0 && d < CL && lr >= 0 && lr + 1 < L.RW, "H=%d CL=%d row %d -> (%d, %d)", H,
                CL, o, d, lr);
          CHECK(d1 == d && lr1 == lr + 1, "H=%d CL=%d rows %d, %d split between owners", H, CL,
                o, o + 1);
          // the owner holds the unit of row o at the right receive column
          const int unit = o % (CL * Hs);
          const int want_lr = (reverse ? 0 : (o >= CL * Hs ? Hs : 0)) + unit % Hs;
          CHECK(d == unit / Hs && lr == want_lr, "H=%d CL=%d row %d owner (%d, %d)", H, CL, o, d,
                lr);
          if (d < 0 || d >= CL) continue;
          for (int m = 0; m < nm; ++m)
            for (int half = 0; half < 2; ++half) {
              const int b = m * 16 + (lane >> 2) + 8 * half;
              const uint32_t off = cluster_recv_offset(slot, b, lr, L.RW);
              CHECK(off % 8 == 0 && off + 8 <= L.recv_bytes, "H=%d CL=%d offset %u", H, CL, off);
              if (off + 8 > L.recv_bytes) continue;
              hits[d][off / 4] += 1;
              hits[d][off / 4 + 1] += 1;
              bytes[d] += 8;
            }
        }
    }
  const uint32_t tx = cluster_tx(L, CL, nm);
  for (int d = 0; d < CL; ++d) {
    CHECK(bytes[d] == (long)tx, "H=%d Hs=%d CL=%d rev=%d nm=%d: CTA %d gets %ld bytes, expects %u",
          H, Hs, CL, (int)reverse, nm, d, bytes[d], tx);
    for (int slot = 0; slot < CL * L.KG; ++slot)
      for (int b = 0; b < kSeq; ++b)
        for (int lr = 0; lr < L.RW; ++lr) {
          const int want = b < nm * 16 ? 1 : 0;
          const int got = hits[d][cluster_recv_offset(slot, b, lr, L.RW) / 4];
          CHECK(got == want, "H=%d CL=%d CTA %d slot %d b %d col %d written %d times", H, CL, d,
                slot, b, lr, got);
        }
  }
}

// Both phases of the epilogue's store staging: a bijection onto the warp's
// 2 KB, and each quarter-warp (eight lanes, one 128-byte wavefront of 16-byte
// accesses) touches eight distinct 16-byte bank groups.
static void check_store_staging() {
  std::vector<int> seen(128, 0);
  for (int r = 0; r < 32; ++r)
    for (int q = 0; q < 4; ++q) {
      const int off = stage_unit_offset(r, q);
      CHECK(off % 16 == 0 && off >= 0 && off < 2048, "staging offset %d", off);
      if (off >= 0 && off < 2048) seen[off / 16] += 1;
    }
  for (int u = 0; u < 128; ++u) CHECK(seen[u] == 1, "staging unit %d used %d times", u, seen[u]);
  // write phase: lane = row, fixed q per instruction
  for (int q = 0; q < 4; ++q)
    for (int phase = 0; phase < 4; ++phase) {
      int groups = 0;
      for (int l = phase * 8; l < phase * 8 + 8; ++l) groups |= 1 << ((stage_unit_offset(l, q) / 16) % 8);
      CHECK(groups == 0xff, "write q=%d phase %d bank groups %x", q, phase, groups);
    }
  // read phase: lane -> (row it*8 + lane/4, unit lane%4)
  for (int it = 0; it < 4; ++it)
    for (int phase = 0; phase < 4; ++phase) {
      int groups = 0;
      for (int l = phase * 8; l < phase * 8 + 8; ++l)
        groups |= 1 << ((stage_unit_offset(it * 8 + (l >> 2), l & 3) / 16) % 8);
      CHECK(groups == 0xff, "read it=%d phase %d bank groups %x", it, phase, groups);
    }
}

// The read's row kernels store the [B, T, Np] planes (weights, score
// gradients) of a 256-column chunk for a 64-row block only when the chunk is
// live for the 128-row GEMM tile holding the block; the GEMMs that read the
// planes must then never touch an unwritten region.  Checked for random
// group minima (any values: the argument does not need them sorted), for the
// tcgen05 GEMMs (64-wide K slices, 128-entry bank tiles) and the mma.sync
// fallback (32-wide slices).
// `write_tile`: the row tile whose last row decides the stores (128, as the
// kernels do; 64 is the deliberately wrong rule the check must catch).
// Returns the number of unwritten reads found.
static int row_plane_misses(int T, int Np, unsigned seed, int write_tile) {
  int misses = 0;
  const int ldj = Np / 32, RB = 64, RCC = 256, BM = 128;
  std::vector<int> jm(ldj);
  unsigned x = seed;
  for (int g = 0; g < ldj; ++g) {
    x = x * 1664525u + 1013904223u;
    jm[g] = (int)(x % (unsigned)(T + T / 4));  // some groups after every query
  }
  auto written = [&](int t, int col) {  // does the row kernel store (t, col)?
    const int r0 = t / RB * RB;
    const int c0 = col / RCC * RCC;
    return groups_live(jm.data(), ldj, c0 / 32, (c0 + RCC) / 32,
                       row_tile_last(r0, T, write_tile));
  };
  for (int bk : {64, 32}) {
    const int gps = bk / 32;  // groups per K slice
    // value / gradient products: rows = queries (128-row tiles), K = bank
    for (int m0 = 0; m0 < T; m0 += BM) {
      const int t_last = std::min(m0 + BM - 1, T - 1);
      for (int k0 = 0; k0 < Np; k0 += bk) {
        if (!groups_live(jm.data(), ldj, k0 / 32, k0 / 32 + gps, t_last)) continue;
        for (int t = m0; t <= t_last; t += 16)
          for (int col = k0; col < std::min(k0 + bk, Np); col += 8)
            misses += written(t, col) ? 0 : 1;
      }
    }
    // transposed products: rows = bank entries (128-entry tiles), K = queries
    for (int e0 = 0; e0 < Np; e0 += BM) {
      int jmin_rows = INT_MAX;
      for (int g = e0 / 32; g < std::min((e0 + BM) / 32, ldj); ++g)
        jmin_rows = std::min(jmin_rows, jm[g]);
      for (int k0 = 0; k0 < T; k0 += bk) {
        if ((long long)k0 + bk - 1 < (long long)jmin_rows) continue;  // slice dead
        for (int t = k0; t < std::min(k0 + bk, T); t += 8)
          for (int col = e0; col < std::min(e0 + BM, Np); col += 32)
            misses += written(t, col) ? 0 : 1;
      }
    }
  }
  return misses;
}

int main() {
  check_store_staging();
  int wrong_rule = 0;
  for (int T : {64, 200, 1000, 4096})
    for (int Np : {256, 512, 4096})
      for (unsigned seed = 1; seed <= 3; ++seed) {
        CHECK(row_plane_misses(T, Np, seed, 128) == 0,
              "a read GEMM reads a plane region the row kernels did not write");
        wrong_rule += row_plane_misses(T, Np, seed, 64);
      }
  CHECK(wrong_rule > 0, "the plane-coverage check does not catch a wrong store rule");
  const int bns[] = {128, 256};
  for (int bn : bns) {
    check_gemm_order(32768, 32000, 128, bn, 1, 1, 16);
    check_gemm_order(4096, 4224, 128, bn, 3, 2, 16);
    check_gemm_order(300, 520, 128, bn, 2, 3, 16);
    check_gemm_order(129, 64, 128, bn, 1, 1, 16);
    check_gemm_order(2048, 384, 128, bn, 1, 32, 16);
  }
  int n_geometries = 0;
  for (int H = 64; H <= 2368; H += 16)
    for (int Hs : {8, 16}) {
      if (H % Hs) continue;
      for (int CL : {2, 4, 8})
        for (int rev = 0; rev < 2; ++rev)
          for (int nm = 1; nm <= 2; ++nm) {
            const ClusterLayout L = cluster_layout(H, Hs, CL, rev != 0, 512, 520, 2);
            if (!accepted(H, Hs, CL, rev != 0, L)) continue;
            ++n_geometries;
            if (H % 256 == 0 || H == 64 || H == 128 || H == 768)
              check_cluster(H, Hs, CL, rev != 0, nm);
          }
    }
  CHECK(n_geometries > 0, "no cluster geometry accepted");
  if (failures) {
    std::printf("%d failures\n", failures);
    return 1;
  }
  std::printf("ok (%d cluster geometries accepted)\n", n_geometries);
  return 0;
}
