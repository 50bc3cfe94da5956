// Persistent cluster scan for the DABSN recurrent core, forward and reverse.
//
// Mathematics: src/dabsn/kernels/batched_runtime.py:38-158 (forward step) and
// :299-466 (reverse step) of the reference; the recurrence is restated in the
// oracle (oracle/dabsn_oracle.py, core_scan).
//
// Decomposition.  One thread-block cluster of P CTAs advances a tile of Bt
// sequences through all T steps.  CTA r of the cluster owns units
// [r*Hs, (r+1)*Hs) of the state: it keeps those units' budget / energy /
// saturation in registers for the whole scan (one (sequence, unit) element per
// thread) and keeps, in registers too, the rows of [Ug;A] (forward) or the
// columns of [Ug;A] (reverse) that those units need, spread WR values per
// thread (persistent-RNN layout, see reg_dot in matvec.cuh).  A step reads only
// the recurrent input vector from shared memory.  The only cross-unit
// dependence of a step is that product, which needs every unit of y (forward)
// or of [dgate;dexpr] (reverse): each CTA writes its slice of the vector into
// every CTA's shared memory with st.async, which completes transaction bytes
// on the receiving CTA's mbarrier; a CTA waits (bounded) on its own mbarrier
// for the step's bytes before reading the vector (a CTA barrier when P = 1).
// The vector buffer is double buffered, so one phase per step is enough.
// Forward inputs arrive through a cp.async ring several steps ahead of use;
// the reverse pass loads its inputs two steps ahead.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dabsn_b200.h"
#include "common.cuh"
#include "core_math.cuh"
#include "matvec.cuh"

namespace dabsn {


constexpr int kThreads = 256;
// Depth (in steps) of the forward input ring: step tau's inputs are copied
// kRing - 2 steps before their first use.
constexpr int kRing = 8;

struct ScanGeom {
  int B, T, H;
  int P;   // CTAs per cluster
  int Hs;  // units per CTA
  int Bt;  // sequences per cluster (Bt * Hs <= kThreads)
  int Kp;  // shared vector length: >= contraction length and >= WR * L
  int L;   // lanes sharing one output row of the product
  int WR;  // weight values held in registers per thread
};

template <typename Act>
struct CoreFwdArgs {
  const Act* Wx;
  const Act* Wgx;
  const Act* rec;  // [2H, H] = cat(Ug, A) in the activation dtype
  CoreParams p;
  const float* init_b;
  const float* init_e;
  const float* init_c;
  Act* U;      // [B,T,2H]
  Act* nov;    // [B,T,H]
  Act* plast;
  Act* expr;
  Act* write;
  Act* energy;
  Act* sat;
  Act* gate;
  Act* fin_b;  // [B,H]
  Act* fin_e;
  Act* fin_c;
  int* status;  // bounded-wait status word
  ScanGeom g;
};

template <typename Act>
struct CoreBwdArgs {
  // Saved forward tapes (activation dtype).
  const Act* U;       // [B,T,2H]
  const Act* energy;  // e_tape (pre-update energy)
  const Act* sat;     // c_tape (post-update saturation)
  const Act* gate;    // s_tape
  const Act* plast;
  const Act* expr;
  const Act* rec;     // [2H, H] = cat(Ug, A), activation dtype
  CoreParams p;
  const float* init_b;
  const float* init_c;
  // Upstream gradients, FP32; nullptr means zero.
  const float* gU;  // [B,T,2H]
  const float* gnov;  // [B,T,H]
  const float* gp;
  const float* gay;
  const float* gwrite;
  const float* ge;
  const float* gc;
  const float* gfin_b;  // [B,H]
  const float* gfin_e;
  const float* gfin_c;
  // Outputs.
  Act* gWx;   // [B,T,H]   gradient of Wx  (= gpre)
  Act* gWgx;  // [B,T,H]   gradient of Wgx (= dgate_pre)
  Act* day;   // [B,T,H]   expression adjoint (A half of the recurrent gradient)
  float* g_init_b;  // [B,H]
  float* g_init_e;
  float* g_init_c;
  float* partial;   // [B, 19, H] per-sequence parameter-gradient partial sums
  int* status;      // bounded-wait status word
  ScanGeom g;
};

template <typename T>
__device__ __forceinline__ void zero_smem(T* ptr, int count) {
  for (int i = threadIdx.x; i < count; i += blockDim.x) ptr[i] = T(0.0f);
}

// Write one value at byte offset `off` of every cluster CTA's vector buffer
// (`peer` holds their shared::cluster base addresses); a plain shared store
// when the cluster is a single CTA.
__device__ __forceinline__ void publish(float* local_base, const uint32_t* peer, int P,
                                        uint32_t off, float v) {
  if (P == 1) {
    *reinterpret_cast<float*>(reinterpret_cast<char*>(local_base) + off) = v;
  } else {
    for (int r = 0; r < P; ++r) st_cluster_f32(peer[r] + off, v);
  }
}

// Push one value to every cluster CTA (P > 1): an asynchronous store into the
// peer's vector buffer that signals that peer's mbarrier for the buffer.
__device__ __forceinline__ void push(const uint32_t* peer, const uint32_t* peer_bar, int P,
                                     uint32_t off, float v) {
  for (int r = 0; r < P; ++r) st_async_f32(peer[r] + off, v, peer_bar[r]);
}

// One barrier per step: cluster-wide (release/acquire) when the state is
// split over several CTAs, a CTA barrier otherwise.
__device__ __forceinline__ void step_barrier(int P) {
  if (P == 1) {
    __syncthreads();
  } else {
    cluster_sync_all();
  }
}

// Load this thread's register slice of the weight matrix: row o (< NO) and
// columns lk*4 + j*4L + c.  `at(o, k)` returns the element (zero outside).
template <int WR, typename F>
__device__ __forceinline__ void load_reg_weights(float (&w)[WR], int o, int lk, int L, F at) {
#pragma unroll
  for (int j = 0; j < WR / 4; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) w[4 * j + c] = at(o, lk * 4 + j * 4 * L + c);
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename Act, int WR>
__global__ void __launch_bounds__(kThreads, 1) core_scan_fwd_kernel(const CoreFwdArgs<Act> args) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const ScanGeom g = args.g;
  const int H = g.H;
  const int rank = g.P == 1 ? 0 : (int)cluster_ctarank();
  const int u0 = rank * g.Hs;
  const int b0 = blockIdx.y * g.Bt;
  const int nb = min(g.Bt, g.B - b0);  // live sequences in this tile
  const int NO = 2 * g.Hs;

  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);        // [2] one per y buffer
  uint32_t* peer = reinterpret_cast<uint32_t*>(smem_raw + 16);   // [16] peer ybuf bases
  uint32_t* pbar = peer + 16;                                    // [2][16] peer mbarriers
  float* ybuf = reinterpret_cast<float*>(smem_raw + 256);        // [2][Bt][Kp]
  float* acc = ybuf + 2 * g.Bt * g.Kp;                           // [2][Bt][NO]
  // [kRing][2 streams: Wx, Wgx][Bt][Hs] activation-dtype input ring
  unsigned char* ring = reinterpret_cast<unsigned char*>(acc + 2 * g.Bt * NO);
  const int row_bytes = g.Hs * (int)sizeof(Act);
  const int slot_bytes = 2 * g.Bt * row_bytes;
  // Copy the (sequence x unit) slices of Wx[tau] and Wgx[tau] into ring slot
  // tau % kRing with 4-byte asynchronous copies; always commits one group.
  // Each thread copies at most two 4-byte words per step; their source rows
  // and ring offsets are fixed for the whole scan, only tau moves.
  const unsigned char* cp_src[2] = {nullptr, nullptr};
  int cp_dst[2] = {0, 0};
  {
    const int wpr = row_bytes / 4;
    const int lim = (H - u0) * (int)sizeof(Act);  // bytes of real units in this slice
    for (int k = 0; k < 2; ++k) {
      const int wi = threadIdx.x + k * kThreads;
      if (wi >= 2 * nb * wpr) continue;
      const int st = wi / (nb * wpr), rem = wi % (nb * wpr);
      const int b = rem / wpr, off = (rem % wpr) * 4;
      if (off >= lim) continue;
      cp_src[k] = reinterpret_cast<const unsigned char*>((st == 0 ? args.Wx : args.Wgx) +
                                                         ((size_t)(b0 + b) * g.T) * H + u0) +
                  off;
      cp_dst[k] = (st * g.Bt + b) * row_bytes + off;
    }
  }
  const size_t step_bytes = (size_t)H * sizeof(Act);
  auto issue_inputs = [&](int tau) {
    if (tau < g.T) {
      unsigned char* slot = ring + (tau % kRing) * slot_bytes;
#pragma unroll
      for (int k = 0; k < 2; ++k)
        if (cp_src[k]) cp_async4(slot + cp_dst[k], cp_src[k] + (size_t)tau * step_bytes);
    }
    cp_async_commit();
  };
  auto ring_at = [&](int tau, int st, int b, int i) -> float {
    return to_f<Act>(reinterpret_cast<const Act*>(
        ring + (tau % kRing) * slot_bytes + (st * g.Bt + b) * row_bytes)[i]);
  };
  for (int tau = 0; tau < kRing - 1; ++tau) issue_inputs(tau);
  const bool multi = g.P > 1;
  const uint32_t tx = (uint32_t)(nb * H * sizeof(float));        // bytes per y_t

  zero_smem(ybuf, 2 * g.Bt * g.Kp);
  if (threadIdx.x < g.P) {
    peer[threadIdx.x] = map_shared_rank(ybuf, threadIdx.x);
    pbar[threadIdx.x] = map_shared_rank(&bar[0], threadIdx.x);
    pbar[16 + threadIdx.x] = map_shared_rank(&bar[1], threadIdx.x);
  }
  if (threadIdx.x == 0 && multi) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(&bar[0], tx);  // y_0
    if (g.T > 1) mbar_arrive_expect_tx(&bar[1], tx);  // y_1
  }

  // Register weights: local row i <- Ug[u0 + i, :], row Hs + i <- A[u0 + i, :].
  const int mo = threadIdx.x / g.L, lk = threadIdx.x % g.L;
  float w[WR];
  load_reg_weights<WR>(w, mo, lk, g.L, [&](int o, int k) -> float {
    if (o >= NO || k >= H) return 0.f;
    const int i = o < g.Hs ? o : o - g.Hs;
    if (u0 + i >= H) return 0.f;
    const int src = o < g.Hs ? u0 + i : H + u0 + i;
    return to_f<Act>(args.rec[(size_t)src * H + k]);
  });
  const float alpha = sigmoidf_(args.p.logit_alpha[0]);
  const float lam = softplusf_(args.p.log_lambda[0]);
  const float suppress = sigmoidf_(args.p.logit_c_suppress[0]);

  // Element ownership: element e = threadIdx.x = bl * Hs + i.
  const int e = threadIdx.x;
  const int bl = e / g.Hs, i = e % g.Hs, u = u0 + i;
  const bool live = e < nb * g.Hs && u < H;
  UnitConsts uc = live ? load_unit(args.p, u) : UnitConsts{};
  float st_b = 0.f, st_e = 0.f, st_c = 0.f, st_y = 0.f;
  const uint32_t yoff = (uint32_t)((bl * g.Kp + u) * sizeof(float));
  const uint32_t half = (uint32_t)(g.Bt * g.Kp * sizeof(float));
  size_t x0 = 0;
  if (live) {
    const size_t bs = (size_t)(b0 + bl) * H + u;
    st_b = args.init_b[bs];
    st_e = args.init_e[bs];
    st_c = args.init_c[bs];
    x0 = ((size_t)(b0 + bl) * g.T) * H + u;
    st_y = tanh_fast(to_f<Act>(args.Wx[x0]) + st_b);
  }
  // Every CTA's buffers and barriers exist before anyone signals them remotely.
  step_barrier(g.P);
  if (live) {
    if (multi)
      push(peer, pbar, g.P, yoff, round_act<Act>(st_y));
    else
      publish(ybuf, peer, 1, yoff, round_act<Act>(st_y));
  }
  if (!multi) __syncthreads();

  for (int t = 0; t < g.T; ++t) {
    const int cur = t & 1;
    if (multi) {
      // y_t has landed from every CTA; re-arm this buffer for y_{t+2}.
      mbar_wait_bounded(&bar[cur], (t >> 1) & 1, args.status, 1);
      if (threadIdx.x == 0 && t + 2 < g.T) mbar_arrive_expect_tx(&bar[cur], tx);
    }
    // [g_r ; a] for the owned units = y . [Ug;A]^T
    const float* yv = ybuf + cur * g.Bt * g.Kp;
    float* ac = acc + cur * g.Bt * NO;
    for (int b = 0; b < nb; ++b) {
      const float v = reg_dot<WR>(w, yv + b * g.Kp, lk, g.L);
      if (lk == 0 && mo < NO) ac[b * NO + mo] = v;
    }
    // Inputs of steps <= t+1 have landed (the kRing-3 newest copy groups may
    // still be in flight); the barrier makes every thread's copies visible.
    cp_async_wait<kRing - 3>();
    __syncthreads();
    // Slot (t-1) % kRing was last read in step t-1: refill it with t+kRing-1.
    issue_inputs(t + kRing - 1);
    if (live) {
      const float y = st_y, b = st_b, en = st_e;
      const float gr = round_act<Act>(ac[bl * NO + i]);
      const float a = round_act<Act>(ac[bl * NO + g.Hs + i]);
      const float wg_in = ring_at(t, 1, bl, i), wx_in = ring_at(t + 1, 0, bl, i);
      // Critical path first: y_{t+1} needs only the gate, the write and the
      // budget update; it is pushed before the energy / saturation work.
      const float s = hardsigmoidf_(wg_in + gr);
      const float pl = s * en;
      const float wr = pl * a;
      const float bn = (1.0f - alpha) * b + uc.beta + lam * wr;
      if (t + 1 < g.T) {
        st_y = tanh_fast(wx_in + bn);
        if (multi)
          push(peer, pbar + 16 * (cur ^ 1), g.P, (cur ^ 1) * half + yoff, round_act<Act>(st_y));
        else
          publish(ybuf, peer, 1, (cur ^ 1) * half + yoff, round_act<Act>(st_y));
      }
      const float n = tanh_fast(fabsf(a - b));
      const float c = uc.decay * st_c + (1.0f - uc.decay) * (n * (1.0f - en));
      const float neff = n * (1.0f - suppress * c);
      const float tb = tanh_fast(b);
      const float ksig = uc.ks * s + uc.ky * y + uc.kb * tb + uc.kn * neff + uc.kbias + uc.kc * c;
      const float rsig = uc.rs * s + uc.ry * y + uc.rb * tb + uc.rn * neff + uc.rbias + uc.rc * c;
      const float wcost = uc.kappa * exp_fast(0.5f * tanh_fast(ksig));
      const float recov = clamp01(uc.recover * exp_fast(0.5f * tanh_fast(rsig)));
      const float enew = clamp01(en + recov * (1.0f - en) - wcost * pl);
      const size_t row = x0 + (size_t)t * H;
      const size_t bt = (size_t)(b0 + bl) * g.T + t;
      args.U[bt * 2 * H + u] = from_f<Act>(y);
      args.U[bt * 2 * H + H + u] = from_f<Act>(bn);
      args.nov[row] = from_f<Act>(n);
      args.plast[row] = from_f<Act>(pl);
      args.expr[row] = from_f<Act>(a);
      args.write[row] = from_f<Act>(wr);
      args.energy[row] = from_f<Act>(en);
      args.sat[row] = from_f<Act>(c);
      args.gate[row] = from_f<Act>(s);
      st_b = bn;
      st_e = enew;
      st_c = c;
    }
    // Single CTA: publishes y_{t+1}.  Clusters synchronise through the
    // mbarriers instead (the product buffers are double buffered).
    if (!multi) __syncthreads();
  }
  // No CTA leaves while a peer might still write into its shared memory.
  if (multi) cluster_sync_all();

  if (live) {
    const size_t bs = (size_t)(b0 + bl) * H + u;
    args.fin_b[bs] = from_f<Act>(st_b);
    args.fin_e[bs] = from_f<Act>(st_e);
    args.fin_c[bs] = from_f<Act>(st_c);
  }
}

// ---------------------------------------------------------------------------
// Reverse
// ---------------------------------------------------------------------------
template <typename Act>
__device__ __forceinline__ StepIn load_step(const CoreBwdArgs<Act>& a, int b, int u, int t) {
  const int H = a.g.H;
  const size_t bt = (size_t)b * a.g.T + t;
  const size_t row = bt * H + u;
  StepIn s;
  s.y = to_f<Act>(a.U[bt * 2 * H + u]);
  s.b_prev = t > 0 ? to_f<Act>(a.U[(bt - 1) * 2 * H + H + u]) : a.init_b[(size_t)b * H + u];
  s.e_prev = to_f<Act>(a.energy[row]);
  s.c_prev = t > 0 ? to_f<Act>(a.sat[row - H]) : a.init_c[(size_t)b * H + u];
  s.gate = to_f<Act>(a.gate[row]);
  s.p = to_f<Act>(a.plast[row]);
  s.ay = to_f<Act>(a.expr[row]);
  s.c_t = to_f<Act>(a.sat[row]);
  s.gy0 = a.gU ? a.gU[bt * 2 * H + u] : 0.f;
  s.gb = a.gU ? a.gU[bt * 2 * H + H + u] : 0.f;
  s.gc = a.gc ? a.gc[row] : 0.f;
  s.gnov = a.gnov ? a.gnov[row] : 0.f;
  s.gp = a.gp ? a.gp[row] : 0.f;
  s.gay = a.gay ? a.gay[row] : 0.f;
  s.gw = a.gwrite ? a.gwrite[row] : 0.f;
  s.ge = a.ge ? a.ge[row] : 0.f;
  return s;
}

template <typename Act, int WR>
__global__ void __launch_bounds__(kThreads, 1) core_scan_bwd_kernel(const CoreBwdArgs<Act> args) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const ScanGeom g = args.g;
  const int H = g.H;
  const int rank = g.P == 1 ? 0 : (int)cluster_ctarank();
  const int u0 = rank * g.Hs;
  const int b0 = blockIdx.y * g.Bt;
  const int nb = min(g.Bt, g.B - b0);

  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);       // [2] one per vector buffer
  uint32_t* peer = reinterpret_cast<uint32_t*>(smem_raw + 16);  // [16]
  uint32_t* pbar = peer + 16;                                   // [2][16]
  float* vbuf = reinterpret_cast<float*>(smem_raw + 256);       // [2][Bt][Kp], Kp >= 2H
  float* acc = vbuf + 2 * g.Bt * g.Kp;                          // [2][Bt][Hs]
  const bool multi = g.P > 1;
  const uint32_t tx = (uint32_t)(nb * 2 * H * sizeof(float));   // bytes per step
  // Steps use buffer t & 1 from the top down: buffer s first serves top(s).
  const int top0 = ((g.T - 1) & 1) == 0 ? g.T - 1 : g.T - 2;
  const int top1 = ((g.T - 1) & 1) == 1 ? g.T - 1 : g.T - 2;

  zero_smem(vbuf, 2 * g.Bt * g.Kp);
  if (threadIdx.x < g.P) {
    peer[threadIdx.x] = map_shared_rank(vbuf, threadIdx.x);
    pbar[threadIdx.x] = map_shared_rank(&bar[0], threadIdx.x);
    pbar[16 + threadIdx.x] = map_shared_rank(&bar[1], threadIdx.x);
  }
  if (threadIdx.x == 0 && multi) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
    if (top0 >= 0) mbar_arrive_expect_tx(&bar[0], tx);
    if (top1 >= 0) mbar_arrive_expect_tx(&bar[1], tx);
  }
  // Register weights: row i of the local matrix is column u0 + i of [Ug;A].
  const int mo = threadIdx.x / g.L, lk = threadIdx.x % g.L;
  float w[WR];
  load_reg_weights<WR>(w, mo, lk, g.L, [&](int o, int k) -> float {
    if (o >= g.Hs || k >= 2 * H || u0 + o >= H) return 0.f;
    return to_f<Act>(args.rec[(size_t)k * H + u0 + o]);
  });
  const float alpha = sigmoidf_(args.p.logit_alpha[0]);
  const float lam = softplusf_(args.p.log_lambda[0]);
  const float sig_lam = sigmoidf_(args.p.log_lambda[0]);
  const float suppress = sigmoidf_(args.p.logit_c_suppress[0]);

  const int e = threadIdx.x;
  const int bl = e / g.Hs, i = e % g.Hs, u = u0 + i;
  const bool live = e < nb * g.Hs && u < H;
  const UnitConsts uc = live ? load_unit(args.p, u) : UnitConsts{};
  float gbn = 0.f, gen = 0.f, gcn = 0.f;
  float pacc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) pacc[j] = 0.f;
  float sacc0 = 0.f, sacc1 = 0.f, sacc2 = 0.f;
  // Software pipeline: the raw inputs of step t are loaded two steps ahead and
  // their carry-independent part (pre_step) is computed one step ahead, while
  // the CTA waits for its peers; after the wait only the short chain that is
  // linear in the carried adjoints remains on the critical path.
  StepIn nxt = {};
  StepPre pre = {};
  if (live) {
    const size_t bs = (size_t)(b0 + bl) * H + u;
    if (args.gfin_b) gbn = args.gfin_b[bs];
    if (args.gfin_e) gen = args.gfin_e[bs];
    if (args.gfin_c) gcn = args.gfin_c[bs];
    pre = pre_step(load_step(args, b0 + bl, u, g.T - 1), uc, suppress);
    if (g.T > 1) nxt = load_step(args, b0 + bl, u, g.T - 2);
  }
  const uint32_t half = (uint32_t)(g.Bt * g.Kp * sizeof(float));
  const uint32_t o1 = (uint32_t)((bl * g.Kp + u) * sizeof(float));
  const uint32_t o2 = (uint32_t)((bl * g.Kp + H + u) * sizeof(float));
  step_barrier(g.P);

  for (int t = g.T - 1; t >= 0; --t) {
    const int cur = t & 1;
    float k_gy0 = 0.f, k_gyen = 0.f, k_y = 0.f, k_gbstate = 0.f, k_dnov = 0.f;
    if (live) {
      const StepIn& in = pre.in;
      const float y = in.y, b_prev = in.b_prev, e_prev = in.e_prev, c_prev = in.c_prev;
      const float gate = in.gate, p = in.p, ay = in.ay, c_t = in.c_t;
      const float gb_new = in.gb + gbn;
      const float ge_new = gen;
      const float gc_new = gcn + in.gc;
      const float nov = pre.nov, tanh_b = pre.tanh_b, neff = pre.neff;
      const float tanh_k = pre.tanh_k, tanh_r = pre.tanh_r, exp_k = pre.exp_k, exp_r = pre.exp_r;
      const float wcost = pre.wcost, rec_pre = pre.rec_pre, recov = pre.recov;

      const float ge_pre = ge_new * pre.emask;
      const float g_bprev_state = gb_new * (1.0f - alpha);
      const float g_eprev_state = ge_pre * (1.0f - recov);
      float gp = in.gp + gb_new * lam * ay - ge_pre * wcost;
      const float gayv = in.gay + gb_new * lam * p;
      const float g_wcost = -ge_pre * p;
      const float g_recov = ge_pre * (1.0f - e_prev);
      const float d_expr_main = gayv + in.gw * p;
      gp = gp + in.gw * ay;
      const float g_ksig = g_wcost * wcost * 0.5f * (1.0f - tanh_k * tanh_k);
      const float g_rec_pre = g_recov * pre.rec_cg;
      const float g_rsig = g_rec_pre * rec_pre * 0.5f * (1.0f - tanh_r * tanh_r);
      const float g_gate_energy = g_ksig * uc.ks + g_rsig * uc.rs;
      const float gnov_eff = g_ksig * uc.kn + g_rsig * uc.rn;
      const float gc_energy = g_ksig * uc.kc + g_rsig * uc.rc;
      const float dgate_pre = (gp * e_prev + g_gate_energy) * pre.gmask;
      const float g_c_new = gc_new + gc_energy - gnov_eff * nov * suppress;
      const float g_stress = g_c_new * (1.0f - uc.decay);
      const float g_nov = gnov_eff * (1.0f - suppress * pre.c_new) + g_stress * (1.0f - e_prev);
      const float d_nov = (in.gnov + g_nov) * pre.dnov_scale;
      const float d_expr = d_expr_main + d_nov;

      // Publish [dgate_pre ; d_expr] (rounded to the product dtype) first.
      if (multi) {
        push(peer, pbar + 16 * cur, g.P, cur * half + o1, round_act<Act>(dgate_pre));
        push(peer, pbar + 16 * cur, g.P, cur * half + o2, round_act<Act>(d_expr));
      } else {
        publish(vbuf, peer, 1, cur * half + o1, round_act<Act>(dgate_pre));
        publish(vbuf, peer, 1, cur * half + o2, round_act<Act>(d_expr));
      }
      const float gy_energy = g_ksig * uc.ky + g_rsig * uc.ry;
      const float gb_energy = (g_ksig * uc.kb + g_rsig * uc.rb) * (1.0f - tanh_b * tanh_b);
      const float ge_gate = gp * gate;
      const float g_e_prev_cort = -g_stress * nov;
      const float g_c_prev = g_c_new * uc.decay;
      const float stress = pre.stress;
      const size_t row = ((size_t)(b0 + bl) * g.T + t) * H + u;
      args.gWgx[row] = from_f<Act>(dgate_pre);
      args.day[row] = from_f<Act>(d_expr);

      // Parameter-gradient partial sums (batched_runtime.py:431-447).
      pacc[0] += gb_new;
      pacc[1] += g_wcost * exp_k * uc.sigk;
      pacc[2] += g_rec_pre * exp_r * uc.recover * (1.0f - uc.recover);
      pacc[3] += g_ksig * gate;
      pacc[4] += g_ksig * y;
      pacc[5] += g_ksig * tanh_b;
      pacc[6] += g_ksig * neff;
      pacc[7] += g_ksig;
      pacc[8] += g_rsig * gate;
      pacc[9] += g_rsig * y;
      pacc[10] += g_rsig * tanh_b;
      pacc[11] += g_rsig * neff;
      pacc[12] += g_rsig;
      pacc[13] += g_c_new * (c_prev - stress) * uc.decay * (1.0f - uc.decay);
      pacc[14] += g_ksig * c_t;
      pacc[15] += g_rsig * c_t;
      sacc0 += gb_new * (-b_prev) * alpha * (1.0f - alpha);
      sacc1 += gb_new * (p * ay) * sig_lam;
      sacc2 += gnov_eff * nov * (-pre.c_new) * suppress * (1.0f - suppress);

      k_gy0 = in.gy0;
      k_gyen = gy_energy;
      k_y = y;
      k_gbstate = g_bprev_state + gb_energy;
      k_dnov = d_nov;
      gen = g_eprev_state + ge_gate + g_e_prev_cort + in.ge;
      gcn = g_c_prev;
      // Next step's carry-independent part while the peers' vectors arrive.
      if (t >= 1) pre = pre_step(nxt, uc, suppress);
      if (t >= 2) nxt = load_step(args, b0 + bl, u, t - 2);
    }
    if (multi) {
      // [dgate;dexpr] of step t has landed from every CTA; re-arm for t-2.
      const int top = cur ? top1 : top0;
      mbar_wait_bounded(&bar[cur], ((top - t) >> 1) & 1, args.status, 2);
      if (threadIdx.x == 0 && t - 2 >= 0) mbar_arrive_expect_tx(&bar[cur], tx);
    } else {
      __syncthreads();
    }
    // recurrent adjoint for the owned units = [dgate;dexpr] . [Ug;A][:, units]
    const float* vv = vbuf + cur * g.Bt * g.Kp;
    float* ac = acc + cur * g.Bt * g.Hs;
    for (int b = 0; b < nb; ++b) {
      const float v = reg_dot<WR>(w, vv + b * g.Kp, lk, g.L);
      if (lk == 0 && mo < g.Hs) ac[b * g.Hs + mo] = v;
    }
    __syncthreads();
    if (live) {
      const float radj = round_act<Act>(ac[bl * g.Hs + i]);
      const float gy = k_gy0 + k_gyen + radj;
      const float gpre = gy * (1.0f - k_y * k_y);
      gbn = k_gbstate - k_dnov + gpre;
      const size_t row = ((size_t)(b0 + bl) * g.T + t) * H + u;
      args.gWx[row] = from_f<Act>(gpre);
    }
  }

  if (live) {
    const size_t bs = (size_t)(b0 + bl) * H + u;
    args.g_init_b[bs] = gbn;
    args.g_init_e[bs] = gen;
    args.g_init_c[bs] = gcn;
    float* dst = args.partial + (size_t)(b0 + bl) * 19 * H + u;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[(size_t)j * H] = pacc[j];
    dst[(size_t)16 * H] = sacc0;
    dst[(size_t)17 * H] = sacc1;
    dst[(size_t)18 * H] = sacc2;
  }
  // No CTA leaves while a peer might still write into its shared memory.
  step_barrier(g.P);
}

// ---------------------------------------------------------------------------
// Host side: geometry selection and launch.
// ---------------------------------------------------------------------------
namespace {

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

constexpr int kWRChoices[] = {16, 32, 64};

inline size_t scan_smem_bytes(const ScanGeom& g, bool reverse, int act_bytes) {
  const int NO = reverse ? g.Hs : 2 * g.Hs;
  size_t s = 256 + sizeof(float) * ((size_t)2 * g.Bt * g.Kp + (size_t)2 * g.Bt * NO);
  if (!reverse) s += (size_t)kRing * 2 * g.Bt * g.Hs * act_bytes;
  return s;
}

std::mutex g_occ_mu;
std::map<std::tuple<const void*, int, int, int>, int> g_occ;  // (kernel, dev, P, smem) -> clusters

int max_active_clusters(const void* kernel, int P, size_t smem) {
  const int dev = current_device();
  auto key = std::make_tuple(kernel, dev, P, (int)smem);
  {
    std::lock_guard<std::mutex> lock(g_occ_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (!kernel_prepared(kernel, (int)smem) ||
      cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148 / P;
  }
  std::lock_guard<std::mutex> lock(g_occ_mu);
  g_occ[key] = n;
  return n;
}

// Cluster size P: the smallest whose per-thread weight slice fits WR <= 64
// registers (more CTAs per cluster cost a wider barrier, fewer cost registers
// and longer per-step products).  DABSN_B200_CLUSTER forces P.  Then L (lanes
// per output row), WR, and the fewest sequences per cluster that keep every
// cluster of the grid resident at once.
template <typename GetKernel>
bool choose_geom(GetKernel kernel_for, int B, int T, int H, bool reverse, int act_bytes,
                 ScanGeom* out) {
  const int K = reverse ? 2 * H : H;
  const char* force = getenv("DABSN_B200_CLUSTER");
  const int forced = force ? atoi(force) : 0;
  for (int P : {1, 2, 4, 8}) {
    if (forced && P != forced) continue;
    const int Hs = (H + P - 1) / P;
    if (Hs > kThreads) continue;
    // the forward input ring copies 4-byte words of every unit slice
    if (((size_t)H * act_bytes) % 4 || ((size_t)Hs * act_bytes) % 4) continue;
    const int NO = reverse ? Hs : 2 * Hs;
    if (NO > kThreads) continue;
    int L = 1;
    while (L < 32 && 2 * L * NO <= kThreads) L *= 2;
    const int need = round_up(K, 4 * L) / L;
    int WR = 0;
    for (int c : kWRChoices)
      if (!WR && c >= need) WR = c;
    if (!WR) continue;
    ScanGeom g{B, T, H, P, Hs, 1, std::max(round_up(K, 128), WR * L), L, WR};
    const void* kernel = kernel_for(WR);
    const int clusters = max_active_clusters(kernel, P, scan_smem_bytes(g, reverse, act_bytes));
    int Bt = std::max(1, (B + clusters - 1) / clusters);
    g.Bt = std::min(Bt, kThreads / Hs);
    *out = g;
    return true;
  }
  return false;
}

template <typename Kern, typename Args>
int launch_cluster(Kern kernel, const Args& a, size_t smem, cudaStream_t stream,
                   const char* what) {
  if (!kernel_prepared((const void*)kernel, (int)smem)) return DABSN_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.g.P, (a.g.B + a.g.Bt - 1) / a.g.Bt, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.g.P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) {
    set_error("%s launch: %s (P=%d Hs=%d Bt=%d L=%d WR=%d smem=%zu)", what,
              cudaGetErrorString(err), a.g.P, a.g.Hs, a.g.Bt, a.g.L, a.g.WR, smem);
    return DABSN_ERR_LAUNCH;
  }
  return DABSN_OK;
}

template <typename Act>
const void* fwd_kernel_for(int WR) {
  if (WR == 16) return (const void*)core_scan_fwd_kernel<Act, 16>;
  if (WR == 32) return (const void*)core_scan_fwd_kernel<Act, 32>;
  return (const void*)core_scan_fwd_kernel<Act, 64>;
}

template <typename Act>
const void* bwd_kernel_for(int WR) {
  if (WR == 16) return (const void*)core_scan_bwd_kernel<Act, 16>;
  if (WR == 32) return (const void*)core_scan_bwd_kernel<Act, 32>;
  return (const void*)core_scan_bwd_kernel<Act, 64>;
}

template <typename Act>
int core_fwd(CoreFwdArgs<Act>& a, cudaStream_t stream) {
  if (!choose_geom(fwd_kernel_for<Act>, a.g.B, a.g.T, a.g.H, false, sizeof(Act), &a.g)) {
    set_error("core_scan_fwd: hidden width %d does not fit the register-resident scan", a.g.H);
    return DABSN_ERR_UNSUPPORTED;
  }
  const size_t smem = scan_smem_bytes(a.g, false, sizeof(Act));
  if (a.g.WR == 16) return launch_cluster(core_scan_fwd_kernel<Act, 16>, a, smem, stream, "core_scan_fwd");
  if (a.g.WR == 32) return launch_cluster(core_scan_fwd_kernel<Act, 32>, a, smem, stream, "core_scan_fwd");
  return launch_cluster(core_scan_fwd_kernel<Act, 64>, a, smem, stream, "core_scan_fwd");
}

template <typename Act>
int core_bwd(CoreBwdArgs<Act>& a, cudaStream_t stream) {
  if (!choose_geom(bwd_kernel_for<Act>, a.g.B, a.g.T, a.g.H, true, sizeof(Act), &a.g)) {
    set_error("core_scan_bwd: hidden width %d does not fit the register-resident scan", a.g.H);
    return DABSN_ERR_UNSUPPORTED;
  }
  const size_t smem = scan_smem_bytes(a.g, true, sizeof(Act));
  if (a.g.WR == 16) return launch_cluster(core_scan_bwd_kernel<Act, 16>, a, smem, stream, "core_scan_bwd");
  if (a.g.WR == 32) return launch_cluster(core_scan_bwd_kernel<Act, 32>, a, smem, stream, "core_scan_bwd");
  return launch_cluster(core_scan_bwd_kernel<Act, 64>, a, smem, stream, "core_scan_bwd");
}

inline CoreParams to_params(const dabsn_core_params* p) {
  CoreParams q;
  q.beta = p->beta;
  q.log_kappa = p->log_kappa;
  q.logit_recover = p->logit_recover;
  q.k_s = p->k_s;
  q.k_y = p->k_y;
  q.k_b = p->k_b;
  q.k_n = p->k_n;
  q.k_bias = p->k_bias;
  q.r_s = p->r_s;
  q.r_y = p->r_y;
  q.r_b = p->r_b;
  q.r_n = p->r_n;
  q.r_bias = p->r_bias;
  q.logit_c_decay = p->logit_c_decay;
  q.k_c = p->k_c;
  q.r_c = p->r_c;
  q.logit_alpha = p->logit_alpha;
  q.log_lambda = p->log_lambda;
  q.logit_c_suppress = p->logit_c_suppress;
  return q;
}

bool check_sizes(int64_t B, int64_t T, int64_t H, const char* what) {
  if (B < 0 || T < 0 || H <= 0 || B > (1 << 24) || T > (1 << 26) || H > 65536) {
    set_error("%s: bad sizes B=%lld T=%lld H=%lld", what, (long long)B, (long long)T,
              (long long)H);
    return false;
  }
  return true;
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

template <typename Act>
static int core_fwd_entry(int64_t B, int64_t T, int64_t H, const void* Wx, const void* Wgx,
                          const void* rec, const dabsn_core_params* params, const float* init_b,
                          const float* init_e, const float* init_c, void* U, void* nov,
                          void* plast, void* expr, void* write, void* energy, void* sat,
                          void* gate, void* fin_b, void* fin_e, void* fin_c, void* stream) {
  CoreFwdArgs<Act> a;
  a.Wx = (const Act*)Wx;
  a.Wgx = (const Act*)Wgx;
  a.rec = (const Act*)rec;
  a.p = to_params(params);
  a.init_b = init_b;
  a.init_e = init_e;
  a.init_c = init_c;
  a.U = (Act*)U;
  a.nov = (Act*)nov;
  a.plast = (Act*)plast;
  a.expr = (Act*)expr;
  a.write = (Act*)write;
  a.energy = (Act*)energy;
  a.sat = (Act*)sat;
  a.gate = (Act*)gate;
  a.fin_b = (Act*)fin_b;
  a.fin_e = (Act*)fin_e;
  a.fin_c = (Act*)fin_c;
  a.status = device_status();
  a.g = ScanGeom{(int)B, (int)T, (int)H, 1, 1, 1, 128, 1, 1};
  return core_fwd<Act>(a, (cudaStream_t)stream);
}

extern "C" int dabsn_core_scan_fwd(int dtype, int64_t B, int64_t T, int64_t H, const void* Wx,
                                   const void* Wgx, const void* rec,
                                   const dabsn_core_params* params, const float* init_b,
                                   const float* init_e, const float* init_c, void* U, void* nov,
                                   void* plast, void* expr, void* write, void* energy, void* sat,
                                   void* gate, void* fin_b, void* fin_e, void* fin_c,
                                   void* stream) {
  if (!check_sizes(B, T, H, "core_scan_fwd")) return DABSN_ERR_SHAPE;
  if (B == 0) return DABSN_OK;
  if (dtype == DABSN_F32)
    return core_fwd_entry<float>(B, T, H, Wx, Wgx, rec, params, init_b, init_e, init_c, U, nov,
                                 plast, expr, write, energy, sat, gate, fin_b, fin_e, fin_c,
                                 stream);
  if (dtype == DABSN_BF16)
    return core_fwd_entry<__nv_bfloat16>(B, T, H, Wx, Wgx, rec, params, init_b, init_e, init_c,
                                         U, nov, plast, expr, write, energy, sat, gate, fin_b,
                                         fin_e, fin_c, stream);
  set_error("core_scan_fwd: unsupported dtype code %d", dtype);
  return DABSN_ERR_DTYPE;
}

template <typename Act>
static int core_bwd_entry(int64_t B, int64_t T, int64_t H, const void* U, const void* energy,
                          const void* sat, const void* gate, const void* plast, const void* expr,
                          const void* rec, const dabsn_core_params* params, const float* init_b,
                          const float* init_c, const float* gU, const float* gnov,
                          const float* gp, const float* gay, const float* gwrite, const float* ge,
                          const float* gc, const float* gfin_b, const float* gfin_e,
                          const float* gfin_c, void* gWx, void* gWgx, void* day, float* g_init_b,
                          float* g_init_e, float* g_init_c, float* partial, void* stream) {
  CoreBwdArgs<Act> a;
  a.U = (const Act*)U;
  a.energy = (const Act*)energy;
  a.sat = (const Act*)sat;
  a.gate = (const Act*)gate;
  a.plast = (const Act*)plast;
  a.expr = (const Act*)expr;
  a.rec = (const Act*)rec;
  a.p = to_params(params);
  a.init_b = init_b;
  a.init_c = init_c;
  a.gU = gU;
  a.gnov = gnov;
  a.gp = gp;
  a.gay = gay;
  a.gwrite = gwrite;
  a.ge = ge;
  a.gc = gc;
  a.gfin_b = gfin_b;
  a.gfin_e = gfin_e;
  a.gfin_c = gfin_c;
  a.gWx = (Act*)gWx;
  a.gWgx = (Act*)gWgx;
  a.day = (Act*)day;
  a.g_init_b = g_init_b;
  a.g_init_e = g_init_e;
  a.g_init_c = g_init_c;
  a.partial = partial;
  a.status = device_status();
  a.g = ScanGeom{(int)B, (int)T, (int)H, 1, 1, 1, 128, 1, 1};
  return core_bwd<Act>(a, (cudaStream_t)stream);
}

extern "C" int dabsn_core_scan_bwd(int dtype, int64_t B, int64_t T, int64_t H, const void* U,
                                   const void* energy, const void* sat, const void* gate,
                                   const void* plast, const void* expr, const void* rec,
                                   const dabsn_core_params* params, const float* init_b,
                                   const float* init_c, const float* gU, const float* gnov,
                                   const float* gp, const float* gay, const float* gwrite,
                                   const float* ge, const float* gc, const float* gfin_b,
                                   const float* gfin_e, const float* gfin_c, void* gWx,
                                   void* gWgx, void* day, float* g_init_b, float* g_init_e,
                                   float* g_init_c, float* partial, void* stream) {
  if (!check_sizes(B, T, H, "core_scan_bwd")) return DABSN_ERR_SHAPE;
  if (B == 0) return DABSN_OK;
  if (dtype == DABSN_F32)
    return core_bwd_entry<float>(B, T, H, U, energy, sat, gate, plast, expr, rec, params, init_b,
                                 init_c, gU, gnov, gp, gay, gwrite, ge, gc, gfin_b, gfin_e,
                                 gfin_c, gWx, gWgx, day, g_init_b, g_init_e, g_init_c, partial,
                                 stream);
  if (dtype == DABSN_BF16)
    return core_bwd_entry<__nv_bfloat16>(B, T, H, U, energy, sat, gate, plast, expr, rec, params,
                                         init_b, init_c, gU, gnov, gp, gay, gwrite, ge, gc,
                                         gfin_b, gfin_e, gfin_c, gWx, gWgx, day, g_init_b,
                                         g_init_e, g_init_c, partial, stream);
  set_error("core_scan_bwd: unsupported dtype code %d", dtype);
  return DABSN_ERR_DTYPE;
}
