// Readout + mean cross-entropy without materialised logits, on the tcgen05
// GEMM of tc_gemm.cuh (BF16 operands, FP32 accumulation in TMEM).
//
// Reference: src/dabsn/runtime/loss.py:52-231 (`ChunkedLinearCrossEntropy`,
// `chunked_linear_cross_entropy`): logits = hidden W^T + b (BF16 under
// autocast), loss = mean over rows whose target is not ignore_index of
// logsumexp(logits) - logits[target].
//
// Forward: one GEMM over all rows whose epilogue keeps, per row and per
// 128-wide vocabulary tile, the tile's maximum and sum of exponentials and the
// target's logit; a merge kernel turns the tiles into each row's log-sum-exp.
// Reverse: the same GEMM with an epilogue writing BF16
// dlogits = scale (softmax - onehot); then dH = dlogits W (NN) and
// dW = dlogits^T H (TN) on the same tensor cores.
#include "../../include/dabsn_b200.h"
#include "common.cuh"
#include "tc_gemm.cuh"

namespace dabsn {
namespace {

using tcg::bf16;

// Also checks the targets: one that is neither ignore_index nor in [0, V)
// makes the row's target logit NaN (so the loss is NaN) and records status 7,
// raised by the host at its next synchronisation, where the reference's
// gather raises.
__global__ void __launch_bounds__(256) lse_merge_kernel(long long rows, int ntiles,
                                                        const float* part_m,
                                                        const float* part_s, float* lse,
                                                        const int64_t* targets, int ignore_index,
                                                        long long V, float* tgt_logit,
                                                        int* status) {
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const long long tg = targets[r];
  if (tg != ignore_index && (tg < 0 || tg >= V)) {
    tgt_logit[r] = __int_as_float(0x7fc00000);
    if (status) atomicExch(status, 7);
  }
  const float* pm = part_m + (size_t)r * ntiles;
  const float* ps = part_s + (size_t)r * ntiles;
  float m = -INFINITY;
  for (int i = 0; i < ntiles; ++i) m = fmaxf(m, pm[i]);
  float s = 0.f;
  for (int i = 0; i < ntiles; ++i)
    if (pm[i] > -INFINITY) s += ps[i] * __expf(pm[i] - m);
  lse[r] = m + __logf(s);
}

// Output tile width of the readout GEMMs: 256, or 128 with
// DABSN_B200_CE_BN=128 (the workspace is sized for 128, an upper bound).
constexpr int CE_BN = 128;

int ce_bn() {
  const char* e = getenv("DABSN_B200_CE_BN");  // read per launch, like the other switches
  return (e && atoi(e) == 128) ? 128 : 256;
}

template <int BN>
int launch_tc_gemm_bn(int layout, const tcg::Args& t, cudaStream_t st, const char* what) {
  using TL = tcg::Tile<BN>;
  const void* kern = layout == tcg::LNT ? (const void*)tcg::gemm_kernel<tcg::LNT, BN>
                   : layout == tcg::LNN ? (const void*)tcg::gemm_kernel<tcg::LNN, BN>
                                        : (const void*)tcg::gemm_kernel<tcg::LTN, BN>;
  if (!kernel_prepared(kern, (int)TL::SMEM)) return DABSN_ERR_LAUNCH;
  const unsigned grid = tcg::grid_size(t, BN);
  if (layout == tcg::LNT)
    tcg::gemm_kernel<tcg::LNT, BN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  else if (layout == tcg::LNN)
    tcg::gemm_kernel<tcg::LNN, BN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  else
    tcg::gemm_kernel<tcg::LTN, BN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  return launch_status(what);
}

int launch_tc_gemm(int layout, const tcg::Args& t, cudaStream_t st, const char* what) {
  return ce_bn() == 256 ? launch_tc_gemm_bn<256>(layout, t, st, what)
                        : launch_tc_gemm_bn<128>(layout, t, st, what);
}

tcg::Args base_args(int M, int N, int K) {
  tcg::Args t;
  memset(&t, 0, sizeof(t));
  t.nprob = 1;
  t.batch = 1;
  t.M = M;
  t.N = N;
  t.K = K;
  t.skip = tcg::SKIP_NONE;
  t.T = M;
  t.status = device_status();
  return t;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int64_t dabsn_linear_ce_ld(int64_t V) { return (V + 127) / 128 * 128; }

extern "C" size_t dabsn_linear_ce_workspace_floats(int64_t rows, int64_t V) {
  return (size_t)2 * rows * ((V + CE_BN - 1) / CE_BN);
}

extern "C" int dabsn_linear_ce_fwd(int64_t rows, int64_t V, int64_t D, const void* hidden,
                                   const void* weight, const float* bias, const int64_t* targets,
                                   int ignore_index, int round_bf16, float* lse, float* tgt_logit,
                                   float* workspace, void* stream) {
  if (rows <= 0 || V <= 0 || D <= 0 || D % 8 || rows > INT32_MAX || V > INT32_MAX) {
    set_error("linear_ce_fwd: unsupported sizes rows=%lld V=%lld D=%lld (D a multiple of 8)",
              (long long)rows, (long long)V, (long long)D);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (!aligned16(hidden) || !aligned16(weight)) {
    set_error("linear_ce_fwd: hidden and weight must be 16-byte aligned");
    return DABSN_ERR_SHAPE;
  }
  const int ntiles = (int)((V + ce_bn() - 1) / ce_bn());
  tcg::Args t = base_args((int)rows, (int)V, (int)D);
  if (!tcg::make_map_k(&t.p[0].ta, hidden, D, rows, 1, D, rows * D) ||
      !tcg::make_map_k(&t.p[0].tb, weight, D, V, 1, D, V * D, ce_bn())) {
    set_error("linear_ce_fwd: tensor map encoding failed");
    return DABSN_ERR_LAUNCH;
  }
  t.epi.mode = 1;
  t.epi.bias = bias;
  t.epi.targets = targets;
  t.epi.ignore_index = ignore_index;
  t.epi.round_bf16 = round_bf16;
  t.epi.part_m = workspace;
  t.epi.part_s = workspace + (size_t)rows * ntiles;
  t.epi.ldp = ntiles;
  t.epi.tgt_logit = tgt_logit;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = launch_tc_gemm(tcg::LNT, t, st, "linear_ce_logits");
  if (rc) return rc;
  lse_merge_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(
      rows, ntiles, t.epi.part_m, t.epi.part_s, lse, targets, ignore_index, V, tgt_logit,
      device_status());
  return launch_status("linear_ce_lse");
}

extern "C" int dabsn_linear_ce_bwd(int64_t rows, int64_t V, int64_t D, const void* hidden,
                                   const void* weight, const float* bias, const int64_t* targets,
                                   int ignore_index, int round_bf16, const float* lse,
                                   const float* scale, void* dlogits, void* dhidden,
                                   float* dweight, int accumulate, void* stream) {
  if (rows <= 0 || V <= 0 || D <= 0 || D % 8 || rows > INT32_MAX || V > INT32_MAX) {
    set_error("linear_ce_bwd: unsupported sizes rows=%lld V=%lld D=%lld", (long long)rows,
              (long long)V, (long long)D);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (!aligned16(hidden) || !aligned16(weight) || !aligned16(dlogits) || !aligned16(dhidden) ||
      !aligned16(dweight)) {
    set_error("linear_ce_bwd: operands must be 16-byte aligned");
    return DABSN_ERR_SHAPE;
  }
  const int64_t Vp = dabsn_linear_ce_ld(V);
  cudaStream_t st = (cudaStream_t)stream;
  // dlogits = scale (softmax - onehot), [rows][Vp] BF16
  tcg::Args t = base_args((int)rows, (int)V, (int)D);
  if (!tcg::make_map_k(&t.p[0].ta, hidden, D, rows, 1, D, rows * D) ||
      !tcg::make_map_k(&t.p[0].tb, weight, D, V, 1, D, V * D, ce_bn())) {
    set_error("linear_ce_bwd: tensor map encoding failed");
    return DABSN_ERR_LAUNCH;
  }
  t.p[0].C = (bf16*)dlogits;
  t.p[0].sC = rows * Vp;
  t.p[0].ldc = (int)Vp;
  t.epi.mode = 2;
  t.epi.bias = bias;
  t.epi.targets = targets;
  t.epi.ignore_index = ignore_index;
  t.epi.round_bf16 = round_bf16;
  t.epi.lse = lse;
  t.epi.scale = scale;
  int rc = launch_tc_gemm(tcg::LNT, t, st, "linear_ce_dlogits");
  if (rc) return rc;
  // dH = dlogits W: A [rows][V] K-major, B [V][D] MN-major
  tcg::Args h = base_args((int)rows, (int)D, (int)V);
  if (!tcg::make_map_k(&h.p[0].ta, dlogits, V, rows, 1, Vp, rows * Vp) ||
      !tcg::make_map_mn(&h.p[0].tb, weight, D, V, 1, D, V * D)) {
    set_error("linear_ce_bwd: tensor map encoding failed");
    return DABSN_ERR_LAUNCH;
  }
  h.p[0].C = (bf16*)dhidden;
  h.p[0].sC = rows * D;
  h.p[0].ldc = (int)D;
  rc = launch_tc_gemm(tcg::LNN, h, st, "linear_ce_dhidden");
  if (rc) return rc;
  // dW (+)= dlogits^T H in FP32: A stored [rows][V] (MN-major), B [rows][D]
  // (MN-major)
  tcg::Args w = base_args((int)V, (int)D, (int)rows);
  if (!tcg::make_map_mn(&w.p[0].ta, dlogits, V, rows, 1, Vp, rows * Vp) ||
      !tcg::make_map_mn(&w.p[0].tb, hidden, D, rows, 1, D, rows * D)) {
    set_error("linear_ce_bwd: tensor map encoding failed");
    return DABSN_ERR_LAUNCH;
  }
  w.epi.mode = accumulate ? 6 : 5;
  w.epi.C32 = dweight;
  w.epi.ld32 = D;
  w.p[0].ldc = (int)D;
  return launch_tc_gemm(tcg::LTN, w, st, "linear_ce_dweight");
}
