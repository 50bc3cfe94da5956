// The dense products around the core scan on the tcgen05 GEMM of
// tc_gemm.cuh (BF16 operands, FP32 accumulation in tensor memory):
//
//   input projections  Wx = x W^T,  Wgx = x Wg^T + bg      (core.py:280-283)
//     forward: one launch, two problems sharing the A operand x;
//     reverse: dx = dWx W + dWgx Wg (one launch, the two pairs accumulate in
//     one accumulator) and dW = dWx^T x, dWg = dWgx^T x (one launch, two
//     problems);
//   recurrent-matrix gradient  grad[Ug; A] = [dWgx, dA]^T y over all (b, t)
//     (batched_runtime.py:1474-1481): one launch, two problems;
//   read output  out(cat[y, b, retrieved]) + long_gain * long  (read.py:435-438)
//     forward: one launch accumulating three operand pairs (no concatenated
//     copy: y and b are read in place from the U tape) with the bias and the
//     FP32 long-channel term in the epilogue; reverse: the three input
//     gradients as three problems of one launch, and the weight gradient as
//     three problems writing the column blocks of dW.
//
// Under autocast the reference runs these as cuBLAS GEMMs on BF16 casts of
// the FP32 parameters with BF16 outputs (the bias cast to BF16 before it is
// added); the epilogue here follows those rounding points.
#include <climits>

#include "../../include/dabsn_b200.h"
#include "common.cuh"
#include "tc_gemm.cuh"

namespace dabsn {
namespace {

using tcg::bf16;
constexpr int PBN = 256;  // output tile width

tcg::Args proj_args(int M, int N, int K, int nprob) {
  tcg::Args t;
  memset(&t, 0, sizeof(t));
  t.nprob = nprob;
  t.batch = 1;
  t.M = M;
  t.N = N;
  t.K = K;
  t.skip = tcg::SKIP_NONE;
  t.T = M;
  t.status = device_status();
  return t;
}

int launch_proj(int layout, const tcg::Args& t, cudaStream_t st, const char* what) {
  using TL = tcg::Tile<PBN>;
  const void* kern = layout == tcg::LNT ? (const void*)tcg::gemm_kernel<tcg::LNT, PBN>
                   : layout == tcg::LNN ? (const void*)tcg::gemm_kernel<tcg::LNN, PBN>
                                        : (const void*)tcg::gemm_kernel<tcg::LTN, PBN>;
  if (!kernel_prepared(kern, (int)TL::SMEM)) return DABSN_ERR_LAUNCH;
  const unsigned grid = tcg::grid_size(t, PBN);
  if (layout == tcg::LNT)
    tcg::gemm_kernel<tcg::LNT, PBN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  else if (layout == tcg::LNN)
    tcg::gemm_kernel<tcg::LNN, PBN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  else
    tcg::gemm_kernel<tcg::LTN, PBN><<<grid, tcg::THREADS, TL::SMEM, st>>>(t);
  return launch_status(what);
}

bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }

bool sizes_ok(int64_t M, int64_t D, int64_t H, const char* what) {
  if (M <= 0 || D <= 0 || H <= 0 || D % 8 || H % 8 || M > INT32_MAX || D > INT32_MAX ||
      H > INT32_MAX) {
    set_error("%s: unsupported sizes M=%lld D=%lld H=%lld (D and H multiples of 8)", what,
              (long long)M, (long long)D, (long long)H);
    return false;
  }
  return true;
}


// Row-block glue of the projections' reverse passes: 64 rows per CTA, each
// thread owning 8 consecutive columns (16-byte BF16 / 32-byte FP32 words),
// column partial sums per block written to colpart[block][H] (summed by the
// caller: fixed order, no atomics).
constexpr int GLUE_ROWS = 64;
constexpr int GLUE_THREADS = 256;

// The read output projection's incoming FP32 gradient: its BF16 copy for the
// GEMMs, the long channel's gradient long_gain * grad (FP32), per-block column
// sums of the BF16 copy (the bias gradient, as autocast's addmm forms it from
// the BF16 gradient) and per-block partial sums of grad * long (the gain's
// gradient).
__global__ void __launch_bounds__(GLUE_THREADS) read_out_grad_prep_kernel(
    int R, int H, const float* __restrict__ grad, const float* __restrict__ lng,
    const float* __restrict__ lgain, bf16* __restrict__ gb, float* __restrict__ dlong,
    float* __restrict__ colpart, float* __restrict__ dotpart) {
  __shared__ float s_red[GLUE_THREADS / 32];
  const int r0 = blockIdx.x * GLUE_ROWS, r1 = min(R, r0 + GLUE_ROWS);
  const float g0 = lgain[0];
  float dot = 0.f;
  for (int c = threadIdx.x * 8; c < H; c += GLUE_THREADS * 8) {
    float cs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int r = r0; r < r1; ++r) {
      const size_t o = (size_t)r * H + c;
      const float4 ga = *reinterpret_cast<const float4*>(grad + o);
      const float4 gc = *reinterpret_cast<const float4*>(grad + o + 4);
      const float4 la = *reinterpret_cast<const float4*>(lng + o);
      const float4 lc = *reinterpret_cast<const float4*>(lng + o + 4);
      const float g[8] = {ga.x, ga.y, ga.z, ga.w, gc.x, gc.y, gc.z, gc.w};
      const float l[8] = {la.x, la.y, la.z, la.w, lc.x, lc.y, lc.z, lc.w};
      uint4 pk;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        h[e] = __floats2bfloat162_rn(g[2 * e], g[2 * e + 1]);
        const float2 hf = __bfloat1622float2(h[e]);
        cs[2 * e] += hf.x;
        cs[2 * e + 1] += hf.y;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) dot = fmaf(g[e], l[e], dot);
      *reinterpret_cast<uint4*>(gb + o) = pk;
      *reinterpret_cast<float4*>(dlong + o) = make_float4(g0 * g[0], g0 * g[1], g0 * g[2], g0 * g[3]);
      *reinterpret_cast<float4*>(dlong + o + 4) =
          make_float4(g0 * g[4], g0 * g[5], g0 * g[6], g0 * g[7]);
    }
    float* cp = colpart + (size_t)blockIdx.x * H + c;
    *reinterpret_cast<float4*>(cp) = make_float4(cs[0], cs[1], cs[2], cs[3]);
    *reinterpret_cast<float4*>(cp + 4) = make_float4(cs[4], cs[5], cs[6], cs[7]);
  }
  dot = warp_sum(dot);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = dot;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < GLUE_THREADS / 32; ++w) t += s_red[w];
    dotpart[blockIdx.x] = t;
  }
}

// Per-block column sums of a BF16 [R, H] matrix (a bias gradient).
__global__ void __launch_bounds__(GLUE_THREADS) colsum_bf16_kernel(int R, int H,
                                                                  const bf16* __restrict__ x,
                                                                  float* __restrict__ colpart) {
  const int r0 = blockIdx.x * GLUE_ROWS, r1 = min(R, r0 + GLUE_ROWS);
  for (int c = threadIdx.x * 8; c < H; c += GLUE_THREADS * 8) {
    float cs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int r = r0; r < r1; ++r) {
      const uint4 pk = *reinterpret_cast<const uint4*>(x + (size_t)r * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        cs[2 * e] += f.x;
        cs[2 * e + 1] += f.y;
      }
    }
    float* cp = colpart + (size_t)blockIdx.x * H + c;
    *reinterpret_cast<float4*>(cp) = make_float4(cs[0], cs[1], cs[2], cs[3]);
    *reinterpret_cast<float4*>(cp + 4) = make_float4(cs[4], cs[5], cs[6], cs[7]);
  }
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int dabsn_input_proj_fwd(int64_t M, int64_t D, int64_t H, const void* x, int64_t ldx,
                                    const void* W, const void* Wg, const float* bias_g, void* Wx,
                                    void* Wgx, void* stream) {
  if (!sizes_ok(M, D, H, "input_proj_fwd")) return DABSN_ERR_UNSUPPORTED;
  if (!a16(x) || !a16(W) || !a16(Wg) || !a16(Wx) || !a16(Wgx) || ldx % 8) {
    set_error("input_proj_fwd: operands must be 16-byte aligned (row stride a multiple of 8)");
    return DABSN_ERR_SHAPE;
  }
  tcg::Args t = proj_args((int)M, (int)H, (int)D, 2);
  const void* w[2] = {W, Wg};
  void* c[2] = {Wx, Wgx};
  for (int p = 0; p < 2; ++p) {
    if (!tcg::make_map_k(&t.p[p].ta, x, D, M, 1, ldx, M * ldx) ||
        !tcg::make_map_k(&t.p[p].tb, w[p], D, H, 1, D, H * D, PBN)) {
      set_error("input_proj_fwd: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    t.p[p].C = (bf16*)c[p];
    t.p[p].sC = M * H;
    t.p[p].ldc = (int)H;
  }
  t.p[1].bias = bias_g;
  t.epi.mode = 3;
  return launch_proj(tcg::LNT, t, (cudaStream_t)stream, "input_proj_fwd");
}

extern "C" int dabsn_input_proj_bwd(int64_t M, int64_t D, int64_t H, const void* x, int64_t ldx,
                                    const void* W, const void* Wg, const void* gWx,
                                    const void* gWgx, void* dx, void* dW, void* dWg,
                                    void* stream) {
  if (!sizes_ok(M, D, H, "input_proj_bwd")) return DABSN_ERR_UNSUPPORTED;
  if (!a16(x) || !a16(W) || !a16(Wg) || !a16(gWx) || !a16(gWgx) || !a16(dx) || !a16(dW) ||
      !a16(dWg) || ldx % 8) {
    set_error("input_proj_bwd: operands must be 16-byte aligned (row stride a multiple of 8)");
    return DABSN_ERR_SHAPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  // dx = dWx W + dWgx Wg: A [M][H] K-major, B [H][D] MN-major, two pairs
  tcg::Args t = proj_args((int)M, (int)D, (int)H, 1);
  t.dual = 1;
  if (dx) {
    if (!tcg::make_map_k(&t.p[0].ta, gWx, H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&t.p[0].tb, W, D, H, 1, D, H * D) ||
        !tcg::make_map_k(&t.p[0].ta2, gWgx, H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&t.p[0].tb2, Wg, D, H, 1, D, H * D)) {
      set_error("input_proj_bwd: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    t.p[0].C = (bf16*)dx;
    t.p[0].sC = M * D;
    t.p[0].ldc = (int)D;
    const int rc = launch_proj(tcg::LNN, t, st, "input_proj_dx");
    if (rc) return rc;
  }
  // dW = dWx^T x, dWg = dWgx^T x: A [M][H] and B [M][D], both MN-major
  tcg::Args w = proj_args((int)H, (int)D, (int)M, 2);
  const void* g[2] = {gWx, gWgx};
  void* c[2] = {dW, dWg};
  for (int p = 0; p < 2; ++p) {
    if (!tcg::make_map_mn(&w.p[p].ta, g[p], H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&w.p[p].tb, x, D, M, 1, ldx, M * ldx)) {
      set_error("input_proj_bwd: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    w.p[p].C = (bf16*)c[p];
    w.p[p].sC = H * D;
    w.p[p].ldc = (int)D;
  }
  return launch_proj(tcg::LTN, w, st, "input_proj_dw");
}

extern "C" int dabsn_rec_grad(int64_t M, int64_t H, const void* y, int64_t ldy, const void* gWgx,
                              const void* day, void* gUg, void* gA, void* stream) {
  if (!sizes_ok(M, H, H, "rec_grad")) return DABSN_ERR_UNSUPPORTED;
  if (!a16(y) || !a16(gWgx) || !a16(day) || !a16(gUg) || !a16(gA) || ldy % 8) {
    set_error("rec_grad: operands must be 16-byte aligned (row stride a multiple of 8)");
    return DABSN_ERR_SHAPE;
  }
  // grad Ug = dWgx^T y, grad A = dA^T y over the M = B*T rows
  tcg::Args w = proj_args((int)H, (int)H, (int)M, 2);
  const void* g[2] = {gWgx, day};
  void* c[2] = {gUg, gA};
  for (int p = 0; p < 2; ++p) {
    if (!tcg::make_map_mn(&w.p[p].ta, g[p], H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&w.p[p].tb, y, H, M, 1, ldy, M * ldy)) {
      set_error("rec_grad: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    w.p[p].C = (bf16*)c[p];
    w.p[p].sC = H * H;
    w.p[p].ldc = (int)H;
  }
  return launch_proj(tcg::LTN, w, (cudaStream_t)stream, "rec_grad");
}

extern "C" int dabsn_read_out_fwd(int64_t M, int64_t H, const void* y, int64_t ldy,
                                  const void* bud, int64_t ldb, const void* ret, int64_t ldr,
                                  const void* W, const float* bias, const float* addend,
                                  const float* add_scale, float* out, void* stream) {
  if (!sizes_ok(M, H, H, "read_out_fwd")) return DABSN_ERR_UNSUPPORTED;
  if (!a16(y) || !a16(bud) || !a16(ret) || !a16(W) || !a16(out) || !a16(addend) || ldy % 8 ||
      ldb % 8 || ldr % 8) {
    set_error("read_out_fwd: operands must be 16-byte aligned (row strides multiples of 8)");
    return DABSN_ERR_SHAPE;
  }
  // out = bf16(y W0^T + b W1^T + r W2^T + bias) + add_scale * addend, W = [W0 W1 W2]
  tcg::Args t = proj_args((int)M, (int)H, (int)H, 1);
  t.dual = 2;
  const long long ldw = 3 * H;
  if (!tcg::make_map_k(&t.p[0].ta, y, H, M, 1, ldy, M * ldy) ||
      !tcg::make_map_k(&t.p[0].tb, W, H, H, 1, ldw, H * ldw, PBN) ||
      !tcg::make_map_k(&t.p[0].ta2, bud, H, M, 1, ldb, M * ldb) ||
      !tcg::make_map_k(&t.p[0].tb2, (const bf16*)W + H, H, H, 1, ldw, H * ldw, PBN) ||
      !tcg::make_map_k(&t.p[0].ta3, ret, H, M, 1, ldr, M * ldr) ||
      !tcg::make_map_k(&t.p[0].tb3, (const bf16*)W + 2 * H, H, H, 1, ldw, H * ldw, PBN)) {
    set_error("read_out_fwd: tensor map encoding failed");
    return DABSN_ERR_LAUNCH;
  }
  t.p[0].bias = bias;
  t.epi.mode = 4;
  t.epi.C32 = out;
  t.epi.addend = addend;
  t.epi.add_scale = add_scale;
  t.epi.ld32 = H;
  return launch_proj(tcg::LNT, t, (cudaStream_t)stream, "read_out_fwd");
}

extern "C" int dabsn_read_out_bwd(int64_t M, int64_t H, const void* y, int64_t ldy,
                                  const void* bud, int64_t ldb, const void* ret, int64_t ldr,
                                  const void* W, const void* gout, void* dy, void* dbud,
                                  void* dret, void* dW, void* stream) {
  if (!sizes_ok(M, H, H, "read_out_bwd")) return DABSN_ERR_UNSUPPORTED;
  if (!a16(y) || !a16(bud) || !a16(ret) || !a16(W) || !a16(gout) || !a16(dy) || !a16(dbud) ||
      !a16(dret) || !a16(dW) || ldy % 8 || ldb % 8 || ldr % 8) {
    set_error("read_out_bwd: operands must be 16-byte aligned (row strides multiples of 8)");
    return DABSN_ERR_SHAPE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const long long ldw = 3 * H;
  // d input i = gout W_i: A [M][H] K-major, B_i [H][H] (row stride 3H) MN-major
  tcg::Args t = proj_args((int)M, (int)H, (int)H, 3);
  void* din[3] = {dy, dbud, dret};
  for (int p = 0; p < 3; ++p) {
    if (!tcg::make_map_k(&t.p[p].ta, gout, H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&t.p[p].tb, (const bf16*)W + p * H, H, H, 1, ldw, H * ldw)) {
      set_error("read_out_bwd: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    t.p[p].C = (bf16*)din[p];
    t.p[p].sC = M * H;
    t.p[p].ldc = (int)H;
  }
  int rc = launch_proj(tcg::LNN, t, st, "read_out_dinputs");
  if (rc) return rc;
  // dW_i = gout^T input_i: both MN-major, into columns [iH, (i+1)H) of dW
  tcg::Args w = proj_args((int)H, (int)H, (int)M, 3);
  const void* in[3] = {y, bud, ret};
  const long long ld[3] = {ldy, ldb, ldr};
  for (int p = 0; p < 3; ++p) {
    if (!tcg::make_map_mn(&w.p[p].ta, gout, H, M, 1, H, M * H) ||
        !tcg::make_map_mn(&w.p[p].tb, in[p], H, M, 1, ld[p], M * ld[p])) {
      set_error("read_out_bwd: tensor map encoding failed");
      return DABSN_ERR_LAUNCH;
    }
    w.p[p].C = (bf16*)dW + p * H;
    w.p[p].sC = H * ldw;
    w.p[p].ldc = (int)ldw;
  }
  return launch_proj(tcg::LTN, w, st, "read_out_dweight");
}

extern "C" int64_t dabsn_glue_blocks(int64_t R) { return (R + GLUE_ROWS - 1) / GLUE_ROWS; }

extern "C" int dabsn_read_out_grad_prep(int64_t R, int64_t H, const float* grad,
                                        const float* long_channel, const float* long_gain,
                                        void* grad_bf16, float* dlong, float* colpart,
                                        float* dotpart, void* stream) {
  if (R <= 0 || H <= 0 || H % 8 || R > INT32_MAX || H > INT32_MAX) {
    set_error("read_out_grad_prep: unsupported sizes R=%lld H=%lld (H a multiple of 8)",
              (long long)R, (long long)H);
    return DABSN_ERR_UNSUPPORTED;
  }
  const unsigned grid = (unsigned)dabsn_glue_blocks(R);
  read_out_grad_prep_kernel<<<grid, GLUE_THREADS, 0, (cudaStream_t)stream>>>(
      (int)R, (int)H, grad, long_channel, long_gain, (bf16*)grad_bf16, dlong, colpart, dotpart);
  return launch_status("read_out_grad_prep");
}

extern "C" int dabsn_colsum_bf16(int64_t R, int64_t H, const void* x, float* colpart,
                                 void* stream) {
  if (R <= 0 || H <= 0 || H % 8 || R > INT32_MAX || H > INT32_MAX) {
    set_error("colsum_bf16: unsupported sizes R=%lld H=%lld (H a multiple of 8)", (long long)R,
              (long long)H);
    return DABSN_ERR_UNSUPPORTED;
  }
  const unsigned grid = (unsigned)dabsn_glue_blocks(R);
  colsum_bf16_kernel<<<grid, GLUE_THREADS, 0, (cudaStream_t)stream>>>((int)R, (int)H,
                                                                      (const bf16*)x, colpart);
  return launch_status("colsum_bf16");
}
