// The two primitives of the dabsn.kernels surface outside the block path.
//
// permanent_delta_scan (reference: src/dabsn/kernels/permanent.py:56-110,
// 384-431): per sequence a state S [h x h] starts at zero and for t = 0..T-1
//     r_t = S k_t ;  S <- S + beta_t (v_t - r_t) k_t^T
// and the op returns r [B,T,h].  The reverse walks t = T-1..0 with the
// adjoint A = dL/dS_{t+1}:
//     dv_t    = beta_t A k_t
//     dbeta_t = <A k_t, v_t - r_t>
//     dk_t    = S_t^T g_t + beta_t (A^T v_t - S_t^T (A k_t) - A^T r_t)
//     A      <- A + (g_t - beta_t A k_t) k_t^T
// One CTA per sequence keeps S (and A) in shared memory, FP32, h <= 128.  The
// reverse first re-runs the forward storing S every 64 steps, then rebuilds
// S_t = S_{t+1} - beta_t (v_t - r_t) k_t^T from the nearest later checkpoint
// (at most 64 exact-algebra steps, so rounding cannot accumulate over T).
//
// local_field_gather (reference: src/dabsn/kernels/local_field.py:208-240):
// out[b,n,k,:] = x[b, patch[n,k], :]; the reverse sums, per source cell, the
// gradients of the (n, k) slots that read it through an inverse index (CSR,
// built by the caller), deterministic and without atomics.
#include <algorithm>

#include "../../include/dabsn_b200.h"
#include "common.cuh"

namespace dabsn {
namespace {

typedef __nv_bfloat16 bf16;

constexpr int PT = 256;      // threads per CTA
constexpr int CK = 64;       // checkpoint interval (steps)
constexpr int PMAX = 128;    // largest supported h

template <typename Act>
__device__ __forceinline__ void load_vec(float* dst, const Act* src, int h) {
  for (int i = threadIdx.x; i < h; i += blockDim.x) dst[i] = to_f<Act>(src[i]);
}

// r = S k (row v of S times k), rows split over warps, k split over lanes.
__device__ __forceinline__ void matvec_rows(const float* S, int ld, const float* k, float* r,
                                            int h) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int v = warp; v < h; v += nw) {
    float s = 0.f;
    for (int j = lane; j < h; j += 32) s = fmaf(S[v * ld + j], k[j], s);
    s = warp_sum(s);
    if (lane == 0) r[v] = s;
  }
}

template <typename Act>
__global__ void __launch_bounds__(PT) delta_fwd_kernel(int T, int h, const Act* k, const Act* v,
                                                       const Act* beta, Act* out, float* ckpt) {
  extern __shared__ float sm[];
  const int ld = h + 1;
  float* S = sm;                // [h][h+1]
  float* kk = S + h * ld;       // [h]
  float* vv = kk + h;           // [h]
  float* rr = vv + h;           // [h]
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < h * ld; i += blockDim.x) S[i] = 0.f;
  const int nck = (T + CK - 1) / CK;
  __syncthreads();
  for (int t = 0; t < T; ++t) {
    if (ckpt && t % CK == 0) {
      float* dst = ckpt + ((size_t)b * (nck + 1) + t / CK) * h * h;
      for (int i = threadIdx.x; i < h * h; i += blockDim.x) dst[i] = S[(i / h) * ld + i % h];
    }
    const size_t row = ((size_t)b * T + t) * h;
    load_vec<Act>(kk, k + row, h);
    load_vec<Act>(vv, v + row, h);
    const float bt = to_f<Act>(beta[(size_t)b * T + t]);
    __syncthreads();
    matvec_rows(S, ld, kk, rr, h);
    __syncthreads();
    for (int i = threadIdx.x; i < h; i += blockDim.x) out[row + i] = from_f<Act>(rr[i]);
    for (int i = threadIdx.x; i < h * h; i += blockDim.x) {
      const int a = i / h, c = i % h;
      S[a * ld + c] = fmaf(bt * (vv[a] - rr[a]), kk[c], S[a * ld + c]);
    }
    __syncthreads();
  }
  if (ckpt) {
    float* dst = ckpt + ((size_t)b * (nck + 1) + nck) * h * h;  // final state
    for (int i = threadIdx.x; i < h * h; i += blockDim.x) dst[i] = S[(i / h) * ld + i % h];
  }
}

template <typename Act>
__global__ void __launch_bounds__(PT) delta_bwd_kernel(int T, int h, const Act* k, const Act* v,
                                                       const Act* beta, const Act* recon,
                                                       const float* g, const float* ckpt,
                                                       Act* dk, Act* dv, Act* dbeta) {
  extern __shared__ float sm[];
  const int ld = h + 1;
  float* S = sm;                 // [h][h+1]
  float* A = S + h * ld;         // [h][h+1]
  float* kk = A + h * ld;
  float* vv = kk + h;
  float* rr = vv + h;
  float* gg = rr + h;
  float* ak = gg + h;            // A k
  float* w1 = ak + h;            // g - beta A k
  __shared__ float s_dbeta[8];
  const int b = blockIdx.x;
  const int nck = (T + CK - 1) / CK;
  for (int i = threadIdx.x; i < h * ld; i += blockDim.x) A[i] = 0.f;
  for (int t = T - 1; t >= 0; --t) {
    if ((t + 1) % CK == 0 || t == T - 1) {
      // exact state after step t: the checkpoint at t + 1 (or the final state)
      const int c = (t + 1) % CK == 0 ? (t + 1) / CK : nck;
      const float* src = ckpt + ((size_t)b * (nck + 1) + c) * h * h;
      for (int i = threadIdx.x; i < h * h; i += blockDim.x) S[(i / h) * ld + i % h] = src[i];
    }
    const size_t row = ((size_t)b * T + t) * h;
    load_vec<Act>(kk, k + row, h);
    load_vec<Act>(vv, v + row, h);
    load_vec<Act>(rr, recon + row, h);
    for (int i = threadIdx.x; i < h; i += blockDim.x) gg[i] = g[row + i];
    const float bt = to_f<Act>(beta[(size_t)b * T + t]);
    __syncthreads();
    // S_t = S_{t+1} - beta (v - r) k^T
    for (int i = threadIdx.x; i < h * h; i += blockDim.x) {
      const int a = i / h, c = i % h;
      S[a * ld + c] = fmaf(-bt * (vv[a] - rr[a]), kk[c], S[a * ld + c]);
    }
    matvec_rows(A, ld, kk, ak, h);  // A_{t+1} k
    __syncthreads();
    // dv, dbeta (row terms) and w1 = g - beta A k (used for S^T and the update)
    float part = 0.f;
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
      dv[row + i] = from_f<Act>(bt * ak[i]);
      part = fmaf(ak[i], vv[i] - rr[i], part);
      w1[i] = gg[i] - bt * ak[i];
    }
    part = warp_sum(part);
    if ((threadIdx.x & 31) == 0) s_dbeta[threadIdx.x >> 5] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += s_dbeta[w];
      dbeta[(size_t)b * T + t] = from_f<Act>(s);
    }
    // dk = S_t^T (g - beta A k) + beta A^T (v - r), one thread per column
    for (int j = threadIdx.x; j < h; j += blockDim.x) {
      float s1 = 0.f, s2 = 0.f;
      for (int a = 0; a < h; ++a) {
        s1 = fmaf(S[a * ld + j], w1[a], s1);
        s2 = fmaf(A[a * ld + j], vv[a] - rr[a], s2);
      }
      dk[row + j] = from_f<Act>(s1 + bt * s2);
    }
    __syncthreads();
    // A_t = A_{t+1} + (g - beta A k) k^T
    for (int i = threadIdx.x; i < h * h; i += blockDim.x) {
      const int a = i / h, c = i % h;
      A[a * ld + c] = fmaf(w1[a], kk[c], A[a * ld + c]);
    }
    __syncthreads();
  }
}

// x [B, C, D], patch [N, K] (cells of x) -> out [B, N, K, D]
template <typename Act>
__global__ void field_gather_kernel(long long total, int C, int N, int K, int D, const Act* x,
                                    const int64_t* patch, Act* out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    long long r = i / D;
    const int kk = (int)(r % K);
    r /= K;
    const int n = (int)(r % N);
    const long long b = r / N;
    const long long src = patch[(size_t)n * K + kk];
    out[i] = x[(b * C + src) * D + d];
  }
}

// grad_x[b, c, d] = sum over the slots reading cell c (CSR: flat slots
// n*K + k listed in order[offsets[c] .. offsets[c+1]])
template <typename Act>
__global__ void field_scatter_kernel(long long total, int C, int N, int K, int D, const Act* gout,
                                     const int64_t* order, const int64_t* offsets, Act* gx) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const long long bc = i / D;
    const int c = (int)(bc % C);
    const long long b = bc / C;
    float s = 0.f;
    for (long long q = offsets[c]; q < offsets[c + 1]; ++q)
      s += to_f<Act>(gout[(b * N * K + order[q]) * D + d]);
    gx[i] = from_f<Act>(s);
  }
}

size_t delta_fwd_smem(int h) { return ((size_t)h * (h + 1) + 3 * (size_t)h) * sizeof(float); }
size_t delta_bwd_smem(int h) { return ((size_t)2 * h * (h + 1) + 6 * (size_t)h) * sizeof(float); }

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" size_t dabsn_delta_ckpt_floats(int64_t B, int64_t T, int64_t h) {
  return (size_t)B * ((T + CK - 1) / CK + 1) * h * h;
}

extern "C" int dabsn_permanent_delta_fwd(int dtype, int64_t B, int64_t T, int64_t h, const void* k,
                                         const void* v, const void* beta, void* out,
                                         float* ckpt, void* stream) {
  if (B <= 0 || T <= 0 || h <= 0 || h > PMAX) {
    set_error("permanent_delta_fwd: unsupported sizes B=%lld T=%lld h=%lld (h <= %d)",
              (long long)B, (long long)T, (long long)h, PMAX);
    return DABSN_ERR_UNSUPPORTED;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = delta_fwd_smem((int)h);
  if (dtype == DABSN_F32) {
    if (!kernel_prepared((const void*)delta_fwd_kernel<float>, (int)smem)) return DABSN_ERR_LAUNCH;
    delta_fwd_kernel<float><<<(unsigned)B, PT, smem, st>>>((int)T, (int)h, (const float*)k,
                                                          (const float*)v, (const float*)beta,
                                                          (float*)out, ckpt);
  } else if (dtype == DABSN_BF16) {
    if (!kernel_prepared((const void*)delta_fwd_kernel<bf16>, (int)smem)) return DABSN_ERR_LAUNCH;
    delta_fwd_kernel<bf16><<<(unsigned)B, PT, smem, st>>>((int)T, (int)h, (const bf16*)k,
                                                         (const bf16*)v, (const bf16*)beta,
                                                         (bf16*)out, ckpt);
  } else {
    set_error("permanent_delta_fwd: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("permanent_delta_fwd");
}

extern "C" int dabsn_permanent_delta_bwd(int dtype, int64_t B, int64_t T, int64_t h, const void* k,
                                         const void* v, const void* beta, const void* recon,
                                         const float* g, const float* ckpt, void* dk, void* dv,
                                         void* dbeta, void* stream) {
  if (B <= 0 || T <= 0 || h <= 0 || h > PMAX) {
    set_error("permanent_delta_bwd: unsupported sizes B=%lld T=%lld h=%lld (h <= %d)",
              (long long)B, (long long)T, (long long)h, PMAX);
    return DABSN_ERR_UNSUPPORTED;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = delta_bwd_smem((int)h);
  if (dtype == DABSN_F32) {
    if (!kernel_prepared((const void*)delta_bwd_kernel<float>, (int)smem)) return DABSN_ERR_LAUNCH;
    delta_bwd_kernel<float><<<(unsigned)B, PT, smem, st>>>(
        (int)T, (int)h, (const float*)k, (const float*)v, (const float*)beta,
        (const float*)recon, g, ckpt, (float*)dk, (float*)dv, (float*)dbeta);
  } else if (dtype == DABSN_BF16) {
    if (!kernel_prepared((const void*)delta_bwd_kernel<bf16>, (int)smem)) return DABSN_ERR_LAUNCH;
    delta_bwd_kernel<bf16><<<(unsigned)B, PT, smem, st>>>(
        (int)T, (int)h, (const bf16*)k, (const bf16*)v, (const bf16*)beta, (const bf16*)recon, g,
        ckpt, (bf16*)dk, (bf16*)dv, (bf16*)dbeta);
  } else {
    set_error("permanent_delta_bwd: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("permanent_delta_bwd");
}

extern "C" int dabsn_local_field_gather(int dtype, int64_t B, int64_t C, int64_t N, int64_t K,
                                        int64_t D, const void* x, const int64_t* patch,
                                        void* out, void* stream) {
  if (B < 0 || C <= 0 || N <= 0 || K <= 0 || D <= 0) {
    set_error("local_field_gather: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  const long long total = (long long)B * N * K * D;
  if (total == 0) return DABSN_OK;
  const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 16);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32)
    field_gather_kernel<float><<<grid, 256, 0, st>>>(total, (int)C, (int)N, (int)K, (int)D,
                                                      (const float*)x, patch, (float*)out);
  else if (dtype == DABSN_BF16)
    field_gather_kernel<bf16><<<grid, 256, 0, st>>>(total, (int)C, (int)N, (int)K, (int)D,
                                                     (const bf16*)x, patch, (bf16*)out);
  else {
    set_error("local_field_gather: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("local_field_gather");
}

extern "C" int dabsn_local_field_scatter(int dtype, int64_t B, int64_t C, int64_t N, int64_t K,
                                         int64_t D, const void* gout, const int64_t* order,
                                         const int64_t* offsets, void* gx, void* stream) {
  if (B < 0 || C <= 0 || N <= 0 || K <= 0 || D <= 0) {
    set_error("local_field_scatter: bad sizes");
    return DABSN_ERR_SHAPE;
  }
  const long long total = (long long)B * C * D;
  if (total == 0) return DABSN_OK;
  const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 16);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == DABSN_F32)
    field_scatter_kernel<float><<<grid, 256, 0, st>>>(total, (int)C, (int)N, (int)K, (int)D,
                                                       (const float*)gout, order, offsets,
                                                       (float*)gx);
  else if (dtype == DABSN_BF16)
    field_scatter_kernel<bf16><<<grid, 256, 0, st>>>(total, (int)C, (int)N, (int)K, (int)D,
                                                      (const bf16*)gout, order, offsets,
                                                      (bf16*)gx);
  else {
    set_error("local_field_scatter: dtype code %d", dtype);
    return DABSN_ERR_DTYPE;
  }
  return launch_status("local_field_scatter");
}
