// Mean cross-entropy over materialised logits, forward and reverse, in one
// pass over the logits each (HBM-bound).
//
// Reference: src/dabsn/runtime/loss.py:187-231
// (`chunked_cross_entropy_from_logits`, the default loss of
// runtime/api.py:22-31 `train_step`): logits are upcast to FP32 (in chunks,
// or in one piece when rows * V fits the element budget), loss = mean over
// rows whose target is not ignore_index of logsumexp(row) - row[target]; its
// gradient is scale (softmax(row) - onehot(target)), cast back to the logits'
// dtype.
//
// Forward: one CTA per row at a time (grid-stride), 16-byte vector loads, an
// online maximum / sum of exponentials per thread merged across the CTA;
// writes the row's log-sum-exp and target logit (FP32).  Reverse: the same
// sweep writing scale (exp(x - lse) - onehot) in the logits' dtype.  The
// logits are never widened in memory.  A target outside [0, V) that is not
// ignore_index makes the row's target logit NaN and records status code 7.
#include "../../include/dabsn_b200.h"
#include "common.cuh"

namespace dabsn {
namespace {

typedef __nv_bfloat16 bf16;
constexpr int CE_THREADS = 256;
constexpr int CE_STATUS_BAD_TARGET = 7;

template <typename T>
struct Vec;  // 16 bytes of T
template <>
struct Vec<bf16> {
  static constexpr int N = 8;
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[Vec<T>::N]);
template <>
__device__ __forceinline__ void load_vec<bf16>(const bf16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec<float>(const float* p, float (&v)[4]) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = f.x;
  v[1] = f.y;
  v[2] = f.z;
  v[3] = f.w;
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[Vec<T>::N]);
template <>
__device__ __forceinline__ void store_vec<bf16>(bf16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store_vec<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

// (m, s): running maximum and sum of exp(x - m); merge of two partial pairs.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else if (m2 > -INFINITY) {
    s += s2 * __expf(m2 - m);
  }
}

// Rows of 16-byte-aligned vectors: one warp per row (eight rows per CTA at a
// time, grid-stride over rows), each lane sweeping the row in 16-byte words;
// the row's (maximum, sum) is merged with shuffles only, so no CTA barrier
// and no serial tail sit between rows.  The target logit is loaded before
// the sweep.
template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_logits_fwd_warp_kernel(
    long long rows, int V, long long ld, const T* __restrict__ logits,
    const int64_t* __restrict__ targets, long long ignore_index, float* __restrict__ lse,
    float* __restrict__ tgt_logit, int* status) {
  constexpr int VW = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const long long nwarps = (long long)gridDim.x * (CE_THREADS / 32);
  const int nv = V / VW;
  for (long long r = (long long)blockIdx.x * (CE_THREADS / 32) + (threadIdx.x >> 5); r < rows;
       r += nwarps) {
    const T* row = logits + (size_t)r * ld;
    long long t = 0;
    float tl = 0.f;
    if (lane == 0) {
      t = targets[r];
      if (t != ignore_index && t >= 0 && t < V) tl = to_f<T>(row[t]);
    }
    float m = -INFINITY, s = 0.f;
#pragma unroll 4
    for (int i = lane; i < nv; i += 32) {
      float v[VW];
      load_vec<T>(row + (size_t)i * VW, v);
      float vm = v[0];
#pragma unroll
      for (int k = 1; k < VW; ++k) vm = fmaxf(vm, v[k]);
      float vs = 0.f;
#pragma unroll
      for (int k = 0; k < VW; ++k) vs += __expf(v[k] - vm);
      lse_merge(m, s, vm, vs);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      lse[r] = m + __logf(s);
      if (t != ignore_index && (t < 0 || t >= V)) {
        tl = __int_as_float(0x7fc00000);  // NaN: the loss shows the bad target
        if (status) atomicExch(status, CE_STATUS_BAD_TARGET);
      }
      tgt_logit[r] = tl;
    }
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(CE_THREADS) ce_logits_fwd_kernel(
    long long rows, int V, long long ld, const T* __restrict__ logits,
    const int64_t* __restrict__ targets, long long ignore_index, float* __restrict__ lse,
    float* __restrict__ tgt_logit, int* status) {
  __shared__ float sm[CE_THREADS / 32], ss[CE_THREADS / 32];
  constexpr int VW = Vec<T>::N;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = logits + (size_t)r * ld;
    float m = -INFINITY, s = 0.f;
    if (VEC) {
      const int nv = V / VW;
#pragma unroll 4
      for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
        float v[VW];
        load_vec<T>(row + (size_t)i * VW, v);
        float vm = v[0];
#pragma unroll
        for (int k = 1; k < VW; ++k) vm = fmaxf(vm, v[k]);
        float vs = 0.f;
#pragma unroll
        for (int k = 0; k < VW; ++k) vs += __expf(v[k] - vm);
        lse_merge(m, s, vm, vs);
      }
    } else {
      for (int j = threadIdx.x; j < V; j += CE_THREADS) lse_merge(m, s, to_f<T>(row[j]), 1.f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      sm[warp] = m;
      ss[warp] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float M = sm[0], S = ss[0];
      for (int w = 1; w < CE_THREADS / 32; ++w) lse_merge(M, S, sm[w], ss[w]);
      lse[r] = M + __logf(S);
      const long long t = targets[r];
      float tl = 0.f;
      if (t != ignore_index) {
        if (t >= 0 && t < V) {
          tl = to_f<T>(row[t]);
        } else {
          tl = __int_as_float(0x7fc00000);  // NaN: the loss shows the bad target
          if (status) atomicExch(status, CE_STATUS_BAD_TARGET);
        }
      }
      tgt_logit[r] = tl;
    }
    __syncthreads();
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(CE_THREADS) ce_logits_bwd_kernel(
    long long rows, int V, long long ld, const T* __restrict__ logits,
    const int64_t* __restrict__ targets, long long ignore_index, const float* __restrict__ lse,
    const float* __restrict__ scale, T* __restrict__ dlogits, long long ldd) {
  constexpr int VW = Vec<T>::N;
  const float sc = *scale;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = logits + (size_t)r * ld;
    T* drow = dlogits + (size_t)r * ldd;
    const long long t = targets[r];
    const bool valid = t != ignore_index;
    const float L = lse[r];
    const float rs = valid ? sc : 0.f;
    if (VEC) {
      const int nv = V / VW;
#pragma unroll 4
      for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
        float v[VW];
        load_vec<T>(row + (size_t)i * VW, v);
#pragma unroll
        for (int k = 0; k < VW; ++k) {
          const long long j = (long long)i * VW + k;
          v[k] = rs * (__expf(v[k] - L) - (j == t ? 1.f : 0.f));
        }
        store_vec<T>(drow + (size_t)i * VW, v);
      }
    } else {
      for (int j = threadIdx.x; j < V; j += CE_THREADS) {
        const float x = to_f<T>(row[j]);
        drow[j] = from_f<T>(rs * (__expf(x - L) - (j == t ? 1.f : 0.f)));
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned ce_grid(long long rows) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, current_device());
  const long long g = (long long)sms * 8;  // eight 256-thread CTAs per SM
  return (unsigned)(rows < g ? rows : g);
}

}  // namespace
}  // namespace dabsn

using namespace dabsn;

extern "C" int dabsn_ce_logits_fwd(int dtype, int64_t rows, int64_t V, int64_t ld,
                                   const void* logits, const int64_t* targets,
                                   int64_t ignore_index, float* lse, float* tgt_logit,
                                   void* stream) {
  if (rows < 0 || V <= 0 || V > INT32_MAX || ld < V) {
    set_error("ce_logits_fwd: unsupported sizes rows=%lld V=%lld ld=%lld", (long long)rows,
              (long long)V, (long long)ld);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (dtype != DABSN_F32 && dtype != DABSN_BF16) {
    set_error("ce_logits_fwd: logits must be FP32 or BF16");
    return DABSN_ERR_DTYPE;
  }
  if (rows == 0) return DABSN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = ce_grid(rows);
  int* status = device_status();
  if (dtype == DABSN_BF16) {
    const bool vec = V % 8 == 0 && ld % 8 == 0 && aligned16(logits);
    if (vec)
      ce_logits_fwd_warp_kernel<bf16><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const bf16*)logits, targets, ignore_index, lse, tgt_logit, status);
    else
      ce_logits_fwd_kernel<bf16, false><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const bf16*)logits, targets, ignore_index, lse, tgt_logit, status);
  } else {
    const bool vec = V % 4 == 0 && ld % 4 == 0 && aligned16(logits);
    if (vec)
      ce_logits_fwd_warp_kernel<float><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const float*)logits, targets, ignore_index, lse, tgt_logit, status);
    else
      ce_logits_fwd_kernel<float, false><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const float*)logits, targets, ignore_index, lse, tgt_logit, status);
  }
  return launch_status("ce_logits_fwd");
}

extern "C" int dabsn_ce_logits_bwd(int dtype, int64_t rows, int64_t V, int64_t ld,
                                   const void* logits, const int64_t* targets,
                                   int64_t ignore_index, const float* lse, const float* scale,
                                   void* dlogits, void* stream) {
  if (rows < 0 || V <= 0 || V > INT32_MAX || ld < V) {
    set_error("ce_logits_bwd: unsupported sizes rows=%lld V=%lld ld=%lld", (long long)rows,
              (long long)V, (long long)ld);
    return DABSN_ERR_UNSUPPORTED;
  }
  if (dtype != DABSN_F32 && dtype != DABSN_BF16) {
    set_error("ce_logits_bwd: logits must be FP32 or BF16");
    return DABSN_ERR_DTYPE;
  }
  if (rows == 0) return DABSN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = ce_grid(rows);
  // dlogits is a fresh contiguous [rows][V] tensor
  if (dtype == DABSN_BF16) {
    const bool vec = V % 8 == 0 && ld % 8 == 0 && aligned16(logits) && aligned16(dlogits);
    if (vec)
      ce_logits_bwd_kernel<bf16, true><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const bf16*)logits, targets, ignore_index, lse, scale,
          (bf16*)dlogits, V);
    else
      ce_logits_bwd_kernel<bf16, false><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const bf16*)logits, targets, ignore_index, lse, scale,
          (bf16*)dlogits, V);
  } else {
    const bool vec = V % 4 == 0 && ld % 4 == 0 && aligned16(logits) && aligned16(dlogits);
    if (vec)
      ce_logits_bwd_kernel<float, true><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const float*)logits, targets, ignore_index, lse, scale,
          (float*)dlogits, V);
    else
      ce_logits_bwd_kernel<float, false><<<grid, CE_THREADS, 0, st>>>(
          rows, (int)V, ld, (const float*)logits, targets, ignore_index, lse, scale,
          (float*)dlogits, V);
  }
  return launch_status("ce_logits_bwd");
}
