// Small shared-memory matrix-vector products used inside the persistent scans.
//
//   out[b][o] = sum_k X[b][k] * W[o][k]      b < NB, o < NO, k < Kp
//
// X is FP32 (rows padded with zeros to a multiple of TB), W is FP32 or BF16
// (rows padded to a multiple of TO), Kp is a multiple of 128 and both are
// zero-padded in k.  A warp owns a TB x TO output tile; its lanes split k in
// float4 strips (lane*4 + 128*j, conflict-free) and the partial sums are
// combined with a transpose-style shuffle reduction.
#pragma once

#include "common.cuh"

namespace dabsn {

template <typename WT>
__device__ __forceinline__ float4 load4(const WT* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
  __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
  float2 a = __bfloat1622float2(lo);
  float2 b = __bfloat1622float2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

// Reduce N per-lane values across the warp (N a power of two <= 32).  Lane l
// ends up holding the warp-wide sum of value index l / (32 / N).
template <int N>
__device__ __forceinline__ float warp_reduce_many(float (&v)[N]) {
  const int lane = threadIdx.x & 31;
  // Halving exchange: at each level a lane keeps half of its values and sends
  // the other half to its partner, so the shuffle count is N-1 + log2(32/N).
#pragma unroll
  for (int width = N; width > 1; width >>= 1) {
    const int half = width >> 1;
    const int offset = half * (32 / N);  // partner distance
    const bool upper = (lane & offset) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      float send = upper ? v[i] : v[i + half];
      float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, offset);
    }
  }
  float s = v[0];
#pragma unroll
  for (int o = (32 / N) / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

template <typename WT, int TB, int TO>
__device__ __forceinline__ void matvec_tiles(const float* __restrict__ X, int ldx,
                                             const WT* __restrict__ W, int ldw, int NB, int NO,
                                             int Kp, float* __restrict__ out, int ldo, int warp,
                                             int nwarps) {
  const int lane = threadIdx.x & 31;
  const int ngb = (NB + TB - 1) / TB;
  const int ngo = (NO + TO - 1) / TO;
  constexpr int NV = TB * TO;
  for (int g = warp; g < ngb * ngo; g += nwarps) {
    const int b0 = (g / ngo) * TB;
    const int o0 = (g % ngo) * TO;
    float acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = 0.0f;
    for (int k = lane * 4; k < Kp; k += 128) {
      float4 xv[TB];
#pragma unroll
      for (int tb = 0; tb < TB; ++tb) xv[tb] = *reinterpret_cast<const float4*>(X + (b0 + tb) * ldx + k);
#pragma unroll
      for (int to = 0; to < TO; ++to) {
        float4 wv = load4<WT>(W + (size_t)(o0 + to) * ldw + k);
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) {
          float a = acc[tb * TO + to];
          a = fmaf(xv[tb].x, wv.x, a);
          a = fmaf(xv[tb].y, wv.y, a);
          a = fmaf(xv[tb].z, wv.z, a);
          a = fmaf(xv[tb].w, wv.w, a);
          acc[tb * TO + to] = a;
        }
      }
    }
    // After the reduction lane l holds the total of value l / (32 / NV).
    float s = warp_reduce_many<NV>(acc);
    if ((lane % (32 / NV)) == 0) {
      const int idx = lane / (32 / NV);
      const int tb = idx / TO, to = idx % TO;
      const int b = b0 + tb, o = o0 + to;
      if (b < NB && o < NO) out[b * ldo + o] = s;
    }
  }
}

}  // namespace dabsn

namespace dabsn {

// ---------------------------------------------------------------------------
// Register-resident products for the persistent scans.
//
// Thread t of the CTA owns output row o = t / L and the columns
// k = lk*4 + j*4L + c (lk = t % L, j < WR/4, c < 4) of the weight matrix, held
// in registers for the whole scan.  A step reads only the input vector from
// shared memory: the L lanes of a group read consecutive float4s and every
// group reads the same ones (broadcast), so the read is conflict-free, and the
// L partial sums are combined with log2(L) shuffles.  L is a power of two,
// L <= 32, so a group never straddles a warp.
// ---------------------------------------------------------------------------
template <int WR>
__device__ __forceinline__ float reg_dot(const float (&w)[WR], const float* __restrict__ x, int lk,
                                         int L) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int j = 0; j < WR / 4; ++j) {
    const float4 xv = *reinterpret_cast<const float4*>(x + lk * 4 + j * 4 * L);
    a0 = fmaf(w[4 * j + 0], xv.x, a0);
    a1 = fmaf(w[4 * j + 1], xv.y, a1);
    a2 = fmaf(w[4 * j + 2], xv.z, a2);
    a3 = fmaf(w[4 * j + 3], xv.w, a3);
  }
  float v = (a0 + a1) + (a2 + a3);
  for (int off = L >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

}  // namespace dabsn
