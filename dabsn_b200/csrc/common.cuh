// Shared device helpers for the DABSN sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dabsn {

// ---------------------------------------------------------------------------
// Activation element types.  Tapes and activations are either FP32 or BF16;
// all recurrent state and every reduction is FP32.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round an FP32 value through the activation type (identity for FP32).
template <typename T>
__device__ __forceinline__ float round_act(float v) { return to_f<T>(from_f<T>(v)); }

// ---------------------------------------------------------------------------
// Scalar math with PyTorch's definitions.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// torch.nn.functional.hardsigmoid: min(max(x + 3, 0), 6) / 6.
__device__ __forceinline__ float hardsigmoidf_(float x) {
  return fminf(fmaxf(x + 3.0f, 0.0f), 6.0f) / 6.0f;
}

__device__ __forceinline__ float clamp01(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }

// torch.sign: -1, 0 or +1.
__device__ __forceinline__ float signf_(float x) { return (float)((x > 0.0f) - (x < 0.0f)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Thread-block-cluster primitives (distributed shared memory), inline PTX.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Map a local shared-memory address to the same offset in CTA `rank` of this
// cluster (a shared::cluster address).
__device__ __forceinline__ uint32_t map_shared_rank(const void* smem_ptr, uint32_t rank) {
  uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(smem_ptr));
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Full cluster barrier: every thread of every CTA in the cluster arrives
// (release) and waits (acquire); orders shared::cluster stores before it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace dabsn

// Status codes returned by every C-ABI entry point.
#define DABSN_OK 0
#define DABSN_ERR_SHAPE 1
#define DABSN_ERR_DTYPE 2
#define DABSN_ERR_LAUNCH 3
#define DABSN_ERR_UNSUPPORTED 4
#define DABSN_ERR_TIMEOUT 5

// ---------------------------------------------------------------------------
// Host-side helpers shared by the C-ABI launchers (defined in runtime.cu).
// ---------------------------------------------------------------------------
namespace dabsn {
void set_error(const char* fmt, ...);
// Cache of per-device kernel attribute set-up, keyed by kernel pointer.
bool kernel_prepared(const void* kernel, int smem_bytes);
int current_device();
int launch_status(const char* what);
}  // namespace dabsn
