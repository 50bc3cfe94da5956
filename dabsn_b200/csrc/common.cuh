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

// torch.nn.functional.hardsigmoid: min(max(x + 3, 0), 6) / 6, with the
// division taken as a multiplication by 1/6 (within one ulp of it; an IEEE
// division would sit on the scan's serial per-step chain).
__device__ __forceinline__ float hardsigmoidf_(float x) {
  return fminf(fmaxf(x + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);
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

// ---------------------------------------------------------------------------
// mbarrier primitives and asynchronous distributed-shared-memory stores.
// ---------------------------------------------------------------------------
namespace dabsn {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive once on a local mbarrier and raise its expected transaction bytes.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cta(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity`: gives up after `limit` polls, records `code`
// in *status (when given) and returns false, so a lost signal ends the kernel
// with an error status instead of hanging the device.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status,
                                                  int code, uint32_t limit = (1u << 25)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
  if (status) atomicExch(status, code);
  return false;
}

// Asynchronous 4-byte store into a cluster CTA's shared memory that signals
// 4 transaction bytes on that CTA's mbarrier when it lands.
__device__ __forceinline__ void st_async_f32(uint32_t remote_addr, float v,
                                             uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
          remote_addr),
      "r"(__float_as_uint(v)), "r"(remote_bar)
      : "memory");
}

int* device_status();  // per-device status word of the bounded waits (runtime.cu)
const void* current_context();  // identity of the current CUDA context (runtime.cu)

}  // namespace dabsn

namespace dabsn {
// 4-byte asynchronous global -> shared copy (no register staging).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
}  // namespace dabsn

namespace dabsn {
// Low-latency transcendentals for the serial per-step chains of the scans.
// tanh uses the identity tanh(x) = sign(x) * (1 - 2 / (exp(2|x|) + 1)) on top
// of the hardware exponential (__expf) and fast division (__fdividef); its
// absolute error is a few 1e-7, which the parity tests bound against the
// float64 oracle.  exp(x) is __expf (relative error ~1e-7 for |x| <= 1, the
// range the scans use it on).
__device__ __forceinline__ float tanh_fast(float x) {
  const float e = __expf(2.0f * fabsf(x));
  const float r = 1.0f - __fdividef(2.0f, e + 1.0f);
  return copysignf(r, x);
}
__device__ __forceinline__ float exp_fast(float x) { return __expf(x); }
}  // namespace dabsn
