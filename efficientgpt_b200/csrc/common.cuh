// Shared device helpers for the batch-1 int8 decode kernels (sm_100a only).
//
// Everything here is hand-written PTX or plain CUDA: bf16 rounding that matches PyTorch's eager casts
// (round-to-nearest-even), 1-D bulk copies (cp.async.bulk, no multicast) completing on an mbarrier,
// programmatic-dependent-launch controls, and bounded waits that record an error instead of hanging.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/egpt_b200.h"

#ifndef __CUDA_ARCH__
#define EGPT_HOST_ONLY 1
#endif

namespace egpt {

// ------------------------------------------------------------------------------------------------ errors
// Device-side error word shared by every kernel of the library. A kernel that gives up on a wait stores
// EGPT_ERR_TIMEOUT here (first writer wins) and returns; the host reads it with egpt_device_error().
// Defined here (header guarded): the library is one translation unit, see egpt_b200.cu.
__device__ int g_device_error = 0;

__device__ __forceinline__ void set_device_error(int code) { atomicCAS(&g_device_error, 0, code); }
__device__ __forceinline__ bool device_error_set() {
  return *((volatile int *)&g_device_error) != 0;
}

// Wall-clock bound for any spin: 200 ms of %globaltimer (ns).
constexpr uint64_t kWaitLimitNs = 200ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------ bf16
// Conversions with PyTorch's semantics: float -> bf16 is round-to-nearest-even (NaN kept quiet).
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ------------------------------------------------------------------------------------------------ int8
// Exact int8 -> fp32: flip the sign bit so the byte is q + 128, place it in the low mantissa byte of
// 2^23 (0x4B0000uu == 8388608 + u) and subtract 8388608 + 128. One PRMT and one FADD per value.
__device__ __forceinline__ float i8_to_f32(uint32_t biased_word, int byte_idx) {
  const uint32_t sel = 0x7440u | (uint32_t)byte_idx;
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, sel)) - 8388736.0f;
}

// ------------------------------------------------------------------------------------------------ PDL
// Programmatic dependent launch: launch_dependents lets the next kernel in the stream get scheduled;
// wait blocks until the previous kernel has completed and its writes are visible. Both are no-ops when
// the kernel was not launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------ mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Non-blocking probe of phase `parity`; returns true once that phase has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: spins until the phase completes, the library error word is set, or kWaitLimitNs passes.
// Returns false (after recording EGPT_ERR_TIMEOUT) when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(EGPT_ERR_TIMEOUT);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared (this CTA's memory, no multicast); completes `bytes` of tx on `bar`.
// Both addresses must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same copy with an L2 evict-first hint: streamed weights are read once per token and should not push
// the activations, KV cache and RoPE tables out of L2.
__device__ __forceinline__ void bulk_g2s_stream(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------------------------------------ reductions
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

// Block-wide sum in a fixed order (per-warp butterfly, then warp 0 over the warp partials), so every CTA
// that reduces the same data gets the same float. `red` needs blockDim.x/32 floats.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    t = lane < nw ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  t = red[0];
  __syncthreads();
  return t;
}

// (value, index) argmax merge with PyTorch's rule: larger value wins, equal values keep the lower index,
// NaN counts as the maximum.
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) {
    if (vn && bn) return i < bi;
    return vn;
  }
  return v > bv || (v == bv && i < bi);
}

}  // namespace egpt
