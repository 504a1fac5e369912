// Shared device helpers for the batch-1 int8 decode kernels (sm_100a only).
//
// Everything here is hand-written PTX or plain CUDA: bf16 rounding that matches PyTorch's eager casts
// (round-to-nearest-even), programmatic-dependent-launch controls, warp / block reductions, and the device error
// word that bounded waits set instead of hanging.
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

// ------------------------------------------------------------------------------------------------ PDL
// Programmatic dependent launch: launch_dependents lets the next kernel in the stream get scheduled;
// wait blocks until the previous kernel has completed and its writes are visible. Both are no-ops when
// the kernel was not launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------ shared memory
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

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
