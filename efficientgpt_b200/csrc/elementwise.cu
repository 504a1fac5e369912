// Row-wise kernels of the decode path: per-row int8 quantiser, RMSNorm, LayerNorm (nanoGPT), embedding
// gather and row argmax. All are HBM/L2-bound single-pass kernels: one CTA per row, coalesced loads,
// fixed-order block reductions (the RMSNorm here produces the same bits as the GEMV's fused prologue).
#include "common.cuh"
#include "internal.h"

namespace egpt {

constexpr int kRowThreads = 256;

// s[n] = max(absmax(w[n]) / 127, 1e-12); q = clamp(rint(w / s), -127, 127)   (reference quantize_weight)
// The reference quantises on the GPU, where PyTorch evaluates `tensor / 127.0` (a CPU scalar divisor) as
// tensor * fl32(1 / 127); that product is reproduced here, so q and s are bit-identical to the reference's.
// `w / s` (tensor / tensor) is a true IEEE division in PyTorch and here.
__global__ void __launch_bounds__(kRowThreads) quantize_rows_kernel(int8_t *q, void *scale, int scale_bf16,
                                                                     const void *w, int w_bf16, int64_t k) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float amax = 0.f;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = w_bf16 ? bf16_bits_to_f32(((const uint16_t *)w)[row * k + i]) : ((const float *)w)[row * k + i];
    amax = fmaxf(amax, fabsf(v));
  }
  amax = warp_max(amax);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float s = fmaxf(red[0] * (1.0f / 127.0f), 1e-12f);
  if (threadIdx.x == 0) {
    if (scale_bf16)
      ((uint16_t *)scale)[row] = f32_to_bf16_bits(s);
    else
      ((float *)scale)[row] = s;
  }
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = w_bf16 ? bf16_bits_to_f32(((const uint16_t *)w)[row * k + i]) : ((const float *)w)[row * k + i];
    const float r = fminf(fmaxf(rintf(v / s), -127.f), 127.f);
    q[row * k + i] = (int8_t)(int)r;
  }
}

// y = w * bf16(x * rsqrt(mean(x^2) + eps)), bf16 in/out (HF Qwen3RMSNorm)
__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(uint16_t *out, const uint16_t *x, const uint16_t *w,
                                                               int64_t dim, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const uint16_t *xr = x + row * dim;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = bf16_bits_to_f32(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)dim + eps);
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = bf16_bits_to_f32(xr[i]);
    out[row * dim + i] = f32_to_bf16_bits(round_bf16(v * inv) * bf16_bits_to_f32(w[i]));
  }
}

// nanoGPT LayerNorm, fp32: two-pass mean / biased variance.
__global__ void __launch_bounds__(kRowThreads) layernorm_f32_kernel(float *out, const float *x, const float *w,
                                                                     const float *b, int64_t dim, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const float *xr = x + row * dim;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s, red) / (float)dim;
  float v = 0.f;
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    const float d = xr[i] - mean;
    v = fmaf(d, d, v);
  }
  const float var = block_sum(v, red) / (float)dim;
  const float inv = rsqrtf(var + eps);
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    float y = (xr[i] - mean) * inv * w[i];
    if (b) y += b[i];
    out[row * dim + i] = y;
  }
}

__global__ void embed_kernel(void *out, const int64_t *ids, const void *table, const void *pos_table, int64_t pos0,
                             const int64_t *position, int64_t vocab, int64_t dim, int bf16) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return;
  }
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    if (bf16) {
      ((uint16_t *)out)[row * dim + i] = ((const uint16_t *)table)[id * dim + i];
    } else {
      float v = ((const float *)table)[id * dim + i];
      if (pos_table) v += ((const float *)pos_table)[((position ? *position : 0) + pos0 + row) * dim + i];
      ((float *)out)[row * dim + i] = v;
    }
  }
}

__global__ void __launch_bounds__(kRowThreads) argmax_rows_kernel(int64_t *out, const void *logits, int64_t n,
                                                                   int64_t ld, int bf16) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16 ? bf16_bits_to_f32(((const uint16_t *)logits)[row * ld + i]) : ((const float *)logits)[row * ld + i];
    if (argmax_better(v, (int)i, bv, bi)) {
      bv = v;
      bi = (int)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (argmax_better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    out[row] = bi;
  }
}

}  // namespace egpt

using namespace egpt;

// out[r, i] = bf16(bf16(silu(g)) * u) with g = gu[r, i], u = gu[r, inter + i]: the HF MLP's act_fn(gate) * up in
// eager bf16 (SiLU evaluated in fp32 and rounded, the product rounded), two columns per thread.
__global__ void silu_mul_kernel(uint16_t *out, int64_t ldo, const uint16_t *gu, int64_t ldg, int64_t rows,
                                int64_t inter) {
  const int64_t half = inter / 2, pairs = rows * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / half, c = 2 * (i - r * half);
    const uint32_t g2 = *(const uint32_t *)(gu + r * ldg + c), u2 = *(const uint32_t *)(gu + r * ldg + inter + c);
    const float g0 = bf16_lo(g2), g1 = bf16_hi(g2);
    const float a0 = round_bf16(g0 / (1.0f + expf(-g0))) * bf16_lo(u2);
    const float a1 = round_bf16(g1 / (1.0f + expf(-g1))) * bf16_hi(u2);
    *(uint32_t *)(out + r * ldo + c) = (uint32_t)f32_to_bf16_bits(a0) | ((uint32_t)f32_to_bf16_bits(a1) << 16);
  }
}

extern "C" int egpt_quantize_rows(int8_t *q, void *scale, int scale_dtype, const void *w, int w_dtype, int64_t n,
                                  int64_t k, void *stream) {
  clear_error();
  if (!q || !scale || !w) return set_error(EGPT_ERR_ARG, "quantize_rows: null pointer");
  if (n < 1 || k < 1 || n > 0x7fffffff) return set_error(EGPT_ERR_SHAPE, "quantize_rows: bad shape");
  if ((scale_dtype != EGPT_F32 && scale_dtype != EGPT_BF16) || (w_dtype != EGPT_F32 && w_dtype != EGPT_BF16))
    return set_error(EGPT_ERR_DTYPE, "quantize_rows: dtype");
  return check_launch(launch_kernel((const void *)quantize_rows_kernel, dim3((unsigned)n), dim3(kRowThreads), 0,
                                    (cudaStream_t)stream, false, q, scale, (int)(scale_dtype == EGPT_BF16), w,
                                    (int)(w_dtype == EGPT_BF16), k),
                      "quantize_rows_kernel");
}

extern "C" int egpt_rmsnorm(void *out, const void *x, const void *w, int64_t rows, int64_t dim, float eps, void *stream) {
  clear_error();
  if (!out || !x || !w) return set_error(EGPT_ERR_ARG, "rmsnorm: null pointer");
  if (rows < 1 || dim < 1 || rows > 0x7fffffff) return set_error(EGPT_ERR_SHAPE, "rmsnorm: bad shape");
  return check_launch(launch_kernel((const void *)rmsnorm_kernel, dim3((unsigned)rows), dim3(kRowThreads), 0,
                                    (cudaStream_t)stream, false, (uint16_t *)out, (const uint16_t *)x,
                                    (const uint16_t *)w, dim, eps),
                      "rmsnorm_kernel");
}

extern "C" int egpt_layernorm_f32(float *out, const float *x, const float *w, const float *b, int64_t rows,
                                  int64_t dim, float eps, void *stream) {
  clear_error();
  if (!out || !x || !w) return set_error(EGPT_ERR_ARG, "layernorm: null pointer");
  if (rows < 1 || dim < 1 || rows > 0x7fffffff) return set_error(EGPT_ERR_SHAPE, "layernorm: bad shape");
  return check_launch(launch_kernel((const void *)layernorm_f32_kernel, dim3((unsigned)rows), dim3(kRowThreads), 0,
                                    (cudaStream_t)stream, false, out, x, w, b, dim, eps),
                      "layernorm_f32_kernel");
}

extern "C" int egpt_embed(void *out, const int64_t *ids, int64_t rows, const void *table, const void *pos_table,
                          int64_t pos0, const int64_t *position, int64_t vocab, int64_t dim, int dtype, void *stream) {
  clear_error();
  if (!out || !ids || !table) return set_error(EGPT_ERR_ARG, "embed: null pointer");
  if (rows < 1 || dim < 1 || vocab < 1 || rows > 0x7fffffff) return set_error(EGPT_ERR_SHAPE, "embed: bad shape");
  if (dtype != EGPT_BF16 && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "embed: dtype");
  if (pos_table && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "embed: positional table is fp32 only");
  return check_launch(launch_kernel((const void *)embed_kernel, dim3((unsigned)rows), dim3(256), 0, (cudaStream_t)stream,
                                    false, out, ids, table, pos_table, pos0, position, vocab, dim, (int)(dtype == EGPT_BF16)),
                      "embed_kernel");
}

extern "C" int egpt_argmax_rows(int64_t *out, const void *logits, int64_t rows, int64_t n, int64_t ld, int dtype,
                                void *stream) {
  clear_error();
  if (!out || !logits) return set_error(EGPT_ERR_ARG, "argmax_rows: null pointer");
  if (rows < 1 || n < 1 || ld < n || rows > 0x7fffffff || n > 0x7fffffff) return set_error(EGPT_ERR_SHAPE, "argmax_rows: bad shape");
  if (dtype != EGPT_BF16 && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "argmax_rows: dtype");
  return check_launch(launch_kernel((const void *)argmax_rows_kernel, dim3((unsigned)rows), dim3(kRowThreads), 0,
                                    (cudaStream_t)stream, false, out, logits, n, ld, (int)(dtype == EGPT_BF16)),
                      "argmax_rows_kernel");
}

extern "C" int egpt_silu_mul(void *out, int64_t ldo, const void *gu, int64_t ldg, int64_t rows, int64_t inter,
                             void *stream) {
  clear_error();
  if (!out || !gu) return set_error(EGPT_ERR_ARG, "silu_mul: null pointer");
  if (rows < 1 || inter < 2 || inter % 2 || ldo < inter || ldg < 2 * inter)
    return set_error(EGPT_ERR_SHAPE, "silu_mul: bad shape (inter even, ldo >= inter, ldg >= 2 inter)");
  if ((uintptr_t)out % 4 || (uintptr_t)gu % 4 || ldo % 2 || ldg % 2)
    return set_error(EGPT_ERR_ALIGN, "silu_mul: 4-byte aligned rows");
  const int64_t pairs = rows * (inter / 2);
  const unsigned grid = (unsigned)std::min<int64_t>((pairs + kRowThreads - 1) / kRowThreads, (int64_t)num_sms() * 16);
  silu_mul_kernel<<<grid, kRowThreads, 0, (cudaStream_t)stream>>>((uint16_t *)out, ldo, (const uint16_t *)gu, ldg,
                                                                  rows, inter);
  return check_launch(cudaGetLastError(), "silu_mul_kernel");
}
