// Int8 weight-only GEMV / small-M GEMM for B200 (sm_100a), CUDA cores only.
//
// Reference behaviour (BagelsFun/efficientgpt research/realmodel/int8_linear.py:26-98): out[m, n] =
// bf16(s[n] * sum_k bf16(x[m,k]) * q[n,k]) with fp32 accumulation; rows > 16 take the reference's prefill
// branch, bf16(bf16(x @ bf16(q).T) * s) (EGPT_FLAG_DOUBLE_ROUND reproduces that double rounding).
//
// B200 design. Batch-1 decode is a pure weight stream (N*K int8 bytes read once per token). The kernel keeps
// as many bytes in flight per SM as it can and spends as few issue slots per weight byte as possible:
//   * a warp task is 2 logical rows x the full K; a lane reads its 16-byte segments of both rows with
//     128-bit streaming loads (ld.global.nc, no L1 allocation), 4 segments per row per wave, so one wave
//     puts 8 x 16 B in flight per lane; up to 4 CTAs of 8 warps per SM keep ~128 KB in flight per SM;
//   * the first wave is loaded BEFORE griddepcontrol.wait: weights do not depend on the previous kernel, so
//     under programmatic dependent launch (PDL) they stream while the previous kernel finishes; the next
//     task's first wave is issued before each task's reduction and epilogue;
//   * int8 -> fp32 is exact: PRMT places q + 128 in the low mantissa byte of 2^23 and one packed f32x2 SUB
//     removes 2^23 + 128 from two values; the exact products accumulate with packed f32x2 FMA into even/odd
//     partial sums (~2.25 instructions per weight byte), then a fixed-order warp butterfly: every run and
//     every CTA gives the same bits;
//   * the activation rows are staged once per CTA in shared memory as fp32 in a [4][segments] float4 layout
//     (lane l reading segment l is bank-conflict free); RMSNorm and embedding-gather prologues are fused;
//   * epilogues (scale, bias, residual add, SiLU*up, GELU, lm_head argmax with a last-CTA reduction) run on
//     the reduced sums in lane 0.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace egpt {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kRows = 2;                    // logical rows per warp task
constexpr int kWave = 4;                    // 16-byte segments per lane per row per wave (2048 columns)
constexpr int kMaxMT = 8;                   // activation rows per launch (more are split by the host)
constexpr int kXsMaxBytes = 64 * 1024;      // fp32 activation staging limit

struct GemvParams {
  void *out;
  const void *x;
  int64_t m, ldx, ldo;
  const int8_t *w;
  const void *scale;
  int scale_bf16;
  int x_bf16;
  int64_t n, k;
  const void *bias;
  void *residual;
  const void *norm_w;
  float eps;
  const int64_t *token;
  unsigned flags;
  int epilogue;
  int segs;     // 16-byte segments per row (k / 16)
  int xs_smem;  // 1: activations staged in shared memory, 0: read from global memory in the loop
  // lm_head argmax
  int argmax;
  int64_t *tok_out;
  int64_t *position;
  void *logits;
  float *ws_val;
  int *ws_idx;
  unsigned *ws_counter;
};

__device__ __forceinline__ float load_scale(const GemvParams &p, int64_t n) {
  return p.scale_bf16 ? bf16_bits_to_f32(((const uint16_t *)p.scale)[n]) : ((const float *)p.scale)[n];
}
__device__ __forceinline__ float load_act(const void *ptr, int64_t i, int is_bf16) {
  return is_bf16 ? bf16_bits_to_f32(((const uint16_t *)ptr)[i]) : ((const float *)ptr)[i];
}
__device__ __forceinline__ void store_act(void *ptr, int64_t i, float v, int is_bf16) {
  if (is_bf16)
    ((uint16_t *)ptr)[i] = f32_to_bf16_bits(v);
  else
    ((float *)ptr)[i] = v;
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ float gelu_erf_f32(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }

// Physical weight row of logical row `lr`. With SiLU*up the weight is cat(gate, up) ([2I, K]) and the kernel
// walks logical rows interleaved (gate_0, up_0, gate_1, up_1, ...) so both halves of a pair meet in one group.
__device__ __forceinline__ int64_t phys_row(const GemvParams &p, int64_t lr) {
  if (p.epilogue != EGPT_EPI_SILU_MUL) return lr;
  return (lr & 1) ? (p.n >> 1) + (lr >> 1) : (lr >> 1);
}

// Scale + rounding of one accumulated row sum (bf16 path reproduces the reference's rounding points).
__device__ __forceinline__ float scaled_value(const GemvParams &p, int64_t n, float acc) {
  const float s = load_scale(p, n);
  if (!p.x_bf16) {
    float y = acc * s;
    if (p.bias) y += ((const float *)p.bias)[n];
    return y;
  }
  float y = (p.flags & EGPT_FLAG_DOUBLE_ROUND) ? round_bf16(round_bf16(acc) * s) : round_bf16(acc * s);
  if (p.bias) y = round_bf16(y + bf16_bits_to_f32(((const uint16_t *)p.bias)[n]));
  return y;
}

// Same rounding with the scale (and bias) already loaded.
__device__ __forceinline__ float apply_scale(const GemvParams &p, float acc, float s, float bias) {
  if (!p.x_bf16) return acc * s + (p.bias ? bias : 0.f);
  float y = (p.flags & EGPT_FLAG_DOUBLE_ROUND) ? round_bf16(round_bf16(acc) * s) : round_bf16(acc * s);
  if (p.bias) y = round_bf16(y + bias);
  return y;
}

// Epilogue for one (logical row, m); for SiLU*up `acc0` is the gate row (even logical row) and `acc1` its up row.
__device__ __forceinline__ void emit(const GemvParams &p, int64_t lr, int64_t m, float acc0, float acc1) {
  const int bf = p.x_bf16;
  switch (p.epilogue) {
    case EGPT_EPI_SILU_MUL: {
      const int64_t j = lr >> 1;
      const float g = scaled_value(p, j, acc0), u = scaled_value(p, (p.n >> 1) + j, acc1);
      const float out = bf ? round_bf16(round_bf16(silu_f32(g)) * u) : silu_f32(g) * u;
      store_act(p.out, m * p.ldo + j, out, bf);
      break;
    }
    case EGPT_EPI_RESIDUAL: {
      const float y = scaled_value(p, lr, acc0);
      const float r = load_act(p.residual, m * p.ldo + lr, bf);
      store_act(p.out, m * p.ldo + lr, bf ? round_bf16(r + y) : r + y, bf);
      break;
    }
    case EGPT_EPI_GELU:
      store_act(p.out, m * p.ldo + lr, gelu_erf_f32(scaled_value(p, lr, acc0)), bf);
      break;
    default:
      store_act(p.out, m * p.ldo + lr, scaled_value(p, lr, acc0), bf);
  }
}

// ---------------------------------------------------------------------------------------------- f32x2 math
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// acc2 += x[0..15] * q[0..15] (exact products; even/odd values accumulate in the two halves of acc2).
// x2[i] holds the fp32 pair (x[2i], x[2i+1]); wv holds 16 int8 weights.
__device__ __forceinline__ uint64_t dot16x2(const uint64_t (&x2)[8], const uint4 &wv, uint64_t acc2) {
  const uint64_t magic = 0x4B0000804B000080ull;  // (8388736.f, 8388736.f) = 2^23 + 128 in both halves
  const uint32_t w[4] = {wv.x ^ 0x80808080u, wv.y ^ 0x80808080u, wv.z ^ 0x80808080u, wv.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t qa = sub2(pack2(__uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7440)),
                                   __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7441))), magic);
    const uint64_t qb = sub2(pack2(__uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7442)),
                                   __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7443))), magic);
    acc2 = fma2(x2[2 * i], qa, acc2);
    acc2 = fma2(x2[2 * i + 1], qb, acc2);
  }
  return acc2;
}

// 16 activations x[m, 16*seg ..] as 8 fp32 pairs, from the shared-memory stage or from global memory.
__device__ __forceinline__ void load_x16(const GemvParams &p, const float4 *xs, int64_t m, int seg, uint64_t (&x2)[8]) {
  if (p.xs_smem) {
    const ulonglong2 *xb = (const ulonglong2 *)(xs + (size_t)(m * 4) * p.segs + seg);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const ulonglong2 v = xb[(size_t)g * p.segs];
      x2[2 * g] = v.x;
      x2[2 * g + 1] = v.y;
    }
  } else if (p.x_bf16) {
    const uint4 *src = (const uint4 *)((const uint16_t *)p.x + m * p.ldx + 16 * (int64_t)seg);
    const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
    const uint32_t u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) x2[i] = pack2(bf16_lo(u[i]), bf16_hi(u[i]));
  } else {
    const ulonglong2 *src = (const ulonglong2 *)((const float *)p.x + m * p.ldx + 16 * (int64_t)seg);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const ulonglong2 v = __ldg(src + i);
      x2[2 * i] = v.x;
      x2[2 * i + 1] = v.y;
    }
  }
}

__device__ __forceinline__ uint4 ldg_stream(const void *ptr) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr));
  return r;
}

// One warp task = kRows logical rows x the full K, streamed in waves of kWave 16-byte segments per lane.
template <int MT>
__device__ __forceinline__ void load_wave(const GemvParams &p, int64_t g, int wave, uint4 (&wv)[kRows][kWave]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int64_t row = g * kRows + r;
#pragma unroll
    for (int j = 0; j < kWave; ++j) {
      const int seg = (wave * kWave + j) * 32 + lane;
      wv[r][j] = (row < p.n && seg < p.segs) ? ldg_stream(p.w + phys_row(p, row) * p.k + (int64_t)seg * 16)
                                             : make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
    }
  }
}

template <int MT>
__global__ void __launch_bounds__(kGemvThreads, MT == 1 ? 3 : 2) gemv_i8_kernel(const GemvParams p) {
  extern __shared__ __align__(16) float4 xs[];  // MT * 4 * segs (when xs_smem)
  __shared__ float red[32];
  __shared__ float s_bv[kGemvWarps];
  __shared__ int s_bi[kGemvWarps];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * kGemvWarps + warp;
  const int64_t nw = (int64_t)gridDim.x * kGemvWarps;
  const int64_t ngroups = (p.n + kRows - 1) / kRows;
  const int nwaves = (p.segs + 32 * kWave - 1) / (32 * kWave);

  uint4 wv[kRows][kWave];
  int64_t g = gw;
  if (g < ngroups) load_wave<MT>(p, g, 0, wv);  // weights do not depend on the previous kernel

  pdl_wait();
  pdl_launch_dependents();

  // ---- prologue: stage the activation rows (optionally embedding gather + RMSNorm) as fp32 in smem ----
  if (p.xs_smem) {
    const int segs = p.segs;
    for (int64_t mm = 0; mm < p.m; ++mm) {
      const void *xrow;
      if (p.flags & EGPT_FLAG_EMBED) {  // ldx holds the number of table rows in this mode
        int64_t tok = *p.token;
        if (tok < 0 || tok >= p.ldx) {
          if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
          tok = 0;
        }
        xrow = (const uint16_t *)p.x + tok * p.k;
      } else {
        xrow = p.x_bf16 ? (const void *)((const uint16_t *)p.x + mm * p.ldx) : (const void *)((const float *)p.x + mm * p.ldx);
      }
      float inv = 1.f;
      if (p.flags & EGPT_FLAG_RMSNORM) {
        float ss = 0.f;
        for (int64_t i = threadIdx.x; i < p.k; i += blockDim.x) {
          const float v = load_act(xrow, i, p.x_bf16);
          ss = fmaf(v, v, ss);
        }
        ss = block_sum(ss, red);
        inv = rsqrtf(ss / (float)p.k + p.eps);
      }
      float *xsf = (float *)xs;
      for (int64_t i = threadIdx.x; i < p.k; i += blockDim.x) {
        float v = load_act(xrow, i, p.x_bf16);
        if ((p.flags & EGPT_FLAG_EMBED) && blockIdx.x == 0) ((uint16_t *)p.residual)[i] = f32_to_bf16_bits(v);
        if (p.flags & EGPT_FLAG_RMSNORM)
          v = round_bf16(round_bf16(v * inv) * bf16_bits_to_f32(((const uint16_t *)p.norm_w)[i]));
        const int s = (int)(i >> 4), e = (int)(i & 15);
        xsf[(((mm * 4) + (e >> 2)) * segs + s) * 4 + (e & 3)] = v;
      }
    }
    __syncthreads();
  }

  // Epilogue lane mapping: lane e < kRows * MT owns (row r_e = e / MT, activation row m_e = e % MT); it loads
  // that row's scale and residual while the weights stream, then applies the epilogue in parallel.
  const int r_e = lane / MT, m_e = lane % MT;
  const bool e_lane = lane < kRows * MT && m_e < p.m;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (; g < ngroups; g += nw) {
    const int64_t row0 = g * kRows;
    const bool e_ok = e_lane && row0 + r_e < p.n;
    float s_e = 0.f, res_e = 0.f, bias_e = 0.f;
    if (e_ok) {
      const int64_t pr = phys_row(p, row0 + r_e);
      s_e = load_scale(p, pr);
      if (p.bias) bias_e = load_act(p.bias, pr, p.x_bf16);
      if (p.epilogue == EGPT_EPI_RESIDUAL) res_e = load_act(p.residual, m_e * p.ldo + row0 + r_e, p.x_bf16);
    }
    uint64_t acc2[kRows][MT];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) acc2[r][mm] = 0ull;
    for (int wave = 0; wave < nwaves; ++wave) {
      if (wave > 0) load_wave<MT>(p, g, wave, wv);
#pragma unroll
      for (int j = 0; j < kWave; ++j) {
        const int seg = (wave * kWave + j) * 32 + lane;
        if (seg < p.segs) {
#pragma unroll
          for (int mm = 0; mm < MT; ++mm) {
            if (mm < p.m) {
              uint64_t x2[8];
              load_x16(p, xs, mm, seg, x2);
#pragma unroll
              for (int r = 0; r < kRows; ++r) acc2[r][mm] = dot16x2(x2, wv[r][j], acc2[r][mm]);
            }
          }
        }
      }
    }
    // the next task's first wave streams in while this one is reduced and stored
    if (g + nw < ngroups) load_wave<MT>(p, g + nw, 0, wv);
    float mine = 0.f;
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) {
        const float2 t = unpack2(acc2[r][mm]);
        const float tot = warp_sum(t.x + t.y);
        if (r * MT + mm == lane) mine = tot;
      }
    // (gate, up) pairs: the up row's sum and scale sit MT lanes above the gate row's lane
    const float up_tot = __shfl_down_sync(0xffffffffu, mine, MT);
    const float up_s = __shfl_down_sync(0xffffffffu, s_e, MT);
    if (e_ok) {
      const int bf = p.x_bf16;
      const int64_t lr = row0 + r_e;
      if (p.argmax) {
        const float y = apply_scale(p, mine, s_e, bias_e);
        if (p.logits) store_act(p.logits, lr, y, bf);
        if (argmax_better(y, (int)lr, best_v, best_i)) {
          best_v = y;
          best_i = (int)lr;
        }
      } else if (p.epilogue == EGPT_EPI_SILU_MUL) {
        if (r_e == 0) {  // a task is exactly one (gate, up) pair
          const float gt = apply_scale(p, mine, s_e, 0.f), up = apply_scale(p, up_tot, up_s, 0.f);
          const float out = bf ? round_bf16(round_bf16(silu_f32(gt)) * up) : silu_f32(gt) * up;
          store_act(p.out, m_e * p.ldo + (row0 >> 1), out, bf);
        }
      } else {
        const float y = apply_scale(p, mine, s_e, bias_e);
        float out = y;
        if (p.epilogue == EGPT_EPI_RESIDUAL) out = bf ? round_bf16(res_e + y) : res_e + y;
        else if (p.epilogue == EGPT_EPI_GELU) out = gelu_erf_f32(y);
        store_act(p.out, m_e * p.ldo + lr, out, bf);
      }
    }
  }
  if (p.argmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (argmax_better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
  }

  if (p.argmax) {
    // CTA-level (value, index) reduction, then the last CTA to finish reduces the per-CTA partials.
    if (lane == 0) {
      s_bv[warp] = best_v;
      s_bi[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bv = s_bv[0];
      int bi = s_bi[0];
      for (int w = 1; w < kGemvWarps; ++w)
        if (argmax_better(s_bv[w], s_bi[w], bv, bi)) {
          bv = s_bv[w];
          bi = s_bi[w];
        }
      p.ws_val[blockIdx.x] = bv;
      p.ws_idx[blockIdx.x] = bi;
      __threadfence();
      const unsigned prev = atomicAdd(p.ws_counter, 1u);
      s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last) {  // the whole last CTA reduces the per-CTA partials (strided, then warps, then warp 0)
      __threadfence();
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
        const float v = __ldcg(&p.ws_val[b]);
        const int i = __ldcg(&p.ws_idx[b]);
        if (argmax_better(v, i, bv, bi)) {
          bv = v;
          bi = i;
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
      __syncthreads();
      if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < kGemvWarps; ++w)
          if (argmax_better(s_bv[w], s_bi[w], bv, bi)) {
            bv = s_bv[w];
            bi = s_bi[w];
          }
        *p.tok_out = (int64_t)bi;
        if ((p.flags & EGPT_FLAG_ADVANCE) && p.position) *p.position += 1;
        *p.ws_counter = 0u;
      }
    }
  }
}

// Plain-load fallback for shapes the vector path cannot take (k % 16 != 0, unaligned pointers).
// One warp per output row (two rows for SiLU pairs), per-lane strided sums, same epilogues.
__global__ void __launch_bounds__(256) gemv_i8_plain_kernel(const GemvParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int step = p.epilogue == EGPT_EPI_SILU_MUL ? 2 : 1;
  for (int64_t task = gw; task < (p.n / step) * p.m; task += nw) {
    const int64_t row = (task / p.m) * step, mm = task % p.m;
    float a0 = 0.f, a1 = 0.f;
    for (int64_t kk = lane; kk < p.k; kk += 32) {
      const float xv = load_act(p.x, mm * p.ldx + kk, p.x_bf16);
      a0 = fmaf(xv, (float)p.w[phys_row(p, row) * p.k + kk], a0);
      if (step == 2) a1 = fmaf(xv, (float)p.w[phys_row(p, row + 1) * p.k + kk], a1);
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if (lane == 0) emit(p, row, mm, a0, a1);
  }
}

// ------------------------------------------------------------------------------------------------ host side
template <int MT>
static cudaError_t launch_gemv(const GemvParams &p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemv_i8_kernel<MT>;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kXsMaxBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  return launch_kernel((const void *)kern, dim3(grid), dim3(kGemvThreads), smem, st, pdl, p);
}

int gemv_tc_launch(const GemvParams &gp, cudaStream_t st);  // gemv_tc.cu

int gemv_launch(GemvParams p, cudaStream_t st) {
  const bool pdl = (p.flags & EGPT_FLAG_PDL) != 0;
  if (p.m > kMaxMT) {  // the kernel holds up to 8 activation rows: split larger M into row blocks
    GemvParams a = p, b = p;
    a.m = kMaxMT;
    b.m = p.m - kMaxMT;
    b.x = p.x_bf16 ? (const void *)((const uint16_t *)p.x + kMaxMT * p.ldx) : (const void *)((const float *)p.x + kMaxMT * p.ldx);
    const int esz = p.x_bf16 ? 2 : 4;
    b.out = (char *)p.out + (size_t)kMaxMT * p.ldo * esz;
    if (p.residual) b.residual = (char *)p.residual + (size_t)kMaxMT * p.ldo * esz;
    if (int rc = gemv_launch(a, st)) return rc;
    return gemv_launch(b, st);
  }
  const bool aligned = (p.k % 16 == 0) && ((uintptr_t)p.w % 16 == 0);
  const bool x_aligned = ((uintptr_t)p.x % 16 == 0) && ((p.ldx * (p.x_bf16 ? 2 : 4)) % 16 == 0);
  p.segs = (int)((p.k + 15) / 16);
  int mt = 1;
  while (mt < p.m) mt *= 2;
  p.xs_smem = (size_t)mt * p.k * 4 <= (size_t)kXsMaxBytes;
  const bool fast_ok = aligned && !(p.flags & EGPT_FLAG_NO_TMA) && (p.xs_smem || x_aligned);
  if (!fast_ok) {
    if (p.argmax || (p.flags & (EGPT_FLAG_RMSNORM | EGPT_FLAG_EMBED)))
      return set_error(EGPT_ERR_ALIGN, "gemv: argmax/RMSNorm/embedding fusion needs k %% 16 == 0, 16-byte aligned weights "
                                       "and m*k*4 <= 64 KiB");
    const int unit = p.epilogue == EGPT_EPI_SILU_MUL ? 2 : 1;
    const int64_t tasks = (p.n / unit) * p.m;
    const int blocks = (int)std::min<int64_t>((tasks + 7) / 8, 4096);
    return check_launch(launch_kernel((const void *)gemv_i8_plain_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, st,
                                      pdl, p),
                        "gemv_i8_plain_kernel");
  }
  const int64_t groups = (p.n + kRows - 1) / kRows;
  const int per_sm = mt == 1 ? 3 : 2;
  int grid = (int)std::min<int64_t>((groups + kGemvWarps - 1) / kGemvWarps, (int64_t)num_sms() * per_sm);
  if (p.argmax) grid = std::min(grid, kArgmaxMaxCtas);
  grid = std::max(grid, 1);
  const size_t smem = p.xs_smem ? (size_t)mt * p.k * 4 : 16;
  cudaError_t e;
  switch (mt) {
    case 1: e = launch_gemv<1>(p, grid, smem, st, pdl); break;
    case 2: e = launch_gemv<2>(p, grid, smem, st, pdl); break;
    case 4: e = launch_gemv<4>(p, grid, smem, st, pdl); break;
    default: e = launch_gemv<8>(p, grid, smem, st, pdl); break;
  }
  return check_launch(e, "gemv_i8_kernel");
}

}  // namespace egpt

using namespace egpt;

extern "C" int egpt_gemv_i8(void *out, const void *x, int x_dtype, int64_t m, int64_t ldx, int64_t ldo,
                            const int8_t *w, const void *scale, int scale_dtype, int64_t n, int64_t k,
                            const void *bias, void *residual, int epilogue, const void *norm_w, float eps,
                            const int64_t *token, unsigned flags, void *stream) {
  clear_error();
  if (!out || !x || !w || !scale) return set_error(EGPT_ERR_ARG, "gemv: null pointer");
  if (m < 1 || m > 16) return set_error(EGPT_ERR_SHAPE, "gemv: m must be in [1, 16]");
  if (n < 1 || k < 1) return set_error(EGPT_ERR_SHAPE, "gemv: n and k must be positive");
  if (x_dtype != EGPT_BF16 && x_dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "gemv: x dtype");
  if (scale_dtype != EGPT_BF16 && scale_dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "gemv: scale dtype");
  if (epilogue < EGPT_EPI_NONE || epilogue > EGPT_EPI_GELU) return set_error(EGPT_ERR_ARG, "gemv: epilogue");
  if (epilogue == EGPT_EPI_RESIDUAL && !residual) return set_error(EGPT_ERR_ARG, "gemv: residual epilogue needs residual");
  if (epilogue == EGPT_EPI_SILU_MUL && (n % 2)) return set_error(EGPT_ERR_SHAPE, "gemv: SiLU*up needs an even row count");
  if (epilogue == EGPT_EPI_GELU && x_dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "gemv: GELU epilogue is fp32 only");
  if ((flags & EGPT_FLAG_RMSNORM) && (!norm_w || x_dtype != EGPT_BF16))
    return set_error(EGPT_ERR_ARG, "gemv: RMSNorm prologue needs bf16 x and norm_w");
  if ((flags & EGPT_FLAG_EMBED) && (!token || !residual || m != 1 || x_dtype != EGPT_BF16))
    return set_error(EGPT_ERR_ARG, "gemv: embedding prologue needs token, residual, m == 1 and bf16");
  if ((flags & EGPT_FLAG_DOUBLE_ROUND) && x_dtype != EGPT_BF16)
    return set_error(EGPT_ERR_DTYPE, "gemv: double rounding is a bf16 mode");
  if (ldx < k && !(flags & EGPT_FLAG_EMBED)) return set_error(EGPT_ERR_SHAPE, "gemv: ldx < k");
  if ((flags & EGPT_FLAG_EMBED) && ldx < 1) return set_error(EGPT_ERR_SHAPE, "gemv: embedding table rows (ldx) < 1");
  const int64_t out_cols = epilogue == EGPT_EPI_SILU_MUL ? n / 2 : n;
  if (ldo < out_cols) return set_error(EGPT_ERR_SHAPE, "gemv: ldo too small");
  GemvParams p{};
  p.out = out;
  p.x = x;
  p.m = m;
  p.ldx = ldx;
  p.ldo = ldo;
  p.w = w;
  p.scale = scale;
  p.scale_bf16 = scale_dtype == EGPT_BF16;
  p.x_bf16 = x_dtype == EGPT_BF16;
  p.n = n;
  p.k = k;
  p.bias = bias;
  p.residual = residual;
  p.norm_w = norm_w;
  p.eps = eps;
  p.token = token;
  p.flags = flags;
  p.epilogue = epilogue;
  if (flags & EGPT_FLAG_EXACT) return gemv_tc_launch(p, (cudaStream_t)stream);
  return gemv_launch(p, (cudaStream_t)stream);
}

extern "C" size_t egpt_lm_head_ws_bytes(int64_t n) {
  (void)n;
  return (size_t)kArgmaxMaxCtas * 8 + 64;
}

extern "C" int egpt_lm_head_argmax(int64_t *token, int64_t *position, void *logits, const void *x, const int8_t *w,
                                   const void *scale, int scale_dtype, int64_t n, int64_t k, const void *norm_w,
                                   float eps, void *ws, size_t ws_bytes, unsigned flags, void *stream) {
  clear_error();
  if (!token || !x || !w || !scale || !ws) return set_error(EGPT_ERR_ARG, "lm_head_argmax: null pointer");
  if (n < 1 || n > 0x7fffffff || k < 1) return set_error(EGPT_ERR_SHAPE, "lm_head_argmax: bad n or k");
  if (ws_bytes < egpt_lm_head_ws_bytes(n)) return set_error(EGPT_ERR_WORKSPACE, "lm_head_argmax: workspace too small");
  if ((uintptr_t)ws % 16) return set_error(EGPT_ERR_ALIGN, "lm_head_argmax: workspace must be 16-byte aligned");
  if ((flags & EGPT_FLAG_RMSNORM) && !norm_w) return set_error(EGPT_ERR_ARG, "lm_head_argmax: norm_w missing");
  if ((flags & EGPT_FLAG_ADVANCE) && !position) return set_error(EGPT_ERR_ARG, "lm_head_argmax: position missing");
  if (scale_dtype != EGPT_BF16 && scale_dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "lm_head_argmax: scale dtype");
  GemvParams p{};
  p.out = nullptr;
  p.x = x;
  p.m = 1;
  p.ldx = k;
  p.ldo = n;
  p.w = w;
  p.scale = scale;
  p.scale_bf16 = scale_dtype == EGPT_BF16;
  p.x_bf16 = (flags & EGPT_FLAG_X_F32) ? 0 : 1;
  p.n = n;
  p.k = k;
  p.norm_w = norm_w;
  p.eps = eps;
  p.flags = flags & (EGPT_FLAG_RMSNORM | EGPT_FLAG_PDL | EGPT_FLAG_ADVANCE);
  p.epilogue = EGPT_EPI_NONE;
  p.argmax = 1;
  p.tok_out = token;
  p.position = position;
  p.logits = logits;
  p.ws_val = (float *)ws;
  p.ws_idx = (int *)((char *)ws + kArgmaxMaxCtas * 4);
  p.ws_counter = (unsigned *)((char *)ws + kArgmaxMaxCtas * 8);
  if (flags & EGPT_FLAG_EXACT) return gemv_tc_launch(p, (cudaStream_t)stream);
  return gemv_launch(p, (cudaStream_t)stream);
}
