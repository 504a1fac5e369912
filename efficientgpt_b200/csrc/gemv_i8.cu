// Int8 weight-only GEMV / small-M GEMM for B200 (sm_100a), CUDA cores only.
//
// Reference behaviour (BagelsFun/efficientgpt research/realmodel/int8_linear.py:26-98): out[m, n] =
// bf16(s[n] * sum_k bf16(x[m,k]) * q[n,k]) with fp32 accumulation; rows > 16 take the reference's prefill
// branch, bf16(bf16(x @ bf16(q).T) * s) (EGPT_FLAG_DOUBLE_ROUND reproduces that double rounding).
//
// B200 design. Batch-1 decode is a pure weight stream (N*K int8 bytes, read once per token), so the kernel
// is built around keeping HBM busy:
//   * one CTA per SM (grid = #SMs), each owning a contiguous range of output rows;
//   * the CTA's rows are cut into items of 4 rows x 512 columns (2 KB); every warp owns a private ring of
//     kStages item buffers in shared memory filled by 1-D cp.async.bulk copies (TMA, no multicast) that
//     complete on a per-stage mbarrier, so each SM keeps 8 warps x 4 stages x 2 KB = 64 KB in flight;
//   * the first ring fill is issued BEFORE griddepcontrol.wait: weights do not depend on the previous
//     kernel, so under programmatic dependent launch the weight stream overlaps the previous kernel's tail;
//   * the activation row is staged once per CTA in shared memory as fp32, in a [4][segments] float4 layout
//     so that lane l reading segment l is bank-conflict free; the RMSNorm / embedding prologue is fused;
//   * int8 -> fp32 is exact (PRMT into 2^23's mantissa + one FADD); products are exact in fp32 and are
//     summed in a fixed order (16 per lane, warp butterfly, then chunks in column order), so every run and
//     every CTA gives the same bits;
//   * epilogues (scale, bias, residual add, SiLU*up, GELU, lm_head argmax with a last-CTA reduction) run on
//     the per-row sums while they are in shared memory.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace egpt {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kItemRows = 4;                       // rows per item
constexpr int kItemCols = 512;                     // columns per item: one 16-byte segment per lane
constexpr int kStages = 4;                         // ring depth per warp
constexpr int kStageBytes = kItemRows * kItemCols; // 2 KB
constexpr int kPartFloats = 6144;                  // per-window partial sums (24 KB)
constexpr int kXsMaxBytes = 48 * 1024;             // fp32 activation staging limit

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
  int nk;        // column chunks per row
  int segs;      // 16-byte segments per row (k / 16)
  int unit;      // row granularity of the CTA split (2 for SiLU pairs)
  int xs_smem;   // 1: activations staged in shared memory, 0: read from global in the loop
  int win_rows;  // rows per partial-sum window (multiple of kItemRows)
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

// Physical weight row of logical row `lr`. With SiLU*up the weight is cat(gate, up) ([2I, K]) and the kernel
// walks logical rows interleaved (gate_0, up_0, gate_1, up_1, ...) so both halves of a pair meet in one item.
__device__ __forceinline__ int64_t phys_row(const GemvParams &p, int64_t lr) {
  if (p.epilogue != EGPT_EPI_SILU_MUL) return lr;
  return (lr & 1) ? (p.n >> 1) + (lr >> 1) : (lr >> 1);
}

// Epilogue for one (row, m), or for one (gate, up) pair given its even logical row n.
__device__ __forceinline__ void emit(const GemvParams &p, int64_t n, int64_t m, float acc0, float acc1) {
  const int bf = p.x_bf16;
  switch (p.epilogue) {
    case EGPT_EPI_SILU_MUL: {
      const int64_t j = n >> 1;
      const float g = scaled_value(p, j, acc0), u = scaled_value(p, (p.n >> 1) + j, acc1);
      float out;
      if (bf)
        out = round_bf16(round_bf16(silu_f32(g)) * u);
      else
        out = silu_f32(g) * u;
      store_act(p.out, m * p.ldo + j, out, bf);
      break;
    }
    case EGPT_EPI_RESIDUAL: {
      const float y = scaled_value(p, n, acc0);
      const float r = load_act(p.residual, m * p.ldo + n, bf);
      store_act(p.out, m * p.ldo + n, bf ? round_bf16(r + y) : r + y, bf);
      break;
    }
    case EGPT_EPI_GELU: {
      store_act(p.out, m * p.ldo + n, gelu_erf_f32(scaled_value(p, n, acc0)), bf);
      break;
    }
    default:
      store_act(p.out, m * p.ldo + n, scaled_value(p, n, acc0), bf);
  }
}

// Rows [r0, r1) of CTA b, split in multiples of `unit` rows as evenly as possible.
__device__ __forceinline__ void cta_rows(int64_t n, int unit, int64_t b, int64_t g, int64_t &r0, int64_t &r1) {
  const int64_t units = n / unit;
  r0 = unit * ((b * units) / g);
  r1 = unit * (((b + 1) * units) / g);
}

// Exact 16-term dot product of fp32 x[0..15] with 16 int8 weights (fixed order).
__device__ __forceinline__ float dot16(const float4 &x0, const float4 &x1, const float4 &x2, const float4 &x3,
                                       const uint4 &wv, float acc) {
  const uint32_t w0 = wv.x ^ 0x80808080u, w1 = wv.y ^ 0x80808080u, w2 = wv.z ^ 0x80808080u,
                 w3 = wv.w ^ 0x80808080u;
  acc = fmaf(x0.x, i8_to_f32(w0, 0), acc);
  acc = fmaf(x0.y, i8_to_f32(w0, 1), acc);
  acc = fmaf(x0.z, i8_to_f32(w0, 2), acc);
  acc = fmaf(x0.w, i8_to_f32(w0, 3), acc);
  acc = fmaf(x1.x, i8_to_f32(w1, 0), acc);
  acc = fmaf(x1.y, i8_to_f32(w1, 1), acc);
  acc = fmaf(x1.z, i8_to_f32(w1, 2), acc);
  acc = fmaf(x1.w, i8_to_f32(w1, 3), acc);
  acc = fmaf(x2.x, i8_to_f32(w2, 0), acc);
  acc = fmaf(x2.y, i8_to_f32(w2, 1), acc);
  acc = fmaf(x2.z, i8_to_f32(w2, 2), acc);
  acc = fmaf(x2.w, i8_to_f32(w2, 3), acc);
  acc = fmaf(x3.x, i8_to_f32(w3, 0), acc);
  acc = fmaf(x3.y, i8_to_f32(w3, 1), acc);
  acc = fmaf(x3.z, i8_to_f32(w3, 2), acc);
  acc = fmaf(x3.w, i8_to_f32(w3, 3), acc);
  return acc;
}

// Load 16 activations x[m, 16*seg ..] as 4 float4 from global memory (bf16 or fp32).
__device__ __forceinline__ void load_x16_global(const GemvParams &p, int64_t m, int seg, float4 &a, float4 &b,
                                                float4 &c, float4 &d) {
  if (p.x_bf16) {
    const uint4 *src = (const uint4 *)((const uint16_t *)p.x + m * p.ldx + 16 * (int64_t)seg);
    const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
    a = make_float4(bf16_lo(u0.x), bf16_hi(u0.x), bf16_lo(u0.y), bf16_hi(u0.y));
    b = make_float4(bf16_lo(u0.z), bf16_hi(u0.z), bf16_lo(u0.w), bf16_hi(u0.w));
    c = make_float4(bf16_lo(u1.x), bf16_hi(u1.x), bf16_lo(u1.y), bf16_hi(u1.y));
    d = make_float4(bf16_lo(u1.z), bf16_hi(u1.z), bf16_lo(u1.w), bf16_hi(u1.w));
  } else {
    const float4 *src = (const float4 *)((const float *)p.x + m * p.ldx + 16 * (int64_t)seg);
    a = __ldg(src);
    b = __ldg(src + 1);
    c = __ldg(src + 2);
    d = __ldg(src + 3);
  }
}

struct ItemCoord {
  int64_t row0;  // first row of the item (absolute)
  int nrows;     // valid rows (1..4)
  int chunk;     // column chunk
  int bytes;     // bytes per row in this chunk
  int win;       // window index within the CTA
  int local_row; // row offset of row0 inside its window
};

__device__ __forceinline__ ItemCoord item_coord(const GemvParams &p, int64_t r0, int64_t r1, int64_t item) {
  const int64_t rows = r1 - r0;
  const int64_t full_win_items = (int64_t)(p.win_rows / kItemRows) * p.nk;
  const int64_t win = item / full_win_items;
  const int64_t local = item - win * full_win_items;
  const int64_t g = local / p.nk;
  ItemCoord c;
  c.win = (int)win;
  c.chunk = (int)(local - g * p.nk);
  c.local_row = (int)(g * kItemRows);
  c.row0 = r0 + win * p.win_rows + g * kItemRows;
  const int64_t left = rows - (c.row0 - r0);
  c.nrows = (int)(left < kItemRows ? left : kItemRows);
  const int64_t col0 = (int64_t)c.chunk * kItemCols;
  const int64_t cb = p.k - col0;
  c.bytes = (int)(cb < kItemCols ? cb : kItemCols);
  return c;
}

__device__ __forceinline__ int64_t cta_items(const GemvParams &p, int64_t rows) {
  const int64_t full_wins = rows / p.win_rows;
  const int64_t tail = rows - full_wins * p.win_rows;
  return full_wins * (p.win_rows / kItemRows) * p.nk + ((tail + kItemRows - 1) / kItemRows) * p.nk;
}

__device__ __forceinline__ void issue_item(const GemvParams &p, const ItemCoord &c, uint8_t *stage, uint64_t *bar,
                                           uint64_t policy) {
  mbar_arrive_expect_tx(bar, (uint32_t)(c.nrows * c.bytes));
  const int8_t *src = p.w + (int64_t)c.chunk * kItemCols;
  for (int r = 0; r < c.nrows; ++r)
    bulk_g2s_stream(stage + r * kItemCols, src + phys_row(p, c.row0 + r) * p.k, (uint32_t)c.bytes, bar, policy);
}

template <int MT>
__global__ void __launch_bounds__(kGemvThreads, MT <= 2 ? 2 : 1) gemv_i8_tma_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ring = smem;                                                     // kGemvWarps * kStages * kStageBytes
  uint64_t *bars = (uint64_t *)(ring + kGemvWarps * kStages * kStageBytes); // kGemvWarps * kStages
  float *part = (float *)(bars + kGemvWarps * kStages);                     // kPartFloats
  float *red = part + kPartFloats;                                          // 64 floats of scratch
  float4 *xs = (float4 *)(red + 64);                                        // m * 4 * segs (when xs_smem)

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t r0, r1;
  cta_rows(p.n, p.unit, blockIdx.x, gridDim.x, r0, r1);
  const int64_t rows = r1 - r0;
  const int64_t items = rows > 0 ? cta_items(p, rows) : 0;
  const uint64_t policy = l2_policy_evict_first();

  uint8_t *my_ring = ring + warp * kStages * kStageBytes;
  uint64_t *my_bars = bars + warp * kStages;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Prefetch: the first ring fill does not depend on the previous kernel.
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      const int64_t it = warp + (int64_t)s * kGemvWarps;
      if (it < items) issue_item(p, item_coord(p, r0, r1, it), my_ring + s * kStageBytes, &my_bars[s], policy);
    }
  }

  pdl_wait();
  pdl_launch_dependents();

  // ---- prologue: stage the activation rows (optionally embedding lookup + RMSNorm) as fp32 in smem ----
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
  }
  __syncthreads();

  // ---- main loop over this warp's items, window by window ----
  const int per_row = p.nk * MT;  // partial floats per row
  int64_t seq = 0;                // this warp's item sequence number
  int64_t it = warp;
  bool ok = true;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  const int64_t nwin = rows > 0 ? (rows + p.win_rows - 1) / p.win_rows : 0;
  for (int64_t win = 0; win < nwin; ++win) {
    const int64_t win_row0 = r0 + win * p.win_rows;
    const int64_t win_rows = min((int64_t)p.win_rows, r1 - win_row0);
    for (; it < items; it += kGemvWarps, ++seq) {
      const ItemCoord c = item_coord(p, r0, r1, it);
      if (c.win != win) break;
      const int stage = (int)(seq % kStages);
      const uint32_t parity = (uint32_t)((seq / kStages) & 1);
      if (ok) ok = mbar_wait_bounded(&my_bars[stage], parity);
      float acc[kItemRows][MT];
#pragma unroll
      for (int r = 0; r < kItemRows; ++r)
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) acc[r][mm] = 0.f;
      const int seg_in_chunk = lane;
      if (ok && seg_in_chunk * 16 < c.bytes) {
        const uint8_t *st = my_ring + stage * kStageBytes + seg_in_chunk * 16;
        uint4 wv[kItemRows];
#pragma unroll
        for (int r = 0; r < kItemRows; ++r)
          wv[r] = r < c.nrows ? *(const uint4 *)(st + r * kItemCols) : make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        const int seg = c.chunk * (kItemCols / 16) + seg_in_chunk;
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) {
          if (mm < p.m) {
            float4 x0, x1, x2, x3;
            if (p.xs_smem) {
              const float4 *xb = xs + (size_t)(mm * 4) * p.segs + seg;
              x0 = xb[0];
              x1 = xb[p.segs];
              x2 = xb[2 * p.segs];
              x3 = xb[3 * p.segs];
            } else {
              load_x16_global(p, mm, seg, x0, x1, x2, x3);
            }
#pragma unroll
            for (int r = 0; r < kItemRows; ++r) acc[r][mm] = dot16(x0, x1, x2, x3, wv[r], acc[r][mm]);
          }
        }
      }
      // The stage has been read into registers: hand it back to the bulk-copy engine.
      __syncwarp();
      if (lane == 0) {
        fence_proxy_async_smem();
        const int64_t nxt = it + (int64_t)kStages * kGemvWarps;
        if (ok && nxt < items) issue_item(p, item_coord(p, r0, r1, nxt), my_ring + stage * kStageBytes, &my_bars[stage], policy);
      }
#pragma unroll
      for (int r = 0; r < kItemRows; ++r)
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) acc[r][mm] = warp_sum(acc[r][mm]);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kItemRows; ++r)
          if (r < c.nrows)
#pragma unroll
            for (int mm = 0; mm < MT; ++mm)
              if (mm < p.m) part[(c.local_row + r) * per_row + c.chunk * MT + mm] = acc[r][mm];
      }
    }
    __syncthreads();
    // ---- epilogue for this window ----
    if (p.epilogue == EGPT_EPI_SILU_MUL) {
      const int64_t pairs = win_rows / 2;
      for (int64_t t = threadIdx.x; t < pairs * p.m; t += blockDim.x) {
        const int64_t pr = t / p.m, mm = t - pr * p.m;
        float a0 = 0.f, a1 = 0.f;
        for (int ch = 0; ch < p.nk; ++ch) {
          a0 += part[(2 * pr) * per_row + ch * MT + mm];
          a1 += part[(2 * pr + 1) * per_row + ch * MT + mm];
        }
        emit(p, win_row0 + 2 * pr, mm, a0, a1);
      }
    } else if (p.argmax) {
      for (int64_t rr = threadIdx.x; rr < win_rows; rr += blockDim.x) {
        float a = 0.f;
        for (int ch = 0; ch < p.nk; ++ch) a += part[rr * per_row + ch * MT];
        const int64_t nrow = win_row0 + rr;
        const float y = scaled_value(p, nrow, a);
        if (p.logits) ((uint16_t *)p.logits)[nrow] = f32_to_bf16_bits(y);
        if (argmax_better(y, (int)nrow, best_v, best_i)) {
          best_v = y;
          best_i = (int)nrow;
        }
      }
    } else {
      for (int64_t t = threadIdx.x; t < win_rows * p.m; t += blockDim.x) {
        const int64_t rr = t / p.m, mm = t - rr * p.m;
        float a = 0.f;
        for (int ch = 0; ch < p.nk; ++ch) a += part[rr * per_row + ch * MT + mm];
        emit(p, win_row0 + rr, mm, a, 0.f);
      }
    }
    __syncthreads();
  }

  if (p.argmax) {
    // CTA-level (value, index) reduction, then the last CTA to finish reduces the per-CTA partials.
    __shared__ float s_v[kGemvWarps];
    __shared__ int s_i[kGemvWarps];
    __shared__ int s_last;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (argmax_better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      s_v[warp] = best_v;
      s_i[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bv = s_v[0];
      int bi = s_i[0];
      for (int w = 1; w < kGemvWarps; ++w)
        if (argmax_better(s_v[w], s_i[w], bv, bi)) {
          bv = s_v[w];
          bi = s_i[w];
        }
      p.ws_val[blockIdx.x] = bv;
      p.ws_idx[blockIdx.x] = bi;
      __threadfence();
      const unsigned prev = atomicAdd(p.ws_counter, 1u);
      s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
      __threadfence();
      float bv = __ldcg(&p.ws_val[0]);
      int bi = __ldcg(&p.ws_idx[0]);
      for (unsigned b = 1; b < gridDim.x; ++b) {
        const float v = __ldcg(&p.ws_val[b]);
        const int i = __ldcg(&p.ws_idx[b]);
        if (argmax_better(v, i, bv, bi)) {
          bv = v;
          bi = i;
        }
      }
      *p.tok_out = (int64_t)bi;
      if ((p.flags & EGPT_FLAG_ADVANCE) && p.position) *p.position += 1;
      *p.ws_counter = 0u;
    }
  }
  if (!ok) {
    // A stage never completed: make sure no bulk copy still targets this CTA's shared memory before exit.
    if (lane == 0)
      for (int s = 0; s < kStages; ++s) mbar_wait_bounded(&my_bars[s], 0), mbar_wait_bounded(&my_bars[s], 1);
  }
}

// Plain-load fallback for shapes the bulk-copy path cannot take (k % 16 != 0 or unaligned pointers).
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
static size_t tma_smem_bytes(int64_t m, int64_t k, bool xs_smem) {
  size_t b = (size_t)kGemvWarps * kStages * kStageBytes + (size_t)kGemvWarps * kStages * 8 + kPartFloats * 4 + 64 * 4;
  if (xs_smem) b += (size_t)m * k * 4;
  return b;
}

template <int MT>
static cudaError_t launch_tma(const GemvParams &p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  static bool configured = false;
  auto kern = gemv_i8_tma_kernel<MT>;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_kernel((const void *)kern, dim3(grid), dim3(kGemvThreads), smem, st, pdl, p);
}

int gemv_launch(GemvParams p, cudaStream_t st) {
  const bool pdl = (p.flags & EGPT_FLAG_PDL) != 0;
  const bool aligned = (p.k % 16 == 0) && ((uintptr_t)p.w % 16 == 0);
  const bool x_aligned = ((uintptr_t)p.x % 16 == 0) && ((p.ldx * (p.x_bf16 ? 2 : 4)) % 16 == 0);
  p.unit = p.epilogue == EGPT_EPI_SILU_MUL ? 2 : 1;
  p.segs = (int)((p.k + 15) / 16);
  p.nk = (int)((p.k + kItemCols - 1) / kItemCols);
  const bool tma_ok = aligned && !(p.flags & EGPT_FLAG_NO_TMA) && p.m <= 16;
  if (!tma_ok) {
    if (p.argmax || (p.flags & (EGPT_FLAG_RMSNORM | EGPT_FLAG_EMBED)))
      return set_error(EGPT_ERR_ALIGN, "gemv: argmax/RMSNorm/embedding fusion needs k %% 16 == 0 and 16-byte aligned weights");
    const int64_t tasks = (p.n / p.unit) * p.m;
    const int blocks = (int)std::min<int64_t>((tasks + 7) / 8, 4096);
    return check_launch(launch_kernel((const void *)gemv_i8_plain_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, st,
                                      pdl, p),
                        "gemv_i8_plain_kernel");
  }
  p.xs_smem = (size_t)p.m * p.k * 4 <= (size_t)kXsMaxBytes;
  if (!p.xs_smem && (p.flags & (EGPT_FLAG_RMSNORM | EGPT_FLAG_EMBED)))
    return set_error(EGPT_ERR_SHAPE, "gemv: fused RMSNorm/embedding needs m*k*4 <= 48 KiB");
  if (!p.xs_smem && !x_aligned) {
    p.flags |= EGPT_FLAG_NO_TMA;
    return gemv_launch(p, st);
  }
  int mt = 1;
  while (mt < p.m) mt *= 2;
  int win = (int)(kPartFloats / (p.nk * mt));
  win = (win / kItemRows) * kItemRows;
  if (win < kItemRows) return set_error(EGPT_ERR_SHAPE, "gemv: k too large for the partial-sum window");
  p.win_rows = win;
  const int64_t units = p.n / p.unit;
  int grid = (int)std::min<int64_t>(units, num_sms());
  if (p.argmax) grid = std::min(grid, kArgmaxMaxCtas);
  grid = std::max(grid, 1);
  const size_t smem = tma_smem_bytes(mt, p.k, p.xs_smem);
  cudaError_t e;
  switch (mt) {
    case 1: e = launch_tma<1>(p, grid, smem, st, pdl); break;
    case 2: e = launch_tma<2>(p, grid, smem, st, pdl); break;
    case 4: e = launch_tma<4>(p, grid, smem, st, pdl); break;
    case 8: e = launch_tma<8>(p, grid, smem, st, pdl); break;
    default: e = launch_tma<16>(p, grid, smem, st, pdl); break;
  }
  return check_launch(e, "gemv_i8_tma_kernel");
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
  GemvParams p{};
  p.out = nullptr;
  p.x = x;
  p.m = 1;
  p.ldx = k;
  p.ldo = n;
  p.w = w;
  p.scale = scale;
  p.scale_bf16 = scale_dtype == EGPT_BF16;
  p.x_bf16 = 1;
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
  return gemv_launch(p, (cudaStream_t)stream);
}
