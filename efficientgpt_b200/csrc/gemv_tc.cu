// Exact int8 tensor-core GEMV for one activation row (egpt_gemv_i8 with EGPT_FLAG_EXACT).
//
// replaces: research/realmodel/int8_linear.py:26-38,67-85 (_dot16 through int8_matmul) for M = 1, with the
// arithmetic of the persistent decode step's GEMV stages (decode_step.cu): the input row is staged once per CTA
// as fixed point x = X 2^E (|X| < 2^30) in four balanced int8 digit planes, mma.sync.m16n8k32.s8 multiplies
// 16-row x 256-column int8 weight items by the planes (exact int32 per item), the planes fold into exact int64
// row sums, and each row is rounded once before the scale: out = bf16(fp32(sum) * s) (bf16 rounding points of
// the op), or with the residual / SiLU*up epilogues of the decode step.
//
// Work split: tile t (16 rows; gate|up: gate rows 8t..8t+7 then up rows 8t..8t+7) belongs to CTA t % G. With at
// least 16 tiles per CTA every warp owns whole tiles (chunks accumulate in the MMA registers, epilogue in the
// warp); with fewer, a CTA's items (tile, 256-column chunk) go round robin to its 16 warps and the per-item row
// sums meet in shared memory (fixed order, integers). Each warp streams its items through a shared-memory ring
// (cp.async, 2-3 items in flight); the first items are requested before the programmatic-dependent-launch wait,
// since weights do not depend on the previous kernel.
namespace egpt {
namespace tc {

using ps::kChunkCols;
using ps::kCT;
using ps::kItemBytes;
using ps::kNC;
using ps::kTileRows;

struct TcParams {
  uint16_t *out;
  const uint16_t *x, *residual, *norm_w;
  const int64_t *token;  // embedding prologue: x is the table [table_rows, k], row *token; CTA 0 copies it to
  uint16_t *embed_to;    // embed_to (the residual stream)
  int64_t table_rows;
  const int8_t *w;
  const void *s;
  int s_bf16, epi, nk, ring, whole;
  int64_t n, k, tiles;
  float eps;
  int part_bytes;
  // lm_head argmax (out unused, logits nullable): each CTA's best (logit, row) into ws, the last CTA to finish
  // writes the token (first index on ties) and, with advance, position + 1
  int argmax, advance;
  int64_t *tok_out, *position;
  uint16_t *logits;
  float *ws_val;
  int *ws_idx;
  unsigned *ws_counter;
};

__device__ __forceinline__ int64_t tc_row(const TcParams &p, int64_t t, int r) {
  if (p.epi != EGPT_EPI_SILU_MUL) return t * kTileRows + r;
  return r < 8 ? t * 8 + r : (p.n >> 1) + t * 8 + (r - 8);
}
__device__ __forceinline__ float tc_scale(const TcParams &p, int64_t row) {
  return p.s_bf16 ? bf16_bits_to_f32(((const uint16_t *)p.s)[row]) : ((const float *)p.s)[row];
}

// Item j of this warp: whole mode walks its tiles (warp, warp + 16, ...) chunk by chunk; split mode takes the CTA's
// items warp, warp + 16, ... of the (tile-local, chunk) list. Returns false past the end.
__device__ __forceinline__ bool tc_item(const TcParams &p, int ntl, int j, int &tl, int &c) {
  const int warp = threadIdx.x >> 5;
  if (p.whole) {
    tl = warp + kNC * (j / p.nk);
    c = j % p.nk;
    return tl < ntl;
  }
  const int i = warp + kNC * j;
  tl = i / p.nk;
  c = i % p.nk;
  return tl < ntl;
}

// 16 rows x 256 columns of tile `tile`, chunk c, into a ring slot (16-byte pieces, rows XOR-swizzled as in the
// decode step); pieces past the end of the row are skipped (their x digits are zero).
__device__ __forceinline__ void tc_fill(const TcParams &p, int64_t tile, int c, uint8_t *slot) {
  const int lane = threadIdx.x & 31, hi = lane >> 4, pc = lane & 15;
  const int64_t col0 = (int64_t)c * kChunkCols;
  if (pc * 16 < p.k - col0) {
    const int8_t *g0 = p.w + tc_row(p, tile, hi) * p.k + col0 + pc * 16;
    const int8_t *g1 = p.w + tc_row(p, tile, 8 + hi) * p.k + col0 + pc * 16;
    uint8_t *d = slot + hi * kChunkCols + 16 * (pc ^ (hi << 2));
#pragma unroll
    for (int i = 0; i < 4; ++i) ps::cp_async16(d + i * 2 * kChunkCols, g0 + (int64_t)i * 2 * p.k);
#pragma unroll
    for (int i = 0; i < 4; ++i) ps::cp_async16(d + (8 + i * 2) * kChunkCols, g1 + (int64_t)i * 2 * p.k);
  }
}

// Output of one (gate, up) or plain row pair from exact sums: y = fp32(T) 2^E, then the op's rounding points.
__device__ __forceinline__ void tc_emit(const TcParams &p, int64_t tile, int r, long long T0, long long T1, int E,
                                        float s0, float s1, float res) {
  const float y0 = ps::mul_pow2(__ll2float_rn(T0), E);
  if (p.epi == EGPT_EPI_SILU_MUL) {
    const float gt = round_bf16(y0 * s0), up = round_bf16(ps::mul_pow2(__ll2float_rn(T1), E) * s1);
    p.out[tile * 8 + r] = f32_to_bf16_bits(round_bf16(gt / (1.0f + expf(-gt))) * up);
  } else if (p.epi == EGPT_EPI_RESIDUAL) {
    p.out[tile * kTileRows + r] = f32_to_bf16_bits(res + round_bf16(y0 * s0));
  } else {
    p.out[tile * kTileRows + r] = f32_to_bf16_bits(y0 * s0);
  }
}

// lm_head logit of one row from its exact sum: bf16(fp32(T) 2^E * s), kept if it beats the thread's best.
__device__ __forceinline__ void tc_best(const TcParams &p, int64_t row, long long T, int E, float s, float &bv, int &bi) {
  const float y = round_bf16(ps::mul_pow2(__ll2float_rn(T), E) * s);
  if (p.logits) p.logits[row] = f32_to_bf16_bits(y);
  if (argmax_better(y, (int)row, bv, bi)) bv = y, bi = (int)row;
}

// All threads: the CTA's best (warps, then thread 0) into ws; the last CTA to arrive reduces every CTA's best.
__device__ void tc_argmax_finish(const TcParams &p, float bv, int bi) {
  __shared__ float s_bv[kNC];
  __shared__ int s_bi[kNC];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) bv = ov, bi = oi;
  }
  if (lane == 0) s_bv[warp] = bv, s_bi[warp] = bi;
  ps::csync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kNC; ++w)
      if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
    p.ws_val[blockIdx.x] = bv;
    p.ws_idx[blockIdx.x] = bi;
    __threadfence();
    s_last = atomicAdd(p.ws_counter, 1u) == gridDim.x - 1;
  }
  ps::csync();
  if (!s_last) return;
  __threadfence();
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += kCT) {
    const float v = __ldcg(&p.ws_val[b]);
    const int i = __ldcg(&p.ws_idx[b]);
    if (argmax_better(v, i, bv, bi)) bv = v, bi = i;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) bv = ov, bi = oi;
  }
  ps::csync();
  if (lane == 0) s_bv[warp] = bv, s_bi[warp] = bi;
  ps::csync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kNC; ++w)
      if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
    *p.tok_out = (int64_t)bi;
    if (p.advance && p.position) *p.position += 1;
    *p.ws_counter = 0u;
  }
}

template <int RING>
__global__ void __launch_bounds__(kCT, 1) gemv_tc_kernel(const TcParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  float *red = (float *)smem;  // 64 floats
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t *ring = smem + 256 + (size_t)warp * RING * kItemBytes;
  long long *part = (long long *)(smem + 256 + (size_t)kNC * RING * kItemBytes);
  int8_t *xd = (int8_t *)((uint8_t *)part + p.part_bytes);
  const int G = gridDim.x;
  const int ntl = (int)(blockIdx.x < p.tiles ? (p.tiles - blockIdx.x + G - 1) / G : 0);

  // weights first (independent of the previous kernel)
  int tl, c;
#pragma unroll
  for (int j = 0; j < RING; ++j) {
    if (tc_item(p, ntl, j, tl, c)) tc_fill(p, blockIdx.x + (int64_t)G * tl, c, ring + j * kItemBytes);
    ps::cp_async_commit();
  }
  ps::NormW nw;
  if (p.norm_w) ps::load_norm(p.norm_w, p.k, nw);
  // split-mode epilogue thread e: row r of tile-local tl_e; its scales now, its residual after the wait
  const int per_tile = p.epi == EGPT_EPI_SILU_MUL ? 8 : kTileRows;
  const int e = threadIdx.x;
  const bool epi = !p.whole && e < ntl * per_tile;
  const int64_t etile = blockIdx.x + (int64_t)G * (e / per_tile);
  const int er = e % per_tile;
  float es0 = 0.f, es1 = 0.f, eres = 0.f;
  if (epi) {
    es0 = tc_scale(p, tc_row(p, etile, er));
    if (p.epi == EGPT_EPI_SILU_MUL) es1 = tc_scale(p, tc_row(p, etile, er + 8));
  }

  pdl_wait();
  pdl_launch_dependents();
  if (epi && p.epi == EGPT_EPI_RESIDUAL) eres = bf16_bits_to_f32(__ldcg(p.residual + etile * kTileRows + er));
  const uint16_t *xrow = p.x;
  if (p.token) {  // embedding row of the current token (bounds-checked), stored by CTA 0 as the residual stream
    int64_t tok = *p.token;
    if (tok < 0 || tok >= p.table_rows) {
      if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
      tok = 0;
    }
    xrow = p.x + tok * p.k;
  }
  const int E = p.k > ps::kMaxPerThread * kCT
                    ? ps::stage_input_wide(xrow, p.k, xd, red)
                    : ps::stage_input<false>(xrow, p.k, p.norm_w ? &nw : nullptr, p.eps, xd, red,
                                             (p.token && blockIdx.x == 0) ? p.embed_to : nullptr, nullptr);

  const int xs = ps::x_stride(p.k);
  int c4[4] = {0, 0, 0, 0};
  float ws0 = 0.f, ws1 = 0.f, wr0 = 0.f, wr1 = 0.f;  // whole mode: the tile's scales / residuals (lanes t == 0)
  int slot = 0;
  float bv = -INFINITY;  // argmax: this thread's best logit and its row
  int bi = 0x7fffffff;
  for (int j = 0; tc_item(p, ntl, j, tl, c); ++j) {
    const int64_t tile = blockIdx.x + (int64_t)G * tl;
    if (!p.whole || c == 0) c4[0] = c4[1] = c4[2] = c4[3] = 0;
    if (p.whole && c == 0 && t == 0) {  // requested at the tile's first chunk, used after its last
      ws0 = tc_scale(p, tc_row(p, tile, g));
      ws1 = tc_scale(p, tc_row(p, tile, g + 8));
      if (p.epi == EGPT_EPI_RESIDUAL) {
        wr0 = bf16_bits_to_f32(__ldcg(p.residual + tile * kTileRows + g));
        wr1 = bf16_bits_to_f32(__ldcg(p.residual + tile * kTileRows + g + 8));
      }
    }
    ps::cp_async_wait<RING - 1>();
    __syncwarp();
    const uint8_t *sl = ring + slot * kItemBytes;
    const int8_t *xb = xd + (int64_t)c * kChunkCols + g * xs + 16 * t;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int sw = 16 * ((4 * q + t) ^ ((g & 1) << 2));
      const uint4 wa = *(const uint4 *)(sl + g * kChunkCols + sw);
      const uint4 wb = *(const uint4 *)(sl + (g + 8) * kChunkCols + sw);
      uint4 xv = make_uint4(0u, 0u, 0u, 0u);
      if (g < 4) xv = *(const uint4 *)(xb + 64 * q);
      ps::mma_s8(c4, wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
      ps::mma_s8(c4, wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
    }
    __syncwarp();  // every lane is done with the slot
    int ntl2, nc2;
    if (tc_item(p, ntl, j + RING, ntl2, nc2)) tc_fill(p, blockIdx.x + (int64_t)G * ntl2, nc2, ring + slot * kItemBytes);
    ps::cp_async_commit();
    slot = slot + 1 == RING ? 0 : slot + 1;
    if (p.whole && c != p.nk - 1) continue;
    // planes 2t, 2t + 1 of rows g, g + 8 sit in lane t: lane t = 0 gathers planes 2, 3 from lane t = 1
    const int o0 = __shfl_down_sync(0xffffffffu, c4[0], 1), o1 = __shfl_down_sync(0xffffffffu, c4[1], 1);
    const int o2 = __shfl_down_sync(0xffffffffu, c4[2], 1), o3 = __shfl_down_sync(0xffffffffu, c4[3], 1);
    if (t != 0) continue;
    const long long T0 = (long long)c4[0] + ((long long)c4[1] << 8) + ((long long)o0 << 16) + ((long long)o1 << 24);
    const long long T1 = (long long)c4[2] + ((long long)c4[3] << 8) + ((long long)o2 << 16) + ((long long)o3 << 24);
    if (!p.whole) {
      part[(tl * p.nk + c) * kTileRows + g] = T0;
      part[(tl * p.nk + c) * kTileRows + g + 8] = T1;
      continue;
    }
    if (p.argmax) {
      tc_best(p, tile * kTileRows + g, T0, E, ws0, bv, bi);
      tc_best(p, tile * kTileRows + g + 8, T1, E, ws1, bv, bi);
    } else if (p.epi == EGPT_EPI_SILU_MUL) {
      tc_emit(p, tile, g, T0, T1, E, ws0, ws1, 0.f);
    } else {
      tc_emit(p, tile, g, T0, 0, E, ws0, 0.f, wr0);
      tc_emit(p, tile, g + 8, T1, 0, E, ws1, 0.f, wr1);
    }
  }
  if (!p.whole) {
    ps::csync();  // all items' sums are in `part`
    if (epi) {
      const int64_t tle = e / per_tile;
      long long T0 = 0, T1 = 0;
      for (int cc = 0; cc < p.nk; ++cc) {
        T0 += part[(tle * p.nk + cc) * kTileRows + er];
        if (p.epi == EGPT_EPI_SILU_MUL) T1 += part[(tle * p.nk + cc) * kTileRows + er + 8];
      }
      if (p.argmax)
        tc_best(p, etile * kTileRows + er, T0, E, es0, bv, bi);
      else
        tc_emit(p, etile, er, T0, T1, E, es0, es1, eres);
    }
  }
  if (p.argmax) tc_argmax_finish(p, bv, bi);
}

}  // namespace tc

// Host side (called by egpt_gemv_i8 with EGPT_FLAG_EXACT; p already validated for the general GEMV).
int gemv_tc_launch(const GemvParams &gp, cudaStream_t st) {
  if (gp.m != 1 || !gp.x_bf16 || gp.bias || (gp.flags & EGPT_FLAG_DOUBLE_ROUND))
    return set_error(EGPT_ERR_ARG, "gemv exact: one bf16 row, no bias, no double rounding");
  const bool embed = (gp.flags & EGPT_FLAG_EMBED) != 0;
  if (embed && (gp.epilogue == EGPT_EPI_RESIDUAL || gp.k > (int64_t)ps::kMaxPerThread * ps::kCT))
    return set_error(EGPT_ERR_ARG, "gemv exact: the embedding prologue takes k up to %d and no residual epilogue",
                     ps::kMaxPerThread * ps::kCT);
  if (gp.epilogue != EGPT_EPI_NONE && gp.epilogue != EGPT_EPI_RESIDUAL && gp.epilogue != EGPT_EPI_SILU_MUL)
    return set_error(EGPT_ERR_ARG, "gemv exact: epilogue must be none, residual or SiLU*up");
  if (gp.argmax && (gp.epilogue != EGPT_EPI_NONE || embed || gp.n > 0x7fffffff))
    return set_error(EGPT_ERR_ARG, "lm_head argmax exact: plain rows only");
  const int64_t n = gp.n, k = gp.k;
  if (n % 16 || k % 16) return set_error(EGPT_ERR_SHAPE, "gemv exact: n and k must be multiples of 16");
  const int64_t reg_max = (int64_t)ps::kMaxPerThread * ps::kCT;
  if (k > 2 * reg_max || ((gp.flags & EGPT_FLAG_RMSNORM) && k > reg_max))
    return set_error(EGPT_ERR_SHAPE, "gemv exact: k above %lld (%lld with the RMSNorm prologue)", (long long)(2 * reg_max),
                     (long long)reg_max);
  if ((uintptr_t)gp.w % 16 || (uintptr_t)gp.x % 16)
    return set_error(EGPT_ERR_ALIGN, "gemv exact: weights and x must be 16-byte aligned");
  tc::TcParams p{};
  p.out = (uint16_t *)gp.out;
  p.x = (const uint16_t *)gp.x;
  p.residual = (const uint16_t *)gp.residual;
  p.norm_w = (gp.flags & EGPT_FLAG_RMSNORM) ? (const uint16_t *)gp.norm_w : nullptr;
  if (embed) {
    p.token = gp.token;
    p.embed_to = (uint16_t *)gp.residual;
    p.table_rows = gp.ldx;  // embedding mode: ldx holds the table's row count
  }
  p.w = gp.w;
  p.s = gp.scale;
  p.s_bf16 = gp.scale_bf16;
  p.epi = gp.epilogue;
  if (gp.argmax) {
    p.argmax = 1;
    p.advance = (gp.flags & EGPT_FLAG_ADVANCE) != 0;
    p.tok_out = gp.tok_out;
    p.position = gp.position;
    p.logits = (uint16_t *)gp.logits;
    p.ws_val = gp.ws_val;
    p.ws_idx = gp.ws_idx;
    p.ws_counter = gp.ws_counter;
  }
  p.n = n;
  p.k = k;
  p.eps = gp.eps;
  p.tiles = n / ps::kTileRows;
  p.nk = (int)((k + ps::kChunkCols - 1) / ps::kChunkCols);
  const int sms = num_sms();
  p.whole = p.tiles >= (int64_t)ps::kNC * sms;
  const int G = (int)std::min<int64_t>(p.tiles, sms);
  const int64_t ntl = (p.tiles + G - 1) / G;
  p.part_bytes = p.whole ? 0 : (int)(ntl * p.nk * ps::kTileRows * 8);
  const size_t fixed = 256 + (size_t)p.part_bytes + 4 * (size_t)ps::x_stride(k);
  const size_t limit = smem_limit() - 1024;
  int ring = 3;
  if (fixed + (size_t)ps::kNC * ring * ps::kItemBytes > limit) ring = 2;
  const size_t smem = fixed + (size_t)ps::kNC * ring * ps::kItemBytes;
  if (smem > limit) return set_error(EGPT_ERR_SHAPE, "gemv exact: %zu bytes of shared memory needed", smem);
  p.ring = ring;
  const void *kern = ring == 3 ? (const void *)tc::gemv_tc_kernel<3> : (const void *)tc::gemv_tc_kernel<2>;
  static int configured[64][2] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev][ring - 2]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit);
    if (e != cudaSuccess) return check_launch(e, "gemv_tc_kernel");
    configured[dev][ring - 2] = 1;
  }
  return check_launch(launch_kernel(kern, dim3(G), dim3(ps::kCT), smem, st, (gp.flags & EGPT_FLAG_PDL) != 0, p),
                      "gemv_tc_kernel");
}

}  // namespace egpt
