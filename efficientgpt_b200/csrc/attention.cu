// Decode attention for B200 (sm_100a): q/k RMSNorm + RoPE + KV-cache append, and split-K GQA flash-decode
// with the log-sum-exp combine done by the last CTA of each kv head (no second launch).
//
// Reference behaviour (BagelsFun/efficientgpt, via transformers' Qwen3Attention, modeling_qwen3.py:258-291):
//   q = RoPE(q_norm(q_proj(x))), k = RoPE(k_norm(k_proj(x))), cache[pos] = (k, v),
//   out = SDPA(q, K[0..pos], V[0..pos], scale = d^-0.5) with GQA (q head h reads kv head h / group).
// Rounding points follow HF eager bf16: RMSNorm rounds x*rsqrt to bf16 then the weight product to bf16;
// RoPE rounds q*cos, rotate_half(q)*sin and their sum to bf16; the cos/sin table is HF's own bf16 table.
// Softmax runs in fp32 (online softmax); for bf16 caches the probabilities enter P.V rounded to bf16 (as in
// the SDPA kernels the reference runs: PyTorch's CPU flash attention and the GPU memory-efficient kernel)
// while the denominator sums fp32 values; the output is rounded once to the activation dtype.
//
// Layout: caches are [nkv][cap][d] per layer, so the keys of one head are one contiguous stream.
// Work split: grid (nkv, max_split, rows). A CTA owns one kv head, all `group` q heads that read it (K/V
// are read once per group) and one key range. Each warp processes 32 keys per step: lane l holds dims
// [l*d/32, (l+1)*d/32) of every key, so K/V rows are read fully coalesced; the 32 partial dot products
// per head are reduced with a transpose-butterfly that leaves lane j holding key j's score.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace egpt {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kKeysPerSplitTarget = 128;

struct AttnParams {
  void *out;
  int64_t ldo;
  const void *q;  // raw qkv rows (APPEND) or rotated q rows
  int64_t ldq;
  void *k_cache, *v_cache;
  int64_t cap;
  const int64_t *position;
  int64_t m;
  int nq, nkv, d, group;
  const void *q_norm_w, *k_norm_w;
  float eps;
  const void *rope_cos, *rope_sin;
  float scale;
  int max_split;
  float *ws_f;
  unsigned *ws_cnt;
  unsigned flags;
};

// ---------------------------------------------------------------------------------------------- head prologue
// Normalise (optional) and rotate (optional) one head vector of length d held as bf16 at `src`; the result
// (bf16-rounded) goes to dst_f (fp32, smem) and, when dst_bf16 is non-null, to global memory as bf16.
// Must be called by the whole block (blockDim >= d); `tmp` holds d floats, `red` 32 floats.
__device__ void head_norm_rope(const uint16_t *src, const void *norm_w, float eps, const void *rope_cos,
                               const void *rope_sin, int64_t pos, int d, float *dst_f, uint16_t *dst_bf16,
                               float *tmp, float *red) {
  const int t = threadIdx.x;
  float v = t < d ? bf16_bits_to_f32(src[t]) : 0.f;
  if (norm_w) {
    const float ss = block_sum(v * v, red);
    const float inv = rsqrtf(ss / (float)d + eps);
    if (t < d) v = round_bf16(round_bf16(v * inv) * bf16_bits_to_f32(((const uint16_t *)norm_w)[t]));
  }
  if (rope_cos) {
    if (t < d) tmp[t] = v;
    __syncthreads();
    if (t < d) {
      const int half = d / 2;
      const int i = t < half ? t : t - half;
      const float c = bf16_bits_to_f32(((const uint16_t *)rope_cos)[pos * half + i]);
      const float s = bf16_bits_to_f32(((const uint16_t *)rope_sin)[pos * half + i]);
      const float rot = t < half ? -tmp[t + half] : tmp[t - half];
      v = round_bf16(round_bf16(v * c) + round_bf16(rot * s));
    }
    __syncthreads();
  }
  if (t < d) {
    dst_f[t] = v;
    if (dst_bf16) dst_bf16[t] = f32_to_bf16_bits(v);
  }
}

// ---------------------------------------------------------------------------------------------- append kernel
// grid (m, nq + 2 nkv), block >= d threads: one head vector per CTA.
__global__ void qk_norm_rope_append_kernel(AttnParams p, int is_bf16) {
  __shared__ float tmp[1024];
  __shared__ float red[32];
  __shared__ float outf[1024];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int head = blockIdx.y;
  const int64_t pos = *p.position + row;
  const int d = p.d;
  if (pos >= p.cap || pos < 0) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return;
  }
  if (is_bf16) {
    const uint16_t *src = (const uint16_t *)p.q + row * p.ldq + (int64_t)head * d;
    if (head < p.nq) {
      uint16_t *dst = (uint16_t *)p.out + row * p.ldo + (int64_t)head * d;
      head_norm_rope(src, p.q_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, d, outf, dst, tmp, red);
    } else if (head < p.nq + p.nkv) {
      const int g = head - p.nq;
      uint16_t *dst = (uint16_t *)p.k_cache + ((int64_t)g * p.cap + pos) * d;
      head_norm_rope(src, p.k_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, d, outf, dst, tmp, red);
    } else {
      const int g = head - p.nq - p.nkv;
      uint16_t *dst = (uint16_t *)p.v_cache + ((int64_t)g * p.cap + pos) * d;
      for (int t = threadIdx.x; t < d; t += blockDim.x) dst[t] = src[t];
    }
  } else {  // fp32 (nanoGPT): no norm, no RoPE, plain copies
    const float *src = (const float *)p.q + row * p.ldq + (int64_t)head * d;
    float *dst;
    if (head < p.nq)
      dst = (float *)p.out + row * p.ldo + (int64_t)head * d;
    else if (head < p.nq + p.nkv)
      dst = (float *)p.k_cache + ((int64_t)(head - p.nq) * p.cap + pos) * d;
    else
      dst = (float *)p.v_cache + ((int64_t)(head - p.nq - p.nkv) * p.cap + pos) * d;
    for (int t = threadIdx.x; t < d; t += blockDim.x) dst[t] = src[t];
  }
}

// ---------------------------------------------------------------------------------------------- split kernel
template <bool BF16>
__device__ __forceinline__ void load_dims(const void *base, int64_t elem_off, float (&v)[4], int dpl) {
  if (BF16) {
    const uint16_t *b = (const uint16_t *)base + elem_off;
    if (dpl == 4) {
      const uint2 u = *(const uint2 *)b;
      v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
    } else if (dpl == 2) {
      const uint32_t u = *(const uint32_t *)b;
      v[0] = bf16_lo(u); v[1] = bf16_hi(u);
    } else {
      v[0] = bf16_bits_to_f32(b[0]);
    }
  } else {
    const float *b = (const float *)base + elem_off;
    if (dpl == 4) {
      const float4 u = *(const float4 *)b;
      v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
    } else if (dpl == 2) {
      const float2 u = *(const float2 *)b;
      v[0] = u.x; v[1] = u.y;
    } else {
      v[0] = b[0];
    }
  }
}

// Transpose-butterfly: on entry lane l holds s[j] = partial for key j (j < 32) from its dims; on exit the
// return value of lane l is the full sum over lanes for key l. 31 shuffles for 32 keys, fixed order.
__device__ __forceinline__ float transpose_reduce32(float (&s)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      // keep half of the keys: lanes with bit w set keep keys [w, 2w) of each 2w block, others [0, w)
      const float send = upper ? s[j] : s[j + w];
      const float keep = upper ? s[j + w] : s[j];
      s[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return s[0];
}

template <int DPL, int GRP, bool BF16>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnParams p) {
  constexpr int D = DPL * 32;
  __shared__ float q_s[GRP][D];
  __shared__ float tmp[D];
  __shared__ float red[32];
  __shared__ float w_m[kAttnWarps][GRP], w_l[kAttnWarps][GRP];
  __shared__ float w_acc[kAttnWarps][GRP][D];
  __shared__ int s_last;

  pdl_wait();
  pdl_launch_dependents();

  const int g = blockIdx.x, split = blockIdx.y;
  const int64_t row = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t pos = *p.position + row;
  const int64_t L = pos + 1;
  if (L > p.cap || pos < 0) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return;
  }
  int nsplit = (int)((L + kKeysPerSplitTarget - 1) / kKeysPerSplitTarget);
  nsplit = nsplit < 1 ? 1 : (nsplit > p.max_split ? p.max_split : nsplit);
  if (split >= nsplit) return;
  const int64_t chunk = (L + nsplit - 1) / nsplit;
  const int64_t k0 = split * chunk;
  const int64_t k1 = min(L, k0 + chunk);

  const int64_t kv_base = (int64_t)g * p.cap * D;
  // ---- q (and, with APPEND, this step's k/v) ----
  if (p.flags & EGPT_FLAG_APPEND) {
    const uint16_t *qkv = (const uint16_t *)p.q + row * p.ldq;
    for (int j = 0; j < GRP; ++j)
      head_norm_rope(qkv + (int64_t)(g * GRP + j) * D, p.q_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, D, q_s[j],
                     nullptr, tmp, red);
    if (pos >= k0 && pos < k1) {  // this CTA's range holds the new slot: write it before reading the range
      uint16_t *kd = (uint16_t *)p.k_cache + kv_base + pos * D;
      head_norm_rope(qkv + (int64_t)(p.nq + g) * D, p.k_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, D, tmp, kd,
                     w_acc[0][0], red);
      const uint16_t *vs = qkv + (int64_t)(p.nq + p.nkv + g) * D;
      uint16_t *vd = (uint16_t *)p.v_cache + kv_base + pos * D;
      for (int t = threadIdx.x; t < D; t += blockDim.x) vd[t] = vs[t];
    }
  } else {
    for (int j = 0; j < GRP; ++j)
      for (int t = threadIdx.x; t < D; t += blockDim.x)
        q_s[j][t] = BF16 ? bf16_bits_to_f32(((const uint16_t *)p.q)[row * p.ldq + (int64_t)(g * GRP + j) * D + t])
                         : ((const float *)p.q)[row * p.ldq + (int64_t)(g * GRP + j) * D + t];
  }
  __syncthreads();

  // ---- per-warp online softmax over 32-key tiles ----
  float qv[GRP][DPL];
#pragma unroll
  for (int j = 0; j < GRP; ++j)
#pragma unroll
    for (int e = 0; e < DPL; ++e) qv[j][e] = q_s[j][lane * DPL + e];
  float m_run[GRP], l_run[GRP], acc[GRP][DPL];
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[j][e] = 0.f;
  }
  const void *K = p.k_cache, *V = p.v_cache;
  for (int64_t t0 = k0 + (int64_t)warp * 32; t0 < k1; t0 += 32 * kAttnWarps) {
    const int nkeys = (int)min((int64_t)32, k1 - t0);
    float sc[GRP];
    {
      float part[GRP][32];
#pragma unroll
      for (int kk = 0; kk < 32; ++kk) {
        float kv[4] = {0.f, 0.f, 0.f, 0.f};
        if (kk < nkeys) load_dims<BF16>(K, kv_base + (t0 + kk) * D + lane * DPL, kv, DPL);
#pragma unroll
        for (int j = 0; j < GRP; ++j) {
          float s = 0.f;
#pragma unroll
          for (int e = 0; e < DPL; ++e) s = fmaf(qv[j][e], kv[e], s);
          part[j][kk] = s;
        }
      }
#pragma unroll
      for (int j = 0; j < GRP; ++j) sc[j] = transpose_reduce32(part[j]) * p.scale;
    }
    // lane l now holds the score of key t0 + l for each head
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      const float s = lane < nkeys ? sc[j] : -INFINITY;
      const float tmax = warp_max(s);
      const float m_new = fmaxf(m_run[j], tmax);
      const float alpha = expf(m_run[j] - m_new);
      const float pj = lane < nkeys ? expf(s - m_new) : 0.f;
      l_run[j] = l_run[j] * alpha + warp_sum(pj);
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[j][e] *= alpha;
      m_run[j] = m_new;
      sc[j] = pj;
    }
    for (int kk = 0; kk < nkeys; ++kk) {
      float vv[4] = {0.f, 0.f, 0.f, 0.f};
      load_dims<BF16>(V, kv_base + (t0 + kk) * D + lane * DPL, vv, DPL);
#pragma unroll
      for (int j = 0; j < GRP; ++j) {
        // bf16 inputs: probabilities enter P.V rounded to bf16 (the SDPA kernels' rounding point), while
        // the denominator l sums the fp32 values.
        const float p32 = __shfl_sync(0xffffffffu, sc[j], kk);
        const float pk = BF16 ? round_bf16(p32) : p32;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[j][e] = fmaf(pk, vv[e], acc[j][e]);
      }
    }
  }
  // ---- merge the warps (fixed order) ----
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    if (lane == 0) {
      w_m[warp][j] = m_run[j];
      w_l[warp][j] = l_run[j];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) w_acc[warp][j][lane * DPL + e] = acc[j][e];
  }
  __syncthreads();
  const bool single = nsplit == 1;
  for (int idx = threadIdx.x; idx < GRP * D; idx += blockDim.x) {
    const int j = idx / D, dd = idx - j * D;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, w_m[w][j]);
    float lsum = 0.f, a = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      if (w_l[w][j] == 0.f) continue;
      const float f = expf(w_m[w][j] - M);
      lsum += w_l[w][j] * f;
      a += w_acc[w][j][dd] * f;
    }
    const int h = g * GRP + j;
    if (single) {
      const float o = a / lsum;
      if (BF16)
        ((uint16_t *)p.out)[row * p.ldo + (int64_t)h * D + dd] = f32_to_bf16_bits(o);
      else
        ((float *)p.out)[row * p.ldo + (int64_t)h * D + dd] = o;
    } else {
      float *slot = p.ws_f + (((row * p.nq + h) * p.max_split) + split) * (D + 2);
      slot[2 + dd] = a;
      if (dd == 0) {
        slot[0] = M;
        slot[1] = lsum;
      }
    }
  }
  if (single) return;
  // ---- last CTA of this (row, kv head) combines the splits ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *cnt = p.ws_cnt + row * p.nkv + g;
    const unsigned prev = atomicAdd(cnt, 1u);
    s_last = prev == (unsigned)(nsplit - 1);
    if (s_last) *cnt = 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < GRP * D; idx += blockDim.x) {
    const int j = idx / D, dd = idx - j * D;
    const int h = g * GRP + j;
    const float *base = p.ws_f + ((row * p.nq + h) * p.max_split) * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(base + s * (D + 2)));
    float lsum = 0.f, a = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ls = __ldcg(base + s * (D + 2) + 1);
      if (ls == 0.f) continue;
      const float f = expf(__ldcg(base + s * (D + 2)) - M);
      lsum += ls * f;
      a += __ldcg(base + s * (D + 2) + 2 + dd) * f;
    }
    const float o = a / lsum;
    if (BF16)
      ((uint16_t *)p.out)[row * p.ldo + (int64_t)h * D + dd] = f32_to_bf16_bits(o);
    else
      ((float *)p.out)[row * p.ldo + (int64_t)h * D + dd] = o;
  }
}

template <int DPL, bool BF16>
static cudaError_t launch_split_grp(const AttnParams &p, dim3 grid, cudaStream_t st, bool pdl) {
  switch (p.group) {
    case 1: return launch_kernel((const void *)attn_split_kernel<DPL, 1, BF16>, grid, dim3(kAttnThreads), 0, st, pdl, p);
    case 2: return launch_kernel((const void *)attn_split_kernel<DPL, 2, BF16>, grid, dim3(kAttnThreads), 0, st, pdl, p);
    default: return launch_kernel((const void *)attn_split_kernel<DPL, 4, BF16>, grid, dim3(kAttnThreads), 0, st, pdl, p);
  }
}

}  // namespace egpt

using namespace egpt;

static int check_heads(int nq, int nkv, int d) {
  if (nq < 1 || nkv < 1 || nq % nkv) return set_error(EGPT_ERR_SHAPE, "attention: nq must be a multiple of nkv");
  const int grp = nq / nkv;
  if (grp != 1 && grp != 2 && grp != 4) return set_error(EGPT_ERR_SHAPE, "attention: group size must be 1, 2 or 4");
  if (d != 32 && d != 64 && d != 128) return set_error(EGPT_ERR_SHAPE, "attention: head_dim must be 32, 64 or 128");
  return EGPT_OK;
}

extern "C" int egpt_qk_norm_rope_kv_append(void *q_out, const void *qkv, int64_t ldqkv, void *k_cache, void *v_cache,
                                           int64_t cap, const int64_t *position, int64_t m, int nq, int nkv, int d,
                                           const void *q_norm_w, const void *k_norm_w, float eps,
                                           const void *rope_cos, const void *rope_sin, int dtype, void *stream) {
  clear_error();
  if (!q_out || !qkv || !k_cache || !v_cache || !position) return set_error(EGPT_ERR_ARG, "append: null pointer");
  if (int rc = check_heads(nq, nkv, d)) return rc;
  if (m < 1 || m > 65535 || cap < 1) return set_error(EGPT_ERR_SHAPE, "append: bad m or cap");
  if (ldqkv < (int64_t)(nq + 2 * nkv) * d) return set_error(EGPT_ERR_SHAPE, "append: ldqkv too small");
  if (dtype != EGPT_BF16 && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "append: dtype");
  if (dtype == EGPT_F32 && (q_norm_w || k_norm_w || rope_cos)) return set_error(EGPT_ERR_DTYPE, "append: fp32 has no norm/RoPE");
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return set_error(EGPT_ERR_ARG, "append: rope_cos/rope_sin");
  AttnParams p{};
  p.out = q_out;
  p.ldo = (int64_t)nq * d;
  p.q = qkv;
  p.ldq = ldqkv;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.cap = cap;
  p.position = position;
  p.m = m;
  p.nq = nq;
  p.nkv = nkv;
  p.d = d;
  p.group = nq / nkv;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.eps = eps;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  const int threads = d < 32 ? 32 : d;
  return check_launch(launch_kernel((const void *)qk_norm_rope_append_kernel, dim3((unsigned)m, nq + 2 * nkv),
                                    dim3(threads), 0, (cudaStream_t)stream, false, p, (int)(dtype == EGPT_BF16)),
                      "qk_norm_rope_append_kernel");
}

extern "C" size_t egpt_attn_ws_bytes(int64_t m, int nq, int nkv, int d, int max_split) {
  const size_t floats = (size_t)m * nq * max_split * (d + 2);
  const size_t fbytes = (floats * 4 + 255) / 256 * 256;
  return fbytes + (size_t)m * nkv * 4;
}

extern "C" int egpt_attn_decode(void *out, int64_t ldo, const void *q, int64_t ldq, void *k_cache, void *v_cache,
                                int64_t cap, const int64_t *position, int64_t m, int nq, int nkv, int d,
                                const void *q_norm_w, const void *k_norm_w, float eps, const void *rope_cos,
                                const void *rope_sin, float scale, int max_split, void *ws, size_t ws_bytes, int dtype,
                                unsigned flags, void *stream) {
  clear_error();
  if (!out || !q || !k_cache || !v_cache || !position) return set_error(EGPT_ERR_ARG, "attn: null pointer");
  if (int rc = check_heads(nq, nkv, d)) return rc;
  if (m < 1 || m > 65535 || cap < 1) return set_error(EGPT_ERR_SHAPE, "attn: bad m or cap");
  if (max_split < 1 || max_split > 1024) return set_error(EGPT_ERR_SHAPE, "attn: max_split must be in [1, 1024]");
  if (dtype != EGPT_BF16 && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "attn: dtype");
  if ((flags & EGPT_FLAG_APPEND) && (m != 1 || dtype != EGPT_BF16))
    return set_error(EGPT_ERR_ARG, "attn: fused append needs m == 1 and bf16");
  if ((flags & EGPT_FLAG_APPEND) && ldq < (int64_t)(nq + 2 * nkv) * d) return set_error(EGPT_ERR_SHAPE, "attn: ldq too small for qkv rows");
  if (!(flags & EGPT_FLAG_APPEND) && ldq < (int64_t)nq * d) return set_error(EGPT_ERR_SHAPE, "attn: ldq too small");
  if (ldo < (int64_t)nq * d) return set_error(EGPT_ERR_SHAPE, "attn: ldo too small");
  if (max_split > 1 && (!ws || ws_bytes < egpt_attn_ws_bytes(m, nq, nkv, d, max_split)))
    return set_error(EGPT_ERR_WORKSPACE, "attn: workspace too small");
  const int esz = dtype == EGPT_BF16 ? 2 : 4;
  if (((uintptr_t)k_cache | (uintptr_t)v_cache) % 16 || ((int64_t)d * esz) % 16)
    return set_error(EGPT_ERR_ALIGN, "attn: caches must be 16-byte aligned");
  AttnParams p{};
  p.out = out;
  p.ldo = ldo;
  p.q = q;
  p.ldq = ldq;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.cap = cap;
  p.position = position;
  p.m = m;
  p.nq = nq;
  p.nkv = nkv;
  p.d = d;
  p.group = nq / nkv;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.eps = eps;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.scale = scale;
  p.max_split = max_split;
  p.ws_f = (float *)ws;
  p.ws_cnt = ws ? (unsigned *)((char *)ws + (egpt_attn_ws_bytes(m, nq, nkv, d, max_split) - (size_t)m * nkv * 4)) : nullptr;
  p.flags = flags;
  const dim3 grid(nkv, max_split, (unsigned)m);
  const bool pdl = (flags & EGPT_FLAG_PDL) != 0;
  cudaError_t e;
  const bool bf = dtype == EGPT_BF16;
  if (d == 128)
    e = bf ? launch_split_grp<4, true>(p, grid, (cudaStream_t)stream, pdl) : launch_split_grp<4, false>(p, grid, (cudaStream_t)stream, pdl);
  else if (d == 64)
    e = bf ? launch_split_grp<2, true>(p, grid, (cudaStream_t)stream, pdl) : launch_split_grp<2, false>(p, grid, (cudaStream_t)stream, pdl);
  else
    e = bf ? launch_split_grp<1, true>(p, grid, (cudaStream_t)stream, pdl) : launch_split_grp<1, false>(p, grid, (cudaStream_t)stream, pdl);
  return check_launch(e, "attn_split_kernel");
}
