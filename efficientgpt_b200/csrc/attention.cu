// Decode attention for B200 (sm_100a): q/k RMSNorm + RoPE + KV-cache append, and split-K GQA flash-decode
// with the log-sum-exp combine done by the last CTA of each kv head (no second launch).
//
// Reference behaviour (BagelsFun/efficientgpt, via transformers' Qwen3Attention, modeling_qwen3.py:258-291):
//   q = RoPE(q_norm(q_proj(x))), k = RoPE(k_norm(k_proj(x))), cache[pos] = (k, v),
//   out = SDPA(q, K[0..pos], V[0..pos], scale = d^-0.5) with GQA (q head h reads kv head h / group).
// Rounding points follow HF eager bf16: RMSNorm rounds x*rsqrt to bf16 then the weight product to bf16;
// RoPE rounds q*cos, rotate_half(q)*sin and their sum to bf16; the cos/sin table is HF's own bf16 table.
// Softmax runs in fp32. For bf16 caches the probabilities enter P.V rounded to bf16 while the denominator
// sums fp32 values, and the reference point of that rounding follows the SDPA kernel the reference runs on the
// GPU (fmha_cutlassF_bf16_aligned_64x128_rf_sm80, named by the reference's own profile of this path): it walks
// the cache in 128-key blocks with a running maximum, so the keys of block j are rounded relative to the
// maximum score over blocks 0..j. The output is rounded once to the activation dtype.
//
// Layout: caches are [nkv][cap][d] per layer, so the keys of one head are one contiguous stream.
// Work split: grid (nkv, max_split, rows). A CTA owns one kv head, all `group` q heads that read it (K/V
// are read once per group) and one range of whole 128-key blocks. Each warp processes 32 keys per step: for the
// scores lane l reads key l's row in 16-byte pieces and dots it with the q heads in shared memory; for P.V each
// half-warp reads whole value rows (lane l holds d/16 dims), the halves take even and odd keys, 8 independent
// row loads per batch.
// Pass A scores the range into shared memory (and prefetches the V rows into L2), the block maxima give the
// running maximum of every block, pass B accumulates bf16(p) V per warp; warps merge in a fixed order and
// split ranges combine by log-sum-exp in the last CTA of each kv head. The running maximum of the blocks
// before the range comes from rescoring the keys [0, k0) (EGPT_FLAG_REF_SOFTMAX) or, in the persistent decode
// step, from the other ranges through global memory; without the flag a range starts its own walk.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace egpt {

constexpr int kAttnThreads = 256;  // 8 warps walk the key tiles
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kRefBlock = 128;     // keys per softmax block of the reference's GPU SDPA kernel
constexpr int kKeyTile = 32;       // keys per warp step

// Keys per split range whose scores fit the scratch ([group][keys] fp32 = 8 KB).
__host__ __device__ constexpr int split_keys_max(int grp) { return 2048 / grp; }
// Blocks per split range: ranges are whole 128-key blocks, at most max_split of them, and at least
// kMinSplitBlocks blocks each: below that a range's keys cost less time than the exchange and combine that a
// second range brings.
constexpr int kMinSplitBlocks = 4;
__host__ __device__ inline int split_blocks(int64_t L, int max_split, int min_blocks = kMinSplitBlocks) {
  const int64_t nb = (L + kRefBlock - 1) / kRefBlock;
  const int64_t b = (nb + max_split - 1) / max_split;
  return (int)(b > min_blocks ? b : min_blocks);
}
// The per-op kernel's ranges may be single blocks: each range is its own CTA, so short contexts spread over more SMs.
constexpr int kMinSplitBlocksOp = 1;
__host__ __device__ inline int split_count(int64_t L, int bps) {
  const int64_t nb = (L + kRefBlock - 1) / kRefBlock;
  return (int)((nb + bps - 1) / bps);
}

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
  int max_split;  // workspace layout: partial slots per (row, head)
  int split_cap;  // ranges actually used (<= max_split): about two CTAs per SM over the grid
  float *ws_f;
  unsigned *ws_cnt;
  unsigned flags;
};

// Rows of one sequence (row i at *position + i, one cache) or, with EGPT_FLAG_RAGGED, m sequences (row i at
// position[i], its own cache: heads [i nkv, (i + 1) nkv) of caches laid out [m nkv][cap][d]).
__device__ __forceinline__ int64_t row_pos(const AttnParams &p, int64_t row) {
  return (p.flags & EGPT_FLAG_RAGGED) ? p.position[row] : *p.position + row;
}
__device__ __forceinline__ int64_t row_kv_head(const AttnParams &p, int64_t row, int g) {
  return (p.flags & EGPT_FLAG_RAGGED) ? row * p.nkv + g : g;
}

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
  const int64_t pos = row_pos(p, row);
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
      const int64_t g = row_kv_head(p, row, head - p.nq);
      uint16_t *dst = (uint16_t *)p.k_cache + (g * p.cap + pos) * d;
      head_norm_rope(src, p.k_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, d, outf, dst, tmp, red);
    } else {
      const int64_t g = row_kv_head(p, row, head - p.nq - p.nkv);
      uint16_t *dst = (uint16_t *)p.v_cache + (g * p.cap + pos) * d;
      for (int t = threadIdx.x; t < d; t += blockDim.x) dst[t] = src[t];
    }
  } else {  // fp32 (nanoGPT): no norm, no RoPE, plain copies
    const float *src = (const float *)p.q + row * p.ldq + (int64_t)head * d;
    float *dst;
    if (head < p.nq)
      dst = (float *)p.out + row * p.ldo + (int64_t)head * d;
    else if (head < p.nq + p.nkv)
      dst = (float *)p.k_cache + (row_kv_head(p, row, head - p.nq) * p.cap + pos) * d;
    else
      dst = (float *)p.v_cache + (row_kv_head(p, row, head - p.nq - p.nkv) * p.cap + pos) * d;
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

// ---------------------------------------------------------------------------------------------- core
// Shared-memory scratch of one attention task (one kv head, its q heads, one key range).
template <int DPL, int GRP>
struct AttnScratch {
  static constexpr int D = DPL * 32;
  static constexpr int KS = split_keys_max(GRP);
  float q[GRP][D];                        // rotated q heads (fp32 values of bf16 numbers)
  float sc[GRP][KS];                      // scores of the range
  float tmax[KS / kKeyTile][GRP];         // per-tile maxima
  float pref[KS / kRefBlock][GRP];        // running maximum of each block of the range
  float mb[GRP];                          // running maximum before the range (-inf: none)
  float w_m[kAttnWarps][GRP], w_l[kAttnWarps][GRP];
  float w_acc[kAttnWarps][GRP][D];
  int flag;
};

template <int NT>
__device__ __forceinline__ void nt_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

struct AttnTask {
  const void *K, *V;  // this kv head's [cap][D] cache rows (global memory, or copies in shared memory)
  int64_t k0, k1;     // key range [k0, k1), k0 a multiple of kRefBlock
  float scale;
  int prefetch_v;     // V in global memory: pass A prefetches the range's V rows into L2
};

// HD consecutive elements of a cache row, kept raw (bf16: 4, 8 or 16 bytes; fp32: 8, 16 or 32 bytes) until
// unpacked to fp32; a row that is not loaded unpacks to zeros.
template <bool BF16, int HD>
struct RawRow {
  static constexpr int W = HD * (BF16 ? 2 : 4) / 4;  // 32-bit words
  uint32_t w[W];
  __device__ __forceinline__ void load(const void *base, int64_t elem_off, bool valid) {
    const char *b = (const char *)base + elem_off * (BF16 ? 2 : 4);
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = 0u;
    if (!valid) return;
    if (W % 4 == 0) {
#pragma unroll
      for (int i = 0; i < W; i += 4) {
        const uint4 u = *(const uint4 *)(b + 4 * i);
        w[i] = u.x, w[(i + 1) % W] = u.y, w[(i + 2) % W] = u.z, w[(i + 3) % W] = u.w;
      }
    } else if (W % 2 == 0) {
#pragma unroll
      for (int i = 0; i < W; i += 2) {
        const uint2 u = *(const uint2 *)(b + 4 * i);
        w[i] = u.x, w[(i + 1) % W] = u.y;
      }
    } else {
      w[0] = *(const uint32_t *)b;
    }
  }
  __device__ __forceinline__ void unpack(float (&v)[HD]) const {
#pragma unroll
    for (int i = 0; i < W; ++i) {
      if (BF16) {
        v[(2 * i) % HD] = bf16_lo(w[i]);
        v[(2 * i + 1) % HD] = bf16_hi(w[i]);
      } else {
        v[i % HD] = __uint_as_float(w[i]);
      }
    }
  }
};

// Scores of keys t0 .. t0 + nkeys - 1 (nkeys <= 32) for every head of the group: lane l reads key t0 + l's row
// in 16-byte pieces (batches of 8 independent loads), starting at piece l mod 8 and wrapping around, so that the
// eight lanes of a shared-memory phase read eight different bank groups when the rows sit in shared memory, and
// dots it with each q head from shared memory, four partial sums per head (dims d = m mod 4, in the lane's piece
// order); lane l returns key t0 + l's scores (0 for lanes past nkeys).
template <int DPL, int GRP, bool BF16>
__device__ __forceinline__ void tile_scores(const void *K, int64_t t0, int nkeys, const AttnScratch<DPL, GRP> &S,
                                            float scale, float (&sc)[GRP]) {
  constexpr int D = DPL * 32;
  constexpr int ESZ = BF16 ? 2 : 4;
  constexpr int EPP = 16 / ESZ;          // elements per 16-byte piece
  constexpr int NP = D * ESZ / 16;       // pieces per row
  constexpr int NB = NP < 8 ? NP : 8;    // pieces per batch
  const int lane = threadIdx.x & 31;
  float acc[GRP][4];
#pragma unroll
  for (int j = 0; j < GRP; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  if (lane < nkeys) {
    const uint4 *row = (const uint4 *)((const char *)K + (t0 + lane) * (int64_t)D * ESZ);
    const int rot = lane & 7;
#pragma unroll 1
    for (int pb = 0; pb < NP; pb += NB) {
      uint4 w[NB];
#pragma unroll
      for (int u = 0; u < NB; ++u) w[u] = row[(pb + u + rot) & (NP - 1)];
#pragma unroll
      for (int u = 0; u < NB; ++u) {
        float kv[EPP];
        if (BF16) {
          const uint32_t x[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
          for (int h = 0; h < 4; ++h) kv[2 * h] = bf16_lo(x[h]), kv[2 * h + 1] = bf16_hi(x[h]);
        } else {
          kv[0] = __uint_as_float(w[u].x), kv[1] = __uint_as_float(w[u].y);
          kv[2] = __uint_as_float(w[u].z), kv[3] = __uint_as_float(w[u].w);
        }
        const int d0 = ((pb + u + rot) & (NP - 1)) * EPP;
#pragma unroll
        for (int j = 0; j < GRP; ++j) {
#pragma unroll
          for (int e = 0; e < EPP; e += 4) {
            const float4 qq = *(const float4 *)&S.q[j][d0 + e];
            acc[j][0] = fmaf(qq.x, kv[e], acc[j][0]);
            acc[j][1] = fmaf(qq.y, kv[e + 1], acc[j][1]);
            acc[j][2] = fmaf(qq.z, kv[e + 2], acc[j][2]);
            acc[j][3] = fmaf(qq.w, kv[e + 3], acc[j][3]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < GRP; ++j) sc[j] = ((acc[j][0] + acc[j][1]) + (acc[j][2] + acc[j][3])) * scale;
}

// Pass A: scores of the range into S.sc, tile maxima into S.tmax, V rows of the range prefetched into L2.
// Needs S.q; the caller synchronises afterwards.
template <int DPL, int GRP, bool BF16>
__device__ void attn_pass_a(const AttnTask &t, AttnScratch<DPL, GRP> &S) {
  constexpr int D = DPL * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp >= kAttnWarps) return;
  const int ntiles = (int)((t.k1 - t.k0 + kKeyTile - 1) / kKeyTile);
  for (int ti = warp; ti < ntiles; ti += kAttnWarps) {
    const int64_t t0 = t.k0 + (int64_t)ti * kKeyTile;
    const int nkeys = (int)min((int64_t)kKeyTile, t.k1 - t0);
    if (t.prefetch_v && lane < nkeys) {
      const char *vr = (const char *)t.V + (t0 + lane) * D * (BF16 ? 2 : 4);
#pragma unroll
      for (int off = 0; off < D * (BF16 ? 2 : 4); off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(vr + off));
    }
    float sc[GRP];
    tile_scores<DPL, GRP, BF16>(t.K, t0, nkeys, S, t.scale, sc);
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      const float sj = lane < nkeys ? sc[j] : -INFINITY;
      if (lane < nkeys) S.sc[j][ti * kKeyTile + lane] = sj;
      const float mx = warp_max(sj);
      if (lane == 0) S.tmax[ti][j] = mx;
    }
  }
}

// Running maximum before the range by rescoring keys [0, k0) into S.mb (uses S.w_m; synchronises inside).
template <int DPL, int GRP, bool BF16, int NT>
__device__ void attn_max_before(const AttnTask &t, AttnScratch<DPL, GRP> &S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp < kAttnWarps) {
    float run[GRP];
#pragma unroll
    for (int j = 0; j < GRP; ++j) run[j] = -INFINITY;
    for (int64_t t0 = (int64_t)warp * kKeyTile; t0 < t.k0; t0 += kKeyTile * kAttnWarps) {
      const int nkeys = (int)min((int64_t)kKeyTile, t.k0 - t0);
      float sc[GRP];
      tile_scores<DPL, GRP, BF16>(t.K, t0, nkeys, S, t.scale, sc);
#pragma unroll
      for (int j = 0; j < GRP; ++j) run[j] = fmaxf(run[j], warp_max(lane < nkeys ? sc[j] : -INFINITY));
    }
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < GRP; ++j) S.w_m[warp][j] = run[j];
  }
  nt_sync<NT>();
  if (threadIdx.x < GRP) {
    float m = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) m = fmaxf(m, S.w_m[w][threadIdx.x]);
    S.mb[threadIdx.x] = m;
  }
}

// Walk the range in chunks of at most KS keys: pass A scores each chunk (SCORED: the caller already ran pass A
// on a range of one chunk), the block maxima extend the running maximum (S.mb on entry: the running
// maximum before the range), then pass B accumulates per warp sum_k bf16(exp(s_k - m_block)) V_k and
// sum_k exp(s_k - m_block), rescaled in fp32 whenever a block raises the maximum. Tile i of the range is
// walked by warp i % 8 in increasing order whatever the chunking. Warp partials end in S.w_*.
template <int DPL, int GRP, bool BF16, int NT, bool SCORED>
__device__ void attn_walk(const AttnTask &t, AttnScratch<DPL, GRP> &S) {
  constexpr int D = DPL * 32;
  constexpr int KS = AttnScratch<DPL, GRP>::KS;
  constexpr int TPB = kRefBlock / kKeyTile;  // tiles per block
  constexpr int HD = 2 * DPL;  // dims per lane: each half-warp covers a whole row, the halves take even / odd keys
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane >> 4;
  float m_run[GRP], l_run[GRP], acc[GRP][HD];
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.f;
#pragma unroll
    for (int e = 0; e < HD; ++e) acc[j][e] = 0.f;
  }
  for (int64_t c0 = t.k0; c0 < t.k1; c0 += KS) {
    AttnTask c = t;
    c.k0 = c0;
    c.k1 = min(t.k1, c0 + (int64_t)KS);
    if (!SCORED) {
      nt_sync<NT>();  // the previous chunk's scores are consumed
      attn_pass_a<DPL, GRP, BF16>(c, S);
    }
    const int ntiles = (int)((c.k1 - c.k0 + kKeyTile - 1) / kKeyTile);
    nt_sync<NT>();
    if (threadIdx.x < GRP) {
      const int j = threadIdx.x;
      const int nblk = (ntiles + TPB - 1) / TPB;
      float run = S.mb[j];
      for (int b = 0; b < nblk; ++b) {
        for (int tt = b * TPB; tt < min((b + 1) * TPB, ntiles); ++tt) run = fmaxf(run, S.tmax[tt][j]);
        S.pref[b][j] = run;
      }
      S.mb[j] = run;  // running maximum before the next chunk
    }
    nt_sync<NT>();
    if (warp >= kAttnWarps) continue;
    for (int ti = warp; ti < ntiles; ti += kAttnWarps) {
      const int64_t t0 = c.k0 + (int64_t)ti * kKeyTile;
      const int nkeys = (int)min((int64_t)kKeyTile, c.k1 - t0);
      const int b = ti / TPB;
      float pj[GRP];
#pragma unroll
      for (int j = 0; j < GRP; ++j) {
        const float mref = S.pref[b][j];
        if (mref != m_run[j]) {  // a block raised the running maximum: bring the sums to it (fp32)
          const float alpha = expf(m_run[j] - mref);
          l_run[j] *= alpha;
#pragma unroll
          for (int e = 0; e < HD; ++e) acc[j][e] *= alpha;
          m_run[j] = mref;
        }
        const float p = lane < nkeys ? expf(S.sc[j][ti * kKeyTile + lane] - mref) : 0.f;
        l_run[j] += warp_sum(p);
        pj[j] = p;
      }
      // V rows: half-warp h takes keys kb + 2u + h, each lane 2 DPL dims of the row, 8 independent loads per
      // batch (16 keys per round trip); keys past the tile's end load nothing and carry p = 0
      for (int kb = 0; kb < nkeys; kb += 16) {
        RawRow<BF16, HD> raw[8];  // loaded first, unpacked when used: 8 rows in flight at HD * 2 or 4 bytes each
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int key = kb + 2 * u + half;
          raw[u].load(t.V, (t0 + (key < nkeys ? key : 0)) * D + (lane & 15) * HD, key < nkeys);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float vv[HD];
          raw[u].unpack(vv);
#pragma unroll
          for (int j = 0; j < GRP; ++j) {
            const float p32 = __shfl_sync(0xffffffffu, pj[j], (kb + 2 * u + half) & 31);
            const float pk = BF16 ? round_bf16(p32) : p32;
#pragma unroll
            for (int e = 0; e < HD; ++e) acc[j][e] = fmaf(pk, vv[e], acc[j][e]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < GRP; ++j)
#pragma unroll
    for (int e = 0; e < HD; ++e) acc[j][e] += __shfl_xor_sync(0xffffffffu, acc[j][e], 16);  // even + odd keys
  const int64_t ntot = (t.k1 - t.k0 + kKeyTile - 1) / kKeyTile;
  if (warp < min((int64_t)kAttnWarps, ntot)) {
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      if (lane == 0) {
        S.w_m[warp][j] = m_run[j];
        S.w_l[warp][j] = l_run[j];
      }
      if (lane < 16)
#pragma unroll
        for (int e = 0; e < HD; ++e) S.w_acc[warp][j][lane * HD + e] = acc[j][e];
    }
  }
}

struct AttnOut {
  void *out;          // this row's output; head h at element offset h * D
  float *part;        // this row's split partials: head h, split s at (h * max_split + s) * (D + 2)
  unsigned *cnt;      // combine counter of this (row, kv head)
  unsigned long long *done;  // nullable: +1 (release) once this kv head's output is written
  int g, split, nsplit, max_split, busy;
};

__device__ __forceinline__ void red_release_add_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <bool BF16>
__device__ __forceinline__ void store_out(void *out, int64_t i, float v) {
  if (BF16)
    ((uint16_t *)out)[i] = f32_to_bf16_bits(v);
  else
    ((float *)out)[i] = v;
}

// Merge the warps (fixed order); one range: write the output; several: write the partial, and the last
// range of this kv head to arrive combines all of them.
template <int DPL, int GRP, bool BF16, int NT>
__device__ void attn_finish(AttnScratch<DPL, GRP> &S, const AttnOut &o) {
  constexpr int D = DPL * 32;
  nt_sync<NT>();
  const bool single = o.nsplit == 1;
  for (int idx = threadIdx.x; idx < GRP * D; idx += NT) {
    const int j = idx / D, dd = idx - j * D;
    float M = -INFINITY;
    for (int w = 0; w < o.busy; ++w) M = fmaxf(M, S.w_m[w][j]);
    float lsum = 0.f, a = 0.f;
    for (int w = 0; w < o.busy; ++w) {
      if (S.w_l[w][j] == 0.f) continue;
      const float f = expf(S.w_m[w][j] - M);
      lsum += S.w_l[w][j] * f;
      a += S.w_acc[w][j][dd] * f;
    }
    const int h = o.g * GRP + j;
    if (single) {
      store_out<BF16>(o.out, (int64_t)h * D + dd, a / lsum);
    } else {
      float *slot = o.part + ((int64_t)h * o.max_split + o.split) * (D + 2);
      slot[2 + dd] = a;
      if (dd == 0) {
        slot[0] = M;
        slot[1] = lsum;
      }
    }
  }
  if (single) {
    if (o.done) {
      nt_sync<NT>();
      if (threadIdx.x == 0) red_release_add_u64(o.done, 1ull);
    }
    return;
  }
  __threadfence();
  nt_sync<NT>();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(o.cnt, 1u);
    S.flag = prev == (unsigned)(o.nsplit - 1);
    if (S.flag) *o.cnt = 0u;
  }
  nt_sync<NT>();
  if (!S.flag) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < GRP * D; idx += NT) {
    const int j = idx / D, dd = idx - j * D;
    const int h = o.g * GRP + j;
    const float *base = o.part + (int64_t)h * o.max_split * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < o.nsplit; ++s) M = fmaxf(M, __ldcg(base + s * (D + 2)));
    float lsum = 0.f, a = 0.f;
    for (int s = 0; s < o.nsplit; ++s) {
      const float ls = __ldcg(base + s * (D + 2) + 1);
      if (ls == 0.f) continue;
      const float f = expf(__ldcg(base + s * (D + 2)) - M);
      lsum += ls * f;
      a += __ldcg(base + s * (D + 2) + 2 + dd) * f;
    }
    store_out<BF16>(o.out, (int64_t)h * D + dd, a / lsum);
  }
  if (o.done) {
    nt_sync<NT>();
    if (threadIdx.x == 0) red_release_add_u64(o.done, 1ull);
  }
}

// ---------------------------------------------------------------------------------------------- split kernel
template <int DPL, int GRP, bool BF16>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnParams p) {
  constexpr int D = DPL * 32;
  __shared__ AttnScratch<DPL, GRP> S;
  __shared__ float tmp[D];
  __shared__ float red[32];

  pdl_wait();
  pdl_launch_dependents();

  const int g = blockIdx.x, split = blockIdx.y;
  const int64_t row = blockIdx.z;
  const int64_t pos = row_pos(p, row);
  const int64_t L = pos + 1;
  if (L > p.cap || pos < 0) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return;
  }
  const int bps = split_blocks(L, p.split_cap, kMinSplitBlocksOp);
  const int nsplit = split_count(L, bps);
  if (split >= nsplit) return;
  const int64_t k0 = (int64_t)split * bps * kRefBlock;
  const int64_t k1 = min(L, k0 + (int64_t)bps * kRefBlock);

  const int64_t kv_base = row_kv_head(p, row, g) * p.cap * D;
  // ---- q (and, with APPEND, this step's k/v) ----
  if (p.flags & EGPT_FLAG_APPEND) {
    const uint16_t *qkv = (const uint16_t *)p.q + row * p.ldq;
    for (int j = 0; j < GRP; ++j)
      head_norm_rope(qkv + (int64_t)(g * GRP + j) * D, p.q_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, D, S.q[j],
                     nullptr, tmp, red);
    if (pos >= k0 && pos < k1) {  // this CTA's range holds the new slot: write it before reading the range
      uint16_t *kd = (uint16_t *)p.k_cache + kv_base + pos * D;
      head_norm_rope(qkv + (int64_t)(p.nq + g) * D, p.k_norm_w, p.eps, p.rope_cos, p.rope_sin, pos, D, tmp, kd,
                     S.w_acc[0][0], red);
      const uint16_t *vs = qkv + (int64_t)(p.nq + p.nkv + g) * D;
      uint16_t *vd = (uint16_t *)p.v_cache + kv_base + pos * D;
      for (int t = threadIdx.x; t < D; t += blockDim.x) vd[t] = vs[t];
    }
  } else {
    for (int j = 0; j < GRP; ++j)
      for (int t = threadIdx.x; t < D; t += blockDim.x)
        S.q[j][t] = BF16 ? bf16_bits_to_f32(((const uint16_t *)p.q)[row * p.ldq + (int64_t)(g * GRP + j) * D + t])
                         : ((const float *)p.q)[row * p.ldq + (int64_t)(g * GRP + j) * D + t];
  }
  __syncthreads();

  const size_t esz = BF16 ? 2 : 4;
  AttnTask t;
  t.K = (const char *)p.k_cache + kv_base * esz;
  t.V = (const char *)p.v_cache + kv_base * esz;
  t.k0 = k0;
  t.k1 = k1;
  t.scale = p.scale;
  t.prefetch_v = 1;
  if ((p.flags & EGPT_FLAG_REF_SOFTMAX) && k0 > 0) {
    attn_max_before<DPL, GRP, BF16, kAttnThreads>(t, S);
  } else if (threadIdx.x < GRP) {
    S.mb[threadIdx.x] = -INFINITY;
  }
  attn_walk<DPL, GRP, BF16, kAttnThreads, false>(t, S);
  AttnOut o;
  o.out = (char *)p.out + row * p.ldo * esz;
  o.part = p.ws_f ? p.ws_f + row * p.nq * p.max_split * (D + 2) : nullptr;
  o.cnt = p.ws_cnt ? p.ws_cnt + row * p.nkv + g : nullptr;
  o.done = nullptr;
  o.g = g;
  o.split = split;
  o.nsplit = nsplit;
  o.max_split = p.max_split;
  o.busy = (int)min((int64_t)kAttnWarps, (k1 - k0 + kKeyTile - 1) / kKeyTile);
  attn_finish<DPL, GRP, BF16, kAttnThreads>(S, o);
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

// Workspace layout: fp32 split partials [m][nq][max_split][d + 2] and range maxima [m][nq][max_split]
// (padded to 256 bytes), then u32 counters [3][m][nkv]: combine arrivals, max-exchange arrivals and
// max-exchange generation (the last two are used by the persistent decode step).
size_t attn_ws_float_bytes(int64_t m, int nq, int d, int max_split) {
  const size_t floats = (size_t)m * nq * max_split * (d + 3);
  return (floats * 4 + 255) / 256 * 256;
}

extern "C" size_t egpt_attn_ws_bytes(int64_t m, int nq, int nkv, int d, int max_split) {
  return attn_ws_float_bytes(m, nq, d, max_split) + 3 * (size_t)m * nkv * 4;
}

namespace egpt {
// The streamed single-row kernel (attn_stream.cu): which calls it takes, and its launch.
bool attn_stream_applies(const AttnParams &p, int64_t m, int d, int dtype, unsigned flags);
cudaError_t attn_stream_launch(AttnParams p, cudaStream_t st, bool pdl);
}  // namespace egpt

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
  if ((flags & EGPT_FLAG_APPEND) && ((m != 1 && !(flags & EGPT_FLAG_RAGGED)) || dtype != EGPT_BF16))
    return set_error(EGPT_ERR_ARG, "attn: fused append needs bf16 and m == 1 (or EGPT_FLAG_RAGGED)");
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
  // ranges: at most max_split per (row, kv head), and about two CTAs per SM over the whole grid (more ranges cost
  // more in combining than they gain in parallel reads: measured at L = 8192 and 32768, 8 kv heads)
  p.split_cap = std::max(1, std::min(max_split, (int)std::max<int64_t>(1, 2 * (int64_t)num_sms() / ((int64_t)nkv * m))));
  p.ws_f = (float *)ws;
  p.ws_cnt = ws ? (unsigned *)((char *)ws + attn_ws_float_bytes(m, nq, d, max_split)) : nullptr;
  p.flags = flags;
  const dim3 grid(nkv, p.split_cap, (unsigned)m);
  const bool pdl = (flags & EGPT_FLAG_PDL) != 0;
  if (attn_stream_applies(p, m, d, dtype, flags))  // one bf16 row, head_dim 128: K/V streamed by bulk copies
    return check_launch(attn_stream_launch(p, (cudaStream_t)stream, pdl), "attn_stream_kernel");
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

// ---------------------------------------------------------------------------------------------- no-alloc variant
// egpt_attn_decode for callers that may not allocate device memory: the split partials and counters live in
// one file-scope device array of EGPT_ATTN_NOALLOC_SCRATCH_BYTES that every call on a device shares. In host
// code the array's name only stands for the symbol; its device address comes from cudaGetSymbolAddress, once
// per device, on the first call made with that device current.
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[EGPT_ATTN_NOALLOC_SCRATCH_BYTES];

static void *noalloc_scratch(int *rc) {
  static std::mutex mu;
  static void *ptr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = set_error(EGPT_ERR_LAUNCH, "attn_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *rc = set_error(EGPT_ERR_ARG, "attn_decode_noalloc: device ordinal %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *rc = set_error(EGPT_ERR_LAUNCH, "attn_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptr[dev] = p;
  }
  return ptr[dev];
}

extern "C" int egpt_attn_decode_noalloc(void *out, int64_t ldo, const void *q, int64_t ldq, void *k_cache,
                                        void *v_cache, int64_t cap, const int64_t *position, int64_t m, int nq,
                                        int nkv, int d, const void *q_norm_w, const void *k_norm_w, float eps,
                                        const void *rope_cos, const void *rope_sin, float scale, int max_split,
                                        int dtype, unsigned flags, void *stream) {
  clear_error();
  if (m < 1 || m > 65535 || nq < 1 || nkv < 1 || d < 1 || max_split < 1 || max_split > 1024)
    return set_error(EGPT_ERR_SHAPE, "attn_decode_noalloc: bad m, heads, head_dim or max_split");
  const size_t need = egpt_attn_ws_bytes(m, nq, nkv, d, max_split);
  if (need > (size_t)EGPT_ATTN_NOALLOC_SCRATCH_BYTES)
    return set_error(EGPT_ERR_WORKSPACE,
                     "attn_decode_noalloc: m=%lld nq=%d nkv=%d d=%d max_split=%d needs %zu bytes of scratch, above the "
                     "built-in %d; lower max_split or m, or call egpt_attn_decode with a workspace",
                     (long long)m, nq, nkv, d, max_split, need, EGPT_ATTN_NOALLOC_SCRATCH_BYTES);
  int rc = EGPT_OK;
  void *scratch = noalloc_scratch(&rc);
  if (!scratch) return rc;
  // the arrival counters must start at zero (the kernels leave them at zero; an aborted call may not)
  const size_t cnt_off = attn_ws_float_bytes(m, nq, d, max_split);
  cudaError_t e = cudaMemsetAsync((char *)scratch + cnt_off, 0, need - cnt_off, (cudaStream_t)stream);
  if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "attn_decode_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
  return egpt_attn_decode(out, ldo, q, ldq, k_cache, v_cache, cap, position, m, nq, nkv, d, q_norm_w, k_norm_w, eps,
                          rope_cos, rope_sin, scale, max_split, scratch, (size_t)EGPT_ATTN_NOALLOC_SCRATCH_BYTES, dtype,
                          flags, stream);
}
