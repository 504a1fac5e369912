// On-device stochastic decoding for B200: temperature -> top-k -> top-p -> inverse CDF, one token per row, with the
// semantics of BagelsFun/efficientgpt research/phase5/sampling.py:39-71 (filtered_probs, sample_from):
//
//   x = logits.float() / temperature
//   top-k: x < (k-th largest x, duplicates counted) -> -inf           (ties at the k-th value kept)
//   p = softmax(x)
//   top-p: in the stable descending order of p, drop every token whose exclusive prefix mass is >= top_p (the top
//          token is always kept), then p /= sum(kept p)
//   token = first j with cdf[j] > u * cdf[-1], cdf the prefix sums of p in index order, clamped to the last index
//           with p > 0                                                (searchsorted(right=True) + the guard)
//
// No sort and no floating-point atomics: the row is split over kCtas CTAs, and a chain of small kernels (the kernel
// boundaries are the only grid-wide synchronisation, so nothing spins) selects the top-k threshold and the top-p
// boundary by radix descent over an order-preserving integer key, 8 bits per level:
//   * the key orders tokens as x does: for bf16 logits the 16-bit key of the logit itself (x = l / T keeps the order
//     of l, and distinct bf16 values stay distinct after the division), for fp32 logits the 32-bit key of x;
//   * level histograms hold counts (u32) and probability mass in fixed point (u64, units of 2^-60): integer
//     atomics, so every sum is independent of the order in which CTAs and threads add, and the result is
//     deterministic run to run;
//   * top-p's stable order among equal p is index order; equal keys have equal p, so the boundary key group keeps
//     its first t tokens by index, t = ceil((top_p - mass above) / p) (ranks by an index-ordered scan);
//   * the inverse CDF runs on fixed-point masses too (exact prefix sums, target = floor(u * total)).
// Floating-point sums (the softmax denominator) are per-CTA fixed-order reductions in fp64, then the CTA partials in
// CTA order: deterministic. The differences from the reference's fp32 cumsum are confined to draws within a few
// ulps of a CDF boundary and top_p values within a few ulps of a prefix sum.
//
// Workspace per row (zero on the first call; the chain leaves it zeroed): see WsRow.
#include "internal.h"
#include "common.cuh"

namespace egpt {
namespace smp {

constexpr int kThreads = 256;
constexpr int kCtas = 64;       // CTAs per row
constexpr int kMaxLevels = 4;   // 32-bit keys, 8 bits per level
constexpr double kFix = 1152921504606846976.0;  // 2^60

struct Hist {
  unsigned cnt[256];
  unsigned long long mass[256];
};
// Radix-descent state after some levels: prefix of the selected key (high bits) and what lies above it.
struct Sel {
  unsigned prefix;
  int fixed;             // bits fixed so far
  long long rem;         // top-k: rank still to find (1-based) within the prefix
  unsigned long long G;  // top-p: fixed-point mass strictly above the prefix range
  int all;               // top-p: the total mass is below top_p, every token is kept
};
// Decisions the last kernels need, written identically by every CTA of the kernel that makes them.
struct Final {
  unsigned c;            // top-p boundary key
  int all;               // top-p keeps every token with p > 0
  unsigned n;            // tokens in the boundary group
  long long t_keep;      // of which the first t_keep by index are kept
  float s_kept;          // sum of the kept p
};
struct Header {
  unsigned rows_done;    // rows whose draw is complete (the last one advances *u_index)
  unsigned pad[3];
};
struct WsRow {
  Hist topk[kMaxLevels];          // counts of the top-k levels
  Hist topp[kMaxLevels];          // counts and fixed-point mass of the top-p levels
  unsigned tcnt[kCtas][256];      // last top-p level, per CTA: counts (index-ordered tie ranks)
  Sel tk_sel[kMaxLevels + 1];     // top-k state after levels < i (i >= 1)
  Sel tp_sel[kMaxLevels + 1];     // top-p state after levels < i (i >= 1)
  Final fin;
  unsigned maxkey;                // order-preserving key of max x (top-k path; atomicMax, 0 below every float)
  unsigned kth;                   // top-k: keep key >= kth
  int last;                       // last index with q > 0, + 1 (atomicMax; 0 = none)
  unsigned done;                  // CTAs of this row finished with the workspace (k_pick)
  float m_part[kCtas];            // per-CTA maximum of x (softmax)
  double s_part[kCtas];           // per-CTA sum of exp(x - m_part)
  unsigned long long q_part[kCtas];  // per-CTA fixed-point sums of q
};

struct Args {
  const void *logits;
  int bf16;
  int64_t V, ld;
  float temperature;
  int64_t top_k;   // 0: off
  float top_p;     // >= 1: off
  const float *u;
  int64_t u_ld;
  int64_t *u_index;
  int64_t *out;
  int64_t out_ld;
  Header *hdr;
  WsRow *ws;
  int64_t rows;
  int levels;      // key bits / 8
};

__device__ __forceinline__ unsigned fkey(float f) {
  const unsigned b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_dec(unsigned k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }
// Element loops: a thread first issues the loads of kE elements, then uses them (the loads overlap instead of
// each element paying an L2 round trip).
constexpr int kE = 8;
__device__ __forceinline__ unsigned load_raw(const Args &A, int64_t row, int64_t i) {
  return A.bf16 ? (unsigned)((const uint16_t *)A.logits)[row * A.ld + i]
                : __float_as_uint(((const float *)A.logits)[row * A.ld + i]);
}
// x = logit / T and the order-preserving key (bf16: 16 bits of the logit; fp32: 32 bits of x).
__device__ __forceinline__ void decode(const Args &A, unsigned raw, float &x, unsigned &key) {
  if (A.bf16) {
    x = __uint_as_float(raw << 16) / A.temperature;
    key = (raw & 0x8000u) ? (~raw & 0xFFFFu) : (raw | 0x8000u);
  } else {
    x = __uint_as_float(raw) / A.temperature;
    key = fkey(x);
  }
}
// f(i, x, key) over the CTA's elements i = cta_begin + t + j * kThreads, j increasing.
template <class F>
__device__ __forceinline__ void each_strided(const Args &A, int64_t row, F f) {
  const int64_t ce = min(A.V, (int64_t)(blockIdx.x + 1) * ((A.V + kCtas - 1) / kCtas));
  for (int64_t b = (int64_t)blockIdx.x * ((A.V + kCtas - 1) / kCtas) + threadIdx.x; b < ce; b += (int64_t)kE * kThreads) {
    unsigned raw[kE];
#pragma unroll
    for (int j = 0; j < kE; ++j) {
      const int64_t i = b + (int64_t)j * kThreads;
      raw[j] = i < ce ? load_raw(A, row, i) : 0u;
    }
#pragma unroll
    for (int j = 0; j < kE; ++j) {
      const int64_t i = b + (int64_t)j * kThreads;
      if (i < ce) {
        float x;
        unsigned key;
        decode(A, raw[j], x, key);
        f(i, x, key);
      }
    }
  }
}
// f(i, x, key) over [b, e) in index order.
template <class F>
__device__ __forceinline__ void each_range(const Args &A, int64_t row, int64_t b, int64_t e, F f) {
  for (int64_t b0 = b; b0 < e; b0 += kE) {
    unsigned raw[kE];
#pragma unroll
    for (int j = 0; j < kE; ++j) raw[j] = b0 + j < e ? load_raw(A, row, b0 + j) : 0u;
#pragma unroll
    for (int j = 0; j < kE; ++j)
      if (b0 + j < e) {
        float x;
        unsigned key;
        decode(A, raw[j], x, key);
        f(b0 + j, x, key);
      }
  }
}
__device__ __forceinline__ unsigned long long fixmass(float p) {
  return (unsigned long long)__double2ull_rn((double)p * kFix);
}
__device__ __forceinline__ int bits_of(const Args &A) { return 8 * A.levels; }
__device__ __forceinline__ bool topk_on(const Args &A) { return A.top_k > 0 && A.top_k < A.V; }
__device__ __forceinline__ bool topp_on(const Args &A) { return A.top_p < 1.f; }
__device__ __forceinline__ unsigned long long topp_fix(const Args &A) {
  return (unsigned long long)__double2ull_rn((double)A.top_p * kFix);
}
__device__ __forceinline__ int64_t cta_begin(const Args &A) { return (int64_t)blockIdx.x * ((A.V + kCtas - 1) / kCtas); }
__device__ __forceinline__ int64_t cta_end(const Args &A) {
  return min(A.V, (int64_t)(blockIdx.x + 1) * ((A.V + kCtas - 1) / kCtas));
}

// One warp: scan bins 255..0 of `h` for the first bin (from the top) where the running count (or mass) added to
// `base` reaches `target`; returns the bin (-1 if none) and the sum of the bins above it in *above.
template <bool MASS>
__device__ int warp_find(const Hist &h, unsigned long long base, unsigned long long target, unsigned long long *above) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[8], tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // lane l holds bins 255 - 8 l - i
    const int b = 255 - 8 * lane - i;
    v[i] = MASS ? h.mass[b] : (unsigned long long)h.cnt[b];
    tot += v[i];
  }
  unsigned long long incl = tot;  // inclusive scan over lanes (top bins first)
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const unsigned long long excl = incl - tot;
  const unsigned hit = __ballot_sync(0xffffffffu, base + incl >= target);
  if (!hit) {
    *above = __shfl_sync(0xffffffffu, incl, 31);
    return -1;
  }
  const int src = __ffs(hit) - 1;
  int bin = -1;
  unsigned long long ab = 0;
  if (lane == src) {
    unsigned long long run = base + excl;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (bin < 0) {
        if (run + v[i] >= target) {
          bin = 255 - 8 * lane - i;
          ab = run - base;
        } else {
          run += v[i];
        }
      }
    }
  }
  bin = __shfl_sync(0xffffffffu, bin, src);
  *above = __shfl_sync(0xffffffffu, ab, src);
  return bin;
}

__device__ __forceinline__ Sel sel_init(unsigned long long target) {
  Sel s;
  s.prefix = 0, s.fixed = 0, s.rem = (long long)target, s.G = 0, s.all = 0;
  return s;
}
// One level of the descent (one warp): `s` (after the levels above) refined by histogram h.
template <bool MASS>
__device__ Sel descend_one(Sel s, const Hist &h, unsigned long long target) {
  unsigned long long above = 0;
  const int b = MASS ? warp_find<true>(h, s.G, target, &above) : warp_find<false>(h, 0, (unsigned long long)s.rem, &above);
  if (b < 0) {  // count: cannot happen (k <= V); mass: the total is below top_p
    s.all = 1;
    return s;
  }
  if (MASS)
    s.G += above;
  else
    s.rem -= (long long)above;
  s.prefix = (s.prefix << 8) | (unsigned)b;
  s.fixed += 8;
  return s;
}
__device__ __forceinline__ bool in_prefix(unsigned key, const Sel &s, int bits) {
  return s.fixed == 0 || (key >> (bits - s.fixed)) == s.prefix;
}

// Softmax statistics of the row: max x and the denominator, from the per-CTA parts (fixed order).
struct Soft {
  float M, s;
};
__device__ Soft soft_of(const WsRow &W) {  // one warp; lane l takes parts l, l + 32 (a fixed reduction order)
  static_assert(kCtas == 64, "two parts per lane");
  const int lane = threadIdx.x & 31;
  const float m0 = W.m_part[lane], m1 = W.m_part[lane + 32];
  const double s0 = W.s_part[lane], s1 = W.s_part[lane + 32];
  const float M = warp_max(fmaxf(m0, m1));
  double t = (m0 == -INFINITY ? 0.0 : s0 * (double)expf(m0 - M)) + (m1 == -INFINITY ? 0.0 : s1 * (double)expf(m1 - M));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return Soft{M, (float)t};
}

// What every per-element pass needs, prepared by warp 0 and broadcast.
struct Ctx {
  Soft sm;
  int topk;
  unsigned kth;
  int topp;
  Sel tp;         // top-p state for the level being counted (k_topp) or final (k_qsum / k_pick)
  Final fin;
};
__device__ __forceinline__ float p_of(const Ctx &c, float x, unsigned key) {
  if (c.topk && key < c.kth) return 0.f;
  return expf(x - c.sm.M) / c.sm.s;
}

__device__ double block_sum_d(double v) {
  __shared__ double red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}
__device__ float block_max(float v) {
  __shared__ float red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < kThreads / 32; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}
// Block-wide exclusive scan of one u64 per thread (thread order); *total = the block's sum.
__device__ unsigned long long block_scan_u64(unsigned long long v, unsigned long long *total) {
  __shared__ unsigned long long ws[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  unsigned long long before = 0, tot = 0;
  for (int w = 0; w < kThreads / 32; ++w) {
    if (w < warp) before += ws[w];
    tot += ws[w];
  }
  __syncthreads();
  *total = tot;
  return before + incl - v;
}

// Kernel 1. With top-k: max x (atomicMax) and the top-k level-0 counts. Without: this CTA's softmax part
// (max and sum of exp(x - max)).
__global__ void __launch_bounds__(kThreads) k_first(Args A) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ unsigned h[256];
  for (int i = threadIdx.x; i < 256; i += kThreads) h[i] = 0;
  __syncthreads();
  const int bits = bits_of(A);
  const bool tk = topk_on(A);
  float m = -INFINITY;
  each_strided(A, row, [&](int64_t, float x, unsigned key) {
    m = fmaxf(m, x);
    if (tk) atomicAdd(&h[key >> (bits - 8)], 1u);
  });
  if (tk) {
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax(&W.maxkey, fkey(m));
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += kThreads)
      if (h[i]) atomicAdd(&W.topk[0].cnt[i], h[i]);
    return;
  }
  m = block_max(m);
  double acc = 0.0;
  each_strided(A, row, [&](int64_t, float x, unsigned) { acc += (double)expf(x - m); });
  const double t = block_sum_d(acc);
  if (threadIdx.x == 0) W.m_part[blockIdx.x] = m, W.s_part[blockIdx.x] = t;
}

// Top-k level lv >= 1: decide level lv - 1, then count the keys inside the new prefix.
__global__ void __launch_bounds__(kThreads) k_topk(Args A, int lv) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ unsigned h[256];
  __shared__ Sel ss;
  for (int i = threadIdx.x; i < 256; i += kThreads) h[i] = 0;
  if (threadIdx.x < 32) {
    const Sel prev = lv - 1 == 0 ? sel_init((unsigned long long)A.top_k) : W.tk_sel[lv - 1];
    const Sel s = descend_one<false>(prev, W.topk[lv - 1], (unsigned long long)A.top_k);
    if (threadIdx.x == 0) ss = s, W.tk_sel[lv] = s;
  }
  __syncthreads();
  const Sel s = ss;
  const int bits = bits_of(A);
  each_strided(A, row, [&](int64_t, float, unsigned key) {
    if (in_prefix(key, s, bits)) atomicAdd(&h[(key >> (bits - 8 * (lv + 1))) & 255u], 1u);
  });
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += kThreads)
    if (h[i]) atomicAdd(&W.topk[lv].cnt[i], h[i]);
}

// With top-k: decide the last top-k level (the threshold), then this CTA's softmax part over the kept tokens.
__global__ void __launch_bounds__(kThreads) k_sum(Args A) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ unsigned skth;
  if (threadIdx.x < 32) {
    const int L = A.levels;
    const Sel prev = L - 1 == 0 ? sel_init((unsigned long long)A.top_k) : W.tk_sel[L - 1];
    const Sel s = descend_one<false>(prev, W.topk[L - 1], (unsigned long long)A.top_k);
    if (threadIdx.x == 0) skth = s.prefix, W.kth = s.prefix;
  }
  __syncthreads();
  const unsigned kth = skth;
  const float M = fkey_dec(W.maxkey);
  double acc = 0.0;
  each_strided(A, row, [&](int64_t, float x, unsigned key) {
    if (key >= kth) acc += (double)expf(x - M);
  });
  const double t = block_sum_d(acc);
  if (threadIdx.x == 0) W.m_part[blockIdx.x] = M, W.s_part[blockIdx.x] = t;
}

// Warp 0 of every later kernel: softmax statistics and the top-k threshold.
__device__ void ctx_base(const Args &A, const WsRow &W, Ctx &t) {
  t.sm = soft_of(W);
  t.topk = topk_on(A);
  t.kth = t.topk ? W.kth : 0u;
  t.topp = topp_on(A);
  t.tp = sel_init(0);
  t.fin.c = 0, t.fin.all = 1, t.fin.n = 0, t.fin.t_keep = 0, t.fin.s_kept = 1.f;
}

// Top-p level lv: decide level lv - 1 (lv >= 1), then count and weigh (fixed point) the tokens inside the prefix;
// the last level also keeps per-CTA counts for the tie ranks.
__global__ void __launch_bounds__(kThreads) k_topp(Args A, int lv) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ unsigned h[256];
  __shared__ unsigned long long hm[256];
  __shared__ Ctx sc;
  for (int i = threadIdx.x; i < 256; i += kThreads) h[i] = 0, hm[i] = 0ull;
  if (threadIdx.x < 32) {
    Ctx t;
    ctx_base(A, W, t);
    if (lv >= 1) {
      const unsigned long long P = topp_fix(A);
      const Sel prev = lv - 1 == 0 ? sel_init(0) : W.tp_sel[lv - 1];
      t.tp = prev.all ? prev : descend_one<true>(prev, W.topp[lv - 1], P);
      if (threadIdx.x == 0) W.tp_sel[lv] = t.tp;
    }
    if (threadIdx.x == 0) sc = t;
  }
  __syncthreads();
  const Ctx c = sc;
  if (c.tp.all) return;  // a level above found the total below top_p: every token is kept
  const int bits = bits_of(A);
  const bool last = lv == A.levels - 1;
  each_strided(A, row, [&](int64_t, float x, unsigned key) {
    const float p = p_of(c, x, key);
    if (p > 0.f && in_prefix(key, c.tp, bits)) {
      const unsigned b = (key >> (bits - 8 * (lv + 1))) & 255u;
      atomicAdd(&h[b], 1u);
      atomicAdd(&hm[b], fixmass(p));
    }
  });
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += kThreads) {
    if (h[i]) {
      atomicAdd(&W.topp[lv].cnt[i], h[i]);
      atomicAdd(&W.topp[lv].mass[i], hm[i]);
    }
    if (last) W.tcnt[blockIdx.x][i] = h[i];
  }
}

// Whether token (key, p) survives top-p, given its index-ordered rank in the boundary group (read for members).
__device__ __forceinline__ bool kept(const Ctx &c, unsigned key, float p, long long rank) {
  if (p <= 0.f) return false;
  if (!c.topp || c.fin.all) return true;
  if (key != c.fin.c) return key > c.fin.c;
  return rank < c.fin.t_keep;
}
__device__ __forceinline__ unsigned long long qfix(const Ctx &c, float p, bool keep) {
  if (!keep) return 0ull;
  return fixmass((c.topp && !c.fin.all) ? p / c.fin.s_kept : p);
}
__device__ __forceinline__ void thread_range(const Args &A, int64_t &b, int64_t &e) {
  const int64_t cb = cta_begin(A), ce = cta_end(A);
  const int64_t n = ce > cb ? ce - cb : 0, per = (n + kThreads - 1) / kThreads;
  b = min(ce, cb + (int64_t)threadIdx.x * per);
  e = min(ce, b + per);
}
// Index-ordered rank of the thread's first boundary-group member: members in earlier CTAs and earlier threads.
// Only needed when the group is cut (0 < t_keep < n); CTA-uniform condition.
__device__ long long rank_start(const Args &A, const WsRow &W, const Ctx &c, int64_t row, int64_t b, int64_t e) {
  if (!c.topp || c.fin.all || c.fin.t_keep >= (long long)c.fin.n) return 0;
  const unsigned bin = c.fin.c & 255u;
  long long before = 0;
#pragma unroll 16
  for (unsigned i = 0; i < blockIdx.x; ++i) before += W.tcnt[i][bin];
  long long mine = 0;
  each_range(A, row, b, e, [&](int64_t, float x, unsigned key) { mine += (key == c.fin.c && p_of(c, x, key) > 0.f) ? 1 : 0; });
  unsigned long long tot;
  return before + (long long)block_scan_u64((unsigned long long)mine, &tot);
}
struct Walk {
  unsigned long long sum;
  int64_t last;  // last index with q > 0, or -1
};
__device__ Walk walk_range(const Args &A, const Ctx &c, int64_t row, int64_t b, int64_t e, long long rank) {
  Walk w{0ull, -1};
  each_range(A, row, b, e, [&](int64_t i, float x, unsigned key) {
    const float p = p_of(c, x, key);
    const bool k = kept(c, key, p, rank);
    if (p > 0.f && key == c.fin.c) ++rank;
    const unsigned long long q = qfix(c, p, k);
    w.sum += q;
    if (q) w.last = i;
  });
  return w;
}

// Decide the last top-p level (the boundary group and how much of it is kept), then this CTA's fixed-point sum
// of q and its last index with q > 0.
__global__ void __launch_bounds__(kThreads) k_qsum(Args A) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ Ctx sc;
  if (threadIdx.x < 32) {
    Ctx t;
    ctx_base(A, W, t);
    if (t.topp) {
      const int L = A.levels;
      const unsigned long long P = topp_fix(A);
      const Sel prev = L - 1 == 0 ? sel_init(0) : W.tp_sel[L - 1];
      const Sel s = prev.all ? prev : descend_one<true>(prev, W.topp[L - 1], P);
      t.tp = s;
      if (!s.all) {
        const unsigned b = s.prefix & 255u, n = W.topp[L - 1].cnt[b];
        const unsigned long long pc = n ? W.topp[L - 1].mass[b] / n : 0ull;
        long long tk = n;
        if (pc > 0) tk = (long long)((P - s.G + pc - 1) / pc);
        t.fin.c = s.prefix, t.fin.all = 0, t.fin.n = n;
        t.fin.t_keep = tk < (long long)n ? tk : (long long)n;
        t.fin.s_kept = (float)((double)(s.G + (unsigned long long)t.fin.t_keep * pc) / kFix);
      }
      if (threadIdx.x == 0 && blockIdx.x == 0) W.fin = t.fin;
    }
    if (threadIdx.x == 0) sc = t;
  }
  __syncthreads();
  const Ctx c = sc;
  int64_t b, e;
  thread_range(A, b, e);
  const long long r0 = rank_start(A, W, c, row, b, e);
  const Walk w = walk_range(A, c, row, b, e, r0);
  unsigned long long tot;
  block_scan_u64(w.sum, &tot);
  const float lastf = block_max((float)(w.last + 1));  // indices < 2^24: exact in fp32
  if (threadIdx.x == 0) {
    W.q_part[blockIdx.x] = tot;
    if (lastf > 0.f) atomicMax(&W.last, (int)lastf);
  }
}

// The draw: every CTA finds the CTA whose q range holds the target; that CTA finds the token. The last CTA of the
// row to finish zeroes the row's workspace; the last row advances *u_index.
__global__ void __launch_bounds__(kThreads) k_pick(Args A) {
  const int64_t row = blockIdx.y;
  WsRow &W = A.ws[row];
  __shared__ Ctx sc;
  __shared__ int s_last, s_owner;
  __shared__ unsigned long long s_target, s_before;
  if (threadIdx.x < 32) {  // one warp: target = floor(u * total); the CTA whose q range holds it (a warp scan)
    static_assert(kCtas == 64, "two parts per lane");
    const int lane = threadIdx.x;
    const float u = A.u[row * A.u_ld + (A.u_index ? *A.u_index : 0)];
    const unsigned long long q0 = W.q_part[2 * lane], q1 = W.q_part[2 * lane + 1];
    unsigned long long incl = q0 + q1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const unsigned long long total = __shfl_sync(0xffffffffu, incl, 31), excl = incl - q0 - q1;
    const unsigned long long target = (unsigned long long)floor((double)u * (double)total);
    // token = first j with (inclusive prefix of q) > target: the first part whose inclusive prefix exceeds it
    const unsigned hit = __ballot_sync(0xffffffffu, incl > target);
    if (lane == 0) s_owner = -1, s_target = target, s_before = 0;
    if (hit) {
      const int src = __ffs(hit) - 1;
      if (lane == src) {
        const bool first = excl + q0 > target;
        s_owner = first ? 2 * lane : 2 * lane + 1;
        s_before = first ? excl : excl + q0;
      }
    }
  }
  __syncthreads();
  const int owner = s_owner;
  const unsigned long long target = s_target, before = s_before;
  const int64_t lastq = (int64_t)W.last - 1;
  if (owner < 0) {  // u * total == total after rounding: the last token with mass
    if (blockIdx.x == 0 && threadIdx.x == 0) A.out[row * A.out_ld] = lastq >= 0 ? lastq : 0;
  } else if ((int)blockIdx.x == owner) {
    if (threadIdx.x < 32) {
      Ctx t;
      ctx_base(A, W, t);
      if (t.topp) t.fin = W.fin;
      if (threadIdx.x == 0) sc = t;
    }
    __syncthreads();
    const Ctx c = sc;
    int64_t b, e;
    thread_range(A, b, e);
    const long long r0 = rank_start(A, W, c, row, b, e);
    const Walk w = walk_range(A, c, row, b, e, r0);
    unsigned long long ctot;
    const unsigned long long excl = before + block_scan_u64(w.sum, &ctot);
    if (excl <= target && excl + w.sum > target) {  // the crossing is in this thread's range
      unsigned long long run = excl;
      long long rank = r0;
      bool found = false;
      each_range(A, row, b, e, [&](int64_t i, float x, unsigned key) {
        if (found) return;
        const float p = p_of(c, x, key);
        const bool k = kept(c, key, p, rank);
        if (p > 0.f && key == c.fin.c) ++rank;
        run += qfix(c, p, k);
        if (run > target) {
          A.out[row * A.out_ld] = (lastq >= 0 && i > lastq) ? lastq : i;
          found = true;
        }
      });
    }
  }
  // workspace release: every CTA is done reading the row's workspace
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&W.done, 1u) == (unsigned)(kCtas - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  uint4 *w4 = (uint4 *)&W;
  for (size_t i = threadIdx.x; i < sizeof(WsRow) / 16; i += kThreads) w4[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&A.hdr->rows_done, 1u) == (unsigned)(A.rows - 1)) {
      A.hdr->rows_done = 0u;
      if (A.u_index) *A.u_index += 1;
    }
  }
}

}  // namespace smp
}  // namespace egpt

using namespace egpt;

static_assert(sizeof(smp::WsRow) % 16 == 0 && sizeof(smp::Header) == 16, "sampler workspace layout");

extern "C" size_t egpt_sample_ws_bytes(int64_t rows) {
  return rows > 0 ? sizeof(smp::Header) + (size_t)rows * sizeof(smp::WsRow) : 0;
}

extern "C" int egpt_sample(const void *logits, int dtype, int64_t rows, int64_t V, int64_t ld, float temperature,
                           int64_t top_k, float top_p, const float *u, int64_t u_ld, int64_t *u_index, int64_t *out,
                           int64_t out_ld, void *ws, size_t ws_bytes, void *stream) {
  clear_error();
  if (!logits || !u || !out || !ws) return set_error(EGPT_ERR_ARG, "sample: null pointer");
  if (dtype != EGPT_BF16 && dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "sample: logits must be bf16 or fp32");
  if (rows < 1 || rows > 65535 || V < 1 || V > (1 << 24) || ld < V || u_ld < 0 || out_ld < 1)
    return set_error(EGPT_ERR_SHAPE, "sample: bad shape");
  if (!(temperature > 0.f))
    return set_error(EGPT_ERR_ARG, "temperature must be > 0; use the greedy decoders for temperature 0");
  if (top_k < 0) return set_error(EGPT_ERR_ARG, "top_k must be >= 1 (0: off)");
  if (!(top_p > 0.f && top_p <= 1.f)) return set_error(EGPT_ERR_ARG, "top_p must be in (0, 1]");
  if (ws_bytes < egpt_sample_ws_bytes(rows)) return set_error(EGPT_ERR_WORKSPACE, "sample: workspace too small");
  if ((uintptr_t)ws % 16) return set_error(EGPT_ERR_ALIGN, "sample: workspace must be 16-byte aligned");
  smp::Args A{};
  A.logits = logits, A.bf16 = dtype == EGPT_BF16, A.V = V, A.ld = ld, A.temperature = temperature;
  A.top_k = top_k, A.top_p = top_p, A.u = u, A.u_ld = u_ld, A.u_index = u_index, A.out = out, A.out_ld = out_ld;
  A.hdr = (smp::Header *)ws;
  A.ws = (smp::WsRow *)((char *)ws + sizeof(smp::Header));
  A.rows = rows;
  A.levels = A.bf16 ? 2 : 4;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid(smp::kCtas, (unsigned)rows), block(smp::kThreads);
  const bool tk = top_k > 0 && top_k < V, tp = top_p < 1.f;
  smp::k_first<<<grid, block, 0, st>>>(A);
  if (tk) {
    for (int lv = 1; lv < A.levels; ++lv) smp::k_topk<<<grid, block, 0, st>>>(A, lv);
    smp::k_sum<<<grid, block, 0, st>>>(A);
  }
  if (tp)
    for (int lv = 0; lv < A.levels; ++lv) smp::k_topp<<<grid, block, 0, st>>>(A, lv);
  smp::k_qsum<<<grid, block, 0, st>>>(A);
  smp::k_pick<<<grid, block, 0, st>>>(A);
  return check_launch(cudaGetLastError(), "sample");
}
