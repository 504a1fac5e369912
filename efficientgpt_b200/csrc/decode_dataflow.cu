// Dataflow decode step for B200 (sm_100a): the whole token in one cooperative kernel, one CTA per SM, with no grid
// barrier. Same arithmetic as the persistent step of decode_step.cu (exact int8 tensor-core GEMVs on a fixed-point
// stage input, HF rounding points, the reference GPU kernel's softmax rounding), different machinery:
//
//   * Roles: the last NKV CTAs each run the attention of one kv head for every layer; the other W = G - NKV CTAs
//     run every GEMV stage (tile t of a stage belongs to GEMV CTA t mod W) and the lm_head.
//   * Weights: each warp of a GEMV CTA streams its own items (16 rows x 256 columns = 4 KB; item i of the CTA's
//     share of a stage belongs to warp i mod 16, lm_head tiles whole to warp tile mod 16) through its own ring of
//     shared-memory slots: lane 0 issues an item as two TMA tensor loads (no multicast, this GPU's memory) whose
//     transaction count completes the slot's mbarrier, and refills the slot with the item `ring` positions ahead
//     as soon as the warp has consumed it, whatever stage that item belongs to. So while the warp waits for a
//     stage's input, the next stages' weights are already landing. The tensor map views a weight matrix [N, K]
//     as [K/64][N][64] bytes: one box {64, 8, 4} lands as [4][8][64], rows of one 64-column step 64 bytes apart,
//     so the MMA operand reads of a warp hit 32 distinct banks.
//   * Activations: every stage output is published as LL words in global memory: one 8-byte word = two bf16
//     values in the low half and a 32-bit tag (step epoch, layer, site) in the high half, written and read in
//     one piece. A consumer polls the words of its input until every tag is the expected one: the data and the
//     "ready" signal arrive together (no flag, fence, counter or barrier between producer and consumer). Each
//     layer's buffers are separate, so nothing is overwritten within a step; tags make the previous step's words
//     stale. Every poll is bounded and records EGPT_ERR_TIMEOUT instead of hanging.
//   * Attention CTAs keep their kv head's cached K and V rows in shared memory when the cache fits (one bulk
//     copy per layer, issued a layer ahead, so the rows are resident before the layer's q arrives) and run their
//     own shared-memory attention (attn_smem) on them; otherwise the attention core of attention.cu reads the
//     cache in global memory. Both keep the reference GPU kernel's 128-key softmax blocks; they differ only in
//     fp32 summation order.
//   * RMSNorm's sum of squares is accumulated in fp64 (the bf16 squares are exact, so the sum is exact in
//     practice and independent of the thread layout), rounded once to fp32.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace egpt {
namespace df {

constexpr int kW = 16;                // warps per CTA
constexpr int kCT = kW * 32;          // threads per CTA (named barrier 1)
constexpr int kItem = 4096;           // one item: 16 rows x 256 int8 columns
constexpr int kChunkCols = 256;
constexpr int kMaxGroups = 4;         // staged input: up to 4 groups of 4 values per thread (k <= 8192)
constexpr int kMaxK = kMaxGroups * 4 * kCT;
constexpr int kXPad = 64;

enum Kind { QKV = 0, OPROJ = 1, GATEUP = 2, DOWN = 3, LMHEAD = 4 };
constexpr int kMaxLayers = 56;
constexpr int kMaxMaps = 4 * kMaxLayers + 1;  // 225 x 128 B of kernel parameters (the limit is 32764 B)

struct Params {
  int L, H, NQ, NKV, D, I;
  int64_t V, cap;
  float eps, scale;
  int scale_bf16;
  int rw;                           // ring slots per warp
  int kv_smem;                      // attention CTAs hold their K and V rows in shared memory
  int cph;                          // attention CTAs per kv head (2: each takes half of the group's q heads)
  const int8_t *w_lm;
  const egpt_qwen3_layer *layers;  // device array
  const uint16_t *embed, *final_norm, *rope_cos, *rope_sin;
  const void *s_lm;
  int64_t *token, *position;
  uint16_t *logits;
  unsigned long long *ll;           // LL words (layout: LLMap)
  float *lm_val;
  int *lm_idx;
  unsigned *lm_cnt;
  unsigned *epoch;
  int part_bytes, u_bytes;
  unsigned long long *trace;
  // tensor maps of the weights, [4 l + k] (k: q|k|v, o, gate|up, down) and [4 L] (lm_head), in the kernel's
  // parameter space (__grid_constant__)
  CUtensorMap maps[kMaxMaps];
};

// Per-stage description in shared memory (built once per launch; 32 bytes).
struct DStage {
  const CUtensorMap *map;
  const int8_t *w;
  const void *s;
  int k;               // columns
  short ntl;           // this CTA's tiles (tile t belongs to GEMV CTA t mod W)
  unsigned char nk;    // 256-column chunks
  unsigned char kind;
};
static_assert(sizeof(DStage) == 32, "stage table entry");

// ------------------------------------------------------------------------------------------------ LL words
__device__ __forceinline__ void ll_put(unsigned long long *p, uint32_t payload, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | payload;
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_get(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ void ll_get2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool ll_ok(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }

// Poll until word p carries `tag` (bounded); returns the word (whatever it holds after a timeout).
__device__ unsigned long long ll_wait(const unsigned long long *p, uint32_t tag) {
  unsigned long long w = ll_get(p);
  if (ll_ok(w, tag)) return w;
  const uint64_t t0 = globaltimer_ns();
  for (int it = 0;; ++it) {
    w = ll_get(p);
    if (ll_ok(w, tag)) return w;
    if ((it & 31) == 31) {
      if (device_error_set()) return w;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_device_error(EGPT_ERR_TIMEOUT);
        return w;
      }
    }
  }
}

// Word layout: per layer l (stride LW words) the input residual h_l (H/2; unused for l = 0), q|k|v ((NQ+2NKV)D/2),
// attention output (NQ D/2), mid residual (H/2), act (I/2); after the last layer h_L (H/2).
struct LLMap {
  int64_t LW, o_qkv, o_attn, o_mid, o_act;
  __device__ __forceinline__ LLMap(const Params &P) {
    o_qkv = P.H / 2;
    o_attn = o_qkv + (int64_t)(P.NQ + 2 * P.NKV) * P.D / 2;
    o_mid = o_attn + (int64_t)P.NQ * P.D / 2;
    o_act = o_mid + P.H / 2;
    LW = o_act + P.I / 2;
  }
};
__host__ __device__ inline int64_t ll_words(int L, int H, int NQ, int NKV, int D, int I) {
  return (int64_t)L * (H / 2 + (int64_t)(NQ + 2 * NKV) * D / 2 + (int64_t)NQ * D / 2 + H / 2 + I / 2) + H / 2;
}
// Tag of site (layer l, k: 0 q|k|v, 1 attention, 2 mid residual, 3 act, 4 next residual) of step `epoch`; never 0.
__device__ __forceinline__ uint32_t tag_of(const Params &P, unsigned epoch, int l, int k) {
  const unsigned long long n = (unsigned long long)epoch * (5ull * (unsigned long long)P.L) + 5ull * l + k;
  return (uint32_t)(n % 0xFFFFFFFFull) + 1u;
}

// ------------------------------------------------------------------------------------------------ mbarrier / TMA
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait (bounded by time only, whatever other waits reported) for copies still in flight before a CTA exits.
__device__ void mbar_drain(uint64_t *bar, unsigned parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(EGPT_ERR_TIMEOUT);
      return;
    }
}
// Bounded wait for the phase of parity `parity` to complete; false after a timeout or another wait's error.
__device__ bool mbar_wait(uint64_t *bar, unsigned parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (int it = 0;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 15) == 15) {
      if (device_error_set()) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_device_error(EGPT_ERR_TIMEOUT);
        return false;
      }
    }
  }
}
// One box {64 columns, 8 rows, 4 column steps} of a weight matrix viewed as [K/64][N][64] (no multicast; this
// GPU's memory only): 2 KB landing as [4 steps][8 rows][64 bytes].
__device__ __forceinline__ void tma_box(void *dst, const CUtensorMap *map, int row, int step, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)), "l"(map), "r"(0), "r"(row), "r"(step), "r"(smem_u32(bar))
      : "memory");
}
// Contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before its later async-proxy (TMA) writes.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }

// ------------------------------------------------------------------------------------------------ stage input
// RMSNorm weights of a stage input: thread t holds elements 4 (t + kCT j) .. + 3 as loaded bf16 pairs.
struct NormW {
  uint2 u[kMaxGroups];
  __device__ __forceinline__ float w(int e) const {
    const uint32_t x = (e & 2) ? u[e >> 2].y : u[e >> 2].x;
    return (e & 1) ? bf16_hi(x) : bf16_lo(x);
  }
};
__device__ __forceinline__ void load_norm(const uint16_t *nw, int64_t k, NormW &n) {
#pragma unroll
  for (int j = 0; j < kMaxGroups; ++j) {
    const int64_t i = 4 * ((int64_t)threadIdx.x + (int64_t)j * kCT);
    n.u[j] = make_uint2(0u, 0u);
    if (i < k) n.u[j] = *(const uint2 *)(nw + i);
  }
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__host__ __device__ __forceinline__ int x_stride(int64_t k) {
  return (int)((k + kChunkCols - 1) / kChunkCols * kChunkCols) + kXPad;
}

// Stage k values (k a multiple of 4) as the exact GEMV's fixed point: x = X 2^E, |X| < 2^30, four balanced
// base-256 digit planes in xd (zero-padded to whole 256-column chunks). Source: LL words with tag `tag`
// (polled), or plain bf16 values (the embedding row). nw: optional RMSNorm weights (HF rounding points).
// redd / redf: 16 doubles and 48 floats of scratch (redf[32..47]). Returns E.
__device__ int stage_input(const unsigned long long *words, const uint16_t *plain, int64_t k, uint32_t tag,
                           const NormW *nw, float eps, int8_t *xd, double *redd, float *redf) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  unsigned long long w[2 * kMaxGroups];
#pragma unroll
  for (int j = 0; j < kMaxGroups; ++j) {
    const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
    w[2 * j] = w[2 * j + 1] = 0ull;
    if (i < k) {
      if (words) {
        ll_get2(words + i / 2, w[2 * j], w[2 * j + 1]);
      } else {
        const uint2 u = __ldg((const uint2 *)(plain + i));
        w[2 * j] = u.x, w[2 * j + 1] = u.y;
      }
    }
  }
  if (words) {
    // Re-poll, all at once, the pairs whose tags are not there yet (one round trip per pass). Warp 0 polls first
    // while the other warps wait at a CTA barrier: its words come from producers all over the grid, so once they
    // are in the rest normally are too, and the CTA does not flood L2 with polls.
    if (warp != 0) csync();
    uint64_t t0 = 0;
    for (int it = 0;; ++it) {
      bool all = true;
#pragma unroll
      for (int j = 0; j < kMaxGroups; ++j) {
        const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
        if (i < k && !(ll_ok(w[2 * j], tag) && ll_ok(w[2 * j + 1], tag))) {
          ll_get2(words + i / 2, w[2 * j], w[2 * j + 1]);
          all = false;
        }
      }
      if (all) break;
      if ((it & 15) == 15) {
        if (t0 == 0) t0 = globaltimer_ns();
        if (device_error_set()) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_device_error(EGPT_ERR_TIMEOUT);
          break;
        }
      }
    }
    if (warp == 0) csync();
  }
  float v[4 * kMaxGroups];
#pragma unroll
  for (int j = 0; j < kMaxGroups; ++j) {
    const uint32_t a = (uint32_t)w[2 * j], b = (uint32_t)w[2 * j + 1];
    v[4 * j] = bf16_lo(a), v[4 * j + 1] = bf16_hi(a), v[4 * j + 2] = bf16_lo(b), v[4 * j + 3] = bf16_hi(b);
  }
  double ss = 0.0;
  float mx = 0.f;
#pragma unroll
  for (int e = 0; e < 4 * kMaxGroups; ++e) {
    ss += (double)(v[e] * v[e]);  // the square of a bf16 value is exact in fp32
    mx = fmaxf(mx, fabsf(nw ? v[e] * nw->w(e) : v[e]));
  }
  ss = warp_sum_d(ss);
  mx = warp_max(mx);
  if (lane == 0) redd[warp] = ss, redf[32 + warp] = mx;
  csync();
  double tot = 0.0;
  float bound = redf[32];
#pragma unroll
  for (int q = 0; q < kW; ++q) tot += redd[q];
#pragma unroll
  for (int q = 1; q < kW; ++q) bound = fmaxf(bound, redf[32 + q]);
  if (nw) {
    const float inv = rsqrtf((float)tot / (float)k + eps);
#pragma unroll
    for (int e = 0; e < 4 * kMaxGroups; ++e) v[e] = round_bf16(round_bf16(v[e] * inv) * nw->w(e));
    bound = bound * inv * 1.0079f;  // covers the two bf16 roundings of the norm
  }
  const int ex = bound > 0.f ? ((__float_as_int(bound) >> 23) & 0xFF) - 127 : 0;  // floor(log2 bound)
  const int E = ex - 29;
  const int xs = x_stride(k);
  const int64_t kpad = xs - kXPad;
#pragma unroll
  for (int j = 0; j < kMaxGroups; ++j) {
    const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
    if (i < kpad) {
      uint32_t word[4] = {0u, 0u, 0u, 0u};
      if (i < k) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          int d[4];
          ps::digits4(__float2int_rn(ps::mul_pow2(v[4 * j + q], -E)), d);
#pragma unroll
          for (int p = 0; p < 4; ++p) word[p] |= ((uint32_t)d[p] & 0xFFu) << (8 * q);
        }
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) *(uint32_t *)(xd + (int64_t)p * xs + i) = word[p];
    }
  }
  csync();
  return E;
}

// ------------------------------------------------------------------------------------------------ weight stream
// A warp's item stream: its items of every GEMV stage in order. Layer stage s: CTA items i = w, w + 16, ... of
// the stage's ntl * nk (tile-major: tile-local tl = i / nk, chunk c = i % nk); lm_head: the contiguous range
// [lm_lo(w), lm_lo(w + 1)) of those items, so every warp streams the same number of items to within one (whole
// tiles per warp left a quarter of the warps one tile, eight items, behind the rest).
struct Cursor {
  int s;   // stage (4 L + 1 = end)
  int i;   // layer stage: CTA item index; lm_head: tl * nk + c
};
__device__ __forceinline__ int stage_items(const DStage &sd) { return (int)sd.ntl * (int)sd.nk; }
// First lm_head item of warp w (w = kW: the end).
__device__ __forceinline__ int lm_lo(const DStage &sd, int w) { return (int)((int64_t)w * stage_items(sd) / kW); }

__device__ __forceinline__ void cur_seek(const DStage *stab, int nstages, Cursor &cu) {
  const int w = threadIdx.x >> 5;
  while (cu.s < nstages) {
    const DStage &sd = stab[cu.s];
    if (sd.kind == LMHEAD) {
      if (lm_lo(sd, w) < lm_lo(sd, w + 1)) {
        cu.i = lm_lo(sd, w);
        return;
      }
    } else if (w < stage_items(sd)) {
      cu.i = w;
      return;
    }
    ++cu.s;
  }
}
__device__ __forceinline__ void cur_next(const DStage *stab, int nstages, Cursor &cu) {
  const DStage &sd = stab[cu.s];
  if (sd.kind == LMHEAD) {
    ++cu.i;
    if (cu.i < lm_lo(sd, (threadIdx.x >> 5) + 1)) return;
  } else {
    cu.i += kW;
    if (cu.i < stage_items(sd)) return;
  }
  ++cu.s;
  cur_seek(stab, nstages, cu);
}

struct Ring {
  uint8_t *slots;    // this warp's rw slots
  uint64_t *full;    // this warp's rw barriers
  int rw;
  int n;             // items consumed by this warp so far
  int slot;          // n % rw
  unsigned phase;    // (n / rw) & 1
  Cursor fill;       // next item to issue
  int issued;        // items issued so far
};


// Lane 0: issue the fill cursor's item into slot `slot` (two boxes: rows 0-7 and 8-15 of the tile; gate|up: 8 gate
// rows and the 8 matching up rows).
__device__ __forceinline__ void issue_item(const Params &P, const DStage *stab, int nstages, int W, Ring &R, int slot) {
  if (R.fill.s >= nstages) return;
  const DStage &sd = stab[R.fill.s];
  const int tl = R.fill.i / sd.nk, c = R.fill.i - tl * sd.nk;
  const int tile = (int)blockIdx.x + W * tl;
  uint8_t *dst = R.slots + (size_t)slot * kItem;
  uint64_t *bar = R.full + slot;
  mbar_arrive_tx(bar, kItem);
  const int row0 = sd.kind == GATEUP ? tile * 8 : tile * 16;
  const int row8 = sd.kind == GATEUP ? P.I + tile * 8 : tile * 16 + 8;
  tma_box(dst, sd.map, row0, 4 * c, bar);
  tma_box(dst + 2048, sd.map, row8, 4 * c, bar);
  ++R.issued;
  cur_next(stab, nstages, R.fill);
}

// ------------------------------------------------------------------------------------------------ GEMV items
// Exact row sums of one item for lane (g, t): rows g and g + 8 of the tile against the four digit planes of
// columns [256 c, 256 c + 256). Slot layout (two boxes): [half][step][8 rows][64 bytes].
// The four 64-column steps accumulate in four independent registers sets (integer sums: the order does not matter),
// so the MMAs form chains of two instead of one chain of eight.
__device__ __forceinline__ void item_sums(const uint8_t *slot, const int8_t *xd, int c, int xs, int g, int t,
                                          int (&c4)[4]) {
  const int8_t *xb = xd + (int64_t)c * kChunkCols + g * xs + 16 * t;
  uint4 wa[4], wb[4], xv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    wa[j] = *(const uint4 *)(slot + j * 512 + g * 64 + 16 * t);
    wb[j] = *(const uint4 *)(slot + 2048 + j * 512 + g * 64 + 16 * t);
    xv[j] = make_uint4(0u, 0u, 0u, 0u);
    if (g < 4) xv[j] = *(const uint4 *)(xb + 64 * j);
  }
  int acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0;
    ps::mma_s8(acc[j], wa[j].x, wb[j].x, wa[j].y, wb[j].y, xv[j].x, xv[j].y);
    ps::mma_s8(acc[j], wa[j].z, wb[j].z, wa[j].w, wb[j].w, xv[j].z, xv[j].w);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) c4[r] += (acc[0][r] + acc[1][r]) + (acc[2][r] + acc[3][r]);
}
// Fold the digit-plane columns into the exact int64 sums of rows g (T0) and g + 8 (T1); valid in lanes t == 0.
__device__ __forceinline__ void fold_planes(const int (&c4)[4], long long &T0, long long &T1) {
  const int o0 = __shfl_down_sync(0xffffffffu, c4[0], 1), o1 = __shfl_down_sync(0xffffffffu, c4[1], 1);
  const int o2 = __shfl_down_sync(0xffffffffu, c4[2], 1), o3 = __shfl_down_sync(0xffffffffu, c4[3], 1);
  T0 = (long long)c4[0] + ((long long)c4[1] << 8) + ((long long)o0 << 16) + ((long long)o1 << 24);
  T1 = (long long)c4[2] + ((long long)c4[3] << 8) + ((long long)o2 << 16) + ((long long)o3 << 24);
}

// Consume the warp's next item: wait for its slot and run the MMAs (c4 accumulates; the caller zeroes it). The slot
// is refilled by refill(): right away in the lm_head stage, after the stage's last item in the layer stages, so that a
// TMA issue that has to wait for room in the copy engine's queue never delays the stage's own items.
__device__ __forceinline__ void refill(const Params &P, const DStage *stab, int nstages, int W, Ring &R);
__device__ __forceinline__ void consume(const Params &P, const DStage *stab, int nstages, int W, Ring &R,
                                        const int8_t *xd, int c, int xs, int (&c4)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (R.issued <= R.n) refill(P, stab, nstages, W, R);  // a stage with more items than ring slots: issue on demand
  // the MMAs are warp-wide: every lane takes the same branch
  if (__all_sync(0xffffffffu, mbar_wait(R.full + R.slot, R.phase)))
    item_sums(R.slots + (size_t)R.slot * kItem, xd, c, xs, g, t, c4);
  ++R.n;
  if (++R.slot == R.rw) R.slot = 0, R.phase ^= 1u;
}
// Refill every consumed slot that is still empty (the items `rw` positions ahead in the warp's stream).
__device__ __forceinline__ void refill(const Params &P, const DStage *stab, int nstages, int W, Ring &R) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    fence_async_smem();  // the warp's reads of the slots come before the TMA writes into them
    while (R.issued < R.n + R.rw && R.fill.s < nstages) issue_item(P, stab, nstages, W, R, R.issued % R.rw);
  }
  R.fill.s = __shfl_sync(0xffffffffu, R.fill.s, 0);
  R.fill.i = __shfl_sync(0xffffffffu, R.fill.i, 0);
  R.issued = __shfl_sync(0xffffffffu, R.issued, 0);
}

__device__ __forceinline__ float scale_of(const Params &P, uint32_t raw) {
  return P.scale_bf16 ? __uint_as_float(raw << 16) : __uint_as_float(raw);
}
__device__ __forceinline__ uint32_t raw_scale(const Params &P, const void *s, int64_t row) {
  return P.scale_bf16 ? (uint32_t)((const uint16_t *)s)[row] : __float_as_uint(((const float *)s)[row]);
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return (uint32_t)f32_to_bf16_bits(a) | ((uint32_t)f32_to_bf16_bits(b) << 16);
}

// Epilogue of one output word (rows 2 ep, 2 ep + 1 of tile-local tl; gate|up: act rows 8 tile + 2 ep, + 1 from gate
// rows 2 ep, 2 ep + 1 and up rows 8 + 2 ep, 8 + 2 ep + 1): the items' exact sums in chunk order, the reference's
// rounding points, one LL word out.
__device__ __forceinline__ void epilogue(const Params &P, const DStage &sd, const long long *part, int E,
                                         unsigned long long *out, uint32_t out_tag, const unsigned long long *res,
                                         uint32_t res_tag, int etl, int ep, int64_t etile, uint32_t s0, uint32_t s1,
                                         uint32_t s2, uint32_t s3, unsigned long long rw) {
  const int r0 = 2 * ep;
  long long A0 = 0, A1 = 0, B0 = 0, B1 = 0;
  for (int c = 0; c < sd.nk; ++c) {
    const long long *pp = part + (etl * sd.nk + c) * 16;
    A0 += pp[r0];
    A1 += pp[r0 + 1];
    if (sd.kind == GATEUP) {
      B0 += pp[8 + r0];
      B1 += pp[8 + r0 + 1];
    }
  }
  const float y0 = ps::mul_pow2(__ll2float_rn(A0), E), y1 = ps::mul_pow2(__ll2float_rn(A1), E);
  uint32_t payload;
  if (sd.kind == QKV) {
    payload = pack2(y0 * scale_of(P, s0), y1 * scale_of(P, s1));
  } else if (sd.kind == GATEUP) {
    const float g0 = round_bf16(y0 * scale_of(P, s0)), g1 = round_bf16(y1 * scale_of(P, s1));
    const float u0 = round_bf16(ps::mul_pow2(__ll2float_rn(B0), E) * scale_of(P, s2));
    const float u1 = round_bf16(ps::mul_pow2(__ll2float_rn(B1), E) * scale_of(P, s3));
    payload = pack2(round_bf16(g0 / (1.0f + expf(-g0))) * u0, round_bf16(g1 / (1.0f + expf(-g1))) * u1);
  } else {
    if (res && !ll_ok(rw, res_tag)) rw = ll_wait(res + etile * 8 + ep, res_tag);
    const uint32_t r = (uint32_t)rw;
    payload = pack2(bf16_lo(r) + round_bf16(y0 * scale_of(P, s0)), bf16_hi(r) + round_bf16(y1 * scale_of(P, s1)));
  }
  const int64_t word = sd.kind == GATEUP ? etile * 4 + ep : etile * 8 + ep;
  ll_put(out + word, payload, out_tag);
}

// A layer GEMV stage of this CTA: each warp consumes its items (their exact row sums go to `part`), then epilogue
// unit e (one output word) finishes; its scales and residual word were requested before the items. out: the
// stage's output words; res: residual words (o_proj, down_proj; null with res_plain: the embedding row of
// layer 0) with tag res_tag.
template <bool TRACE>
__device__ void gemv_stage(const Params &P, const DStage *stab, int nstages, int W, int s, Ring &R, Cursor &cur,
                           const int8_t *xd, int E, long long *part, unsigned long long *out, uint32_t out_tag,
                           const unsigned long long *res, const uint16_t *res_plain, uint32_t res_tag, int tslot) {
  const DStage &sd = stab[s];
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int per = sd.kind == GATEUP ? 4 : 8;  // output words per tile
  const int e = threadIdx.x;
  const bool epi = e < sd.ntl * per;
  const int etl = e / per, ep = e - etl * per;
  const int64_t etile = blockIdx.x + (int64_t)W * etl;
  uint32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  unsigned long long rw = 0ull;
  if (epi) {
    if (sd.kind == GATEUP) {
      s0 = raw_scale(P, sd.s, etile * 8 + 2 * ep), s1 = raw_scale(P, sd.s, etile * 8 + 2 * ep + 1);
      s2 = raw_scale(P, sd.s, P.I + etile * 8 + 2 * ep), s3 = raw_scale(P, sd.s, P.I + etile * 8 + 2 * ep + 1);
    } else {
      s0 = raw_scale(P, sd.s, etile * 16 + 2 * ep), s1 = raw_scale(P, sd.s, etile * 16 + 2 * ep + 1);
      if (sd.kind == OPROJ || sd.kind == DOWN) {
        const int64_t wi = etile * 8 + ep;  // residual word of rows 2 wi, 2 wi + 1
        if (res)
          rw = ll_get(res + wi);
        else
          rw = (unsigned long long)*(const uint32_t *)(res_plain + 2 * wi);
      }
    }
  }
  const int xs = x_stride(sd.k);
  while (cur.s == s) {
    const int i = cur.i;
    const int tl = i / sd.nk, c = i - tl * sd.nk;
    int c4[4] = {0, 0, 0, 0};
    consume(P, stab, nstages, W, R, xd, c, xs, c4);
    long long T0, T1;
    fold_planes(c4, T0, T1);
    if (t == 0) {
      part[i * 16 + g] = T0;
      part[i * 16 + g + 8] = T1;
    }
    cur_next(stab, nstages, cur);
  }
  csync();  // every item's sums are in `part`
  if (TRACE && tslot >= 0 && P.trace && threadIdx.x == 0) P.trace[tslot] = globaltimer_ns();
  if (epi) epilogue(P, sd, part, E, out, out_tag, res, res_tag, etl, ep, etile, s0, s1, s2, s3, rw);
  refill(P, stab, nstages, W, R);  // off the stage's critical path: the outputs are out
  if (TRACE && tslot >= 0 && P.trace) {
    csync();
    if (threadIdx.x == 0) P.trace[tslot + 1] = globaltimer_ns();
  }
}

// lm_head stage: the warp's range of items; a tile it covers whole is finished in the warp (bf16 logits, argmax),
// the row sums of a tile it covers in part go to shared memory (slot 2w: the range's first tile, 2w + 1: its last),
// and after a CTA barrier warp 0 adds the partial sums of each such tile (integers: exact in any order) and
// finishes it. lm_part: kLmSlots x 16 row sums, then kLmSlots tile ids (-1: unused).
constexpr int kLmSlots = 2 * kW;
constexpr size_t kLmPartBytes = (size_t)kLmSlots * 16 * 8 + (size_t)kLmSlots * 8;
struct Best {
  float v;
  int i;
};
__device__ __forceinline__ void lm_finish(const Params &P, const DStage &sd, int W, int tl, int r, long long T, int E,
                                          float sc, Best &best) {
  const int64_t row = ((int64_t)blockIdx.x + (int64_t)W * tl) * 16 + r;
  const float l = round_bf16(ps::mul_pow2(__ll2float_rn(T), E) * sc);
  if (P.logits) P.logits[row] = f32_to_bf16_bits(l);
  if (argmax_better(l, (int)row, best.v, best.i)) best.v = l, best.i = (int)row;
}
__device__ void lm_stage(const Params &P, const DStage *stab, int nstages, int W, int s, Ring &R, Cursor &cur,
                         const int8_t *xd, int E, Best &best, long long *lm_part) {
  const DStage &sd = stab[s];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int xs = x_stride(sd.k);
  const int lo = lm_lo(sd, warp);
  long long *slot_tile = lm_part + kLmSlots * 16;
  if (lane < 2) slot_tile[2 * warp + lane] = -1;
  int c4[4] = {0, 0, 0, 0};
  float s0 = 0.f, s1 = 0.f;
  while (cur.s == s) {
    const int i = cur.i;
    const int tl = i / sd.nk, c = i - tl * sd.nk;
    if ((c == 0 || i == lo) && t == 0) {  // the tile's scales, requested before its items
      const int64_t tile = blockIdx.x + (int64_t)W * tl;
      s0 = scale_of(P, raw_scale(P, sd.s, tile * 16 + g)), s1 = scale_of(P, raw_scale(P, sd.s, tile * 16 + g + 8));
    }
    consume(P, stab, nstages, W, R, xd, c, xs, c4);
    refill(P, stab, nstages, W, R);
    cur_next(stab, nstages, cur);
    const bool range_end = cur.s != s;
    if (c != sd.nk - 1 && !range_end) continue;
    long long T0, T1;
    fold_planes(c4, T0, T1);
    c4[0] = c4[1] = c4[2] = c4[3] = 0;
    const bool whole = tl * sd.nk >= lo && c == sd.nk - 1;
    if (whole) {
      if (t == 0) {
        lm_finish(P, sd, W, tl, g, T0, E, s0, best);
        lm_finish(P, sd, W, tl, g + 8, T1, E, s1, best);
      }
    } else {
      const int slot = tl * sd.nk < lo ? 2 * warp : 2 * warp + 1;
      if (t == 0) lm_part[slot * 16 + g] = T0, lm_part[slot * 16 + g + 8] = T1;
      if (lane == 0) slot_tile[slot] = tl;
    }
  }
  csync();  // every partial row sum is in shared memory
  if (warp == 0) {
    // the slots in order hold the partial tiles in item order, so the parts of one tile are consecutive
    const int r = lane & 15;
    long long acc = 0;
    int cur_tile = -1;
    for (int sl = 0; sl < kLmSlots; ++sl) {
      const int tile_id = (int)slot_tile[sl];
      if (tile_id < 0) continue;
      if (tile_id != cur_tile) {
        if (cur_tile >= 0 && lane < 16) {
          const int64_t tile = blockIdx.x + (int64_t)W * cur_tile;
          lm_finish(P, sd, W, cur_tile, r, acc, E, scale_of(P, raw_scale(P, sd.s, tile * 16 + r)), best);
        }
        cur_tile = tile_id;
        acc = 0;
      }
      acc += lm_part[sl * 16 + r];
    }
    if (cur_tile >= 0 && lane < 16) {
      const int64_t tile = blockIdx.x + (int64_t)W * cur_tile;
      lm_finish(P, sd, W, cur_tile, r, acc, E, scale_of(P, raw_scale(P, sd.s, tile * 16 + r)), best);
    }
  }
}

// ------------------------------------------------------------------------------------------------ attention
// Cached K and V rows [0, n) of kv head g of layer l into the shared-memory copies (one bulk copy each).
template <int D>
__device__ __forceinline__ void kv_load(const Params &P, int l, int g, int64_t n, uint16_t *Ks, uint16_t *Vs,
                                        uint64_t *bar) {
  const egpt_qwen3_layer &Ly = P.layers[l];
  const size_t bytes = (size_t)n * D * 2;
  const int64_t base = (int64_t)g * P.cap * D;
  mbar_arrive_tx(bar, (unsigned)(2 * bytes));
  if (bytes) {
    bulk_copy(Ks, (const uint16_t *)Ly.k_cache + base, (unsigned)bytes, bar);
    bulk_copy(Vs, (const uint16_t *)Ly.v_cache + base, (unsigned)bytes, bar);
  }
}

// Scratch of the shared-memory attention, carved behind the K and V copies (cap rows each), in floats:
// scores [GRP][capr] | block maxima [GRP][kMaxBlk] (order-preserving ints) | numerators [kW][GRP][D] |
// denominators [kW][GRP]; capr = cap rounded up to 8.
constexpr int kMaxBlk = 8;  // 128-key blocks: caches of at most 1024 rows
__host__ __device__ inline int64_t smem_attn_floats(int64_t cap, int grp, int d) {
  return grp * ((cap + 7) / 8 * 8) + grp * kMaxBlk + (int64_t)kW * grp * d + kW * grp;
}
__device__ __forceinline__ int ord_enc(float f) {  // int order == float order
  const int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float ord_dec(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff); }

// Sums of NV partial values over the 32 lanes (NV = 8, 16 or 32), halving the set at each butterfly step: after
// the call lane l holds the full sum of value l >> (5 - log2 NV) in v[0]. About NV shuffles in all instead of 5 NV.
template <int NV>
__device__ __forceinline__ void reduce_scatter(float (&v)[NV]) {
  const int lane = threadIdx.x & 31;
  int n = NV;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool up = lane & o;
      const int h = n / 2;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        if (i < h) {
          const float send = up ? v[i] : v[i + h];
          const float keep = up ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
}

// Attention over the n keys whose K and V rows sit in shared memory (Ks, Vs: [n][D] bf16), q heads in q (fp32 values
// of bf16 numbers), with the reference GPU kernel's probability rounding: the keys are walked in 128-key blocks
// with a running maximum m_b, p = exp(s - m_b) enters P.V rounded to bf16 and the denominator in fp32, and the
// blocks are brought to the final maximum by exp(m_b - m_final).
//   Scores: warp w takes the 8-key groups w, w + 16, ...; lane l holds dims [l DPL, (l + 1) DPL) of q and of the 8
//   keys, so GRP x 8 partial dot products per lane, summed over the lanes by one reduce-scatter; each group's
//   maximum per head goes to the block maxima by a shared atomic max.
//   P.V: warp w takes the keys [w ck, (w + 1) ck), ck = ceil(n / 16); lane i of a round of 32 computes p of the
//   round's key i (block maxima read directly), then each key's p is broadcast and every lane accumulates its
//   dims; the 16 warps' sums merge in a fixed order in the caller. The block maxima must hold ord_enc(-inf) on
//   entry.
template <int DPL, int GRP>
__device__ void attn_smem(const uint16_t *Ks, const uint16_t *Vs, int n, const float (*q)[DPL * 32], float scale,
                          float *sc, int capr, int *bm, float *wacc, float *wl) {
  constexpr int D = DPL * 32, NV = GRP * 8;
  static_assert(NV == 8 || NV == 16 || NV == 32, "1, 2 or 4 q heads");
  constexpr int SH = NV == 8 ? 2 : NV == 16 ? 1 : 0;  // lane l holds value l >> SH after the reduce-scatter
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float qr[GRP][DPL];
#pragma unroll
  for (int j = 0; j < GRP; ++j)
#pragma unroll
    for (int i = 0; i < DPL; ++i) qr[j][i] = q[j][lane * DPL + i];
  const int ngr = (n + 7) / 8;
  for (int gq = warp; gq < ngr; gq += kW) {
    float v[NV];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int key = min(8 * gq + kk, n - 1);  // past the end: a valid row, its sums are dropped
      float kv[DPL];
      if (DPL == 4) {
        const uint2 u = *(const uint2 *)(Ks + (int64_t)key * D + lane * 4);
        kv[0] = bf16_lo(u.x), kv[1 % DPL] = bf16_hi(u.x), kv[2 % DPL] = bf16_lo(u.y), kv[3 % DPL] = bf16_hi(u.y);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) kv[i] = bf16_bits_to_f32(Ks[(int64_t)key * D + lane * DPL + i]);
      }
#pragma unroll
      for (int j = 0; j < GRP; ++j) {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) d = fmaf(qr[j][i], kv[i], d);
        v[j * 8 + kk] = d;
      }
    }
    reduce_scatter<NV>(v);
    const int idx = lane >> SH;  // value held: head idx / 8, key 8 gq + idx % 8
    const int j = idx >> 3, key = 8 * gq + (idx & 7);
    const float sv = v[0] * scale;
    float m = key < n ? sv : -INFINITY;
    // maximum over the group's 8 keys of head j: the 8 keys' lanes are 2^SH apart, within one head's run of lanes
#pragma unroll
    for (int o = 1 << SH; o < (8 << SH); o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const bool writer = (lane & ((1 << SH) - 1)) == 0;
    if (writer && key < n) sc[j * capr + key] = sv;
    if (writer && (idx & 7) == 0) atomicMax(&bm[j * kMaxBlk + key / kRefBlock], ord_enc(m));
  }
  csync();
  const int nblk = (n + kRefBlock - 1) / kRefBlock;
  float mfin[GRP];
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    float mm = -INFINITY;
    for (int b = 0; b < nblk; ++b) mm = fmaxf(mm, ord_dec(bm[j * kMaxBlk + b]));
    mfin[j] = mm;
  }
  float acc[GRP][DPL], l[GRP];
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[j][i] = 0.f;
  }
  const int ck = (n + kW - 1) / kW, kend = min(n, (warp + 1) * ck);  // warp w: keys [w ck, (w + 1) ck)
  for (int r0 = warp * ck; r0 < kend; r0 += 32) {
    const int kk = r0 + lane;  // lane i: key r0 + i of this round
    float pw[GRP];
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      pw[j] = 0.f;
      if (kk < kend) {
        const int b = kk / kRefBlock;
        float mb = -INFINITY;
        for (int c = 0; c <= b; ++c) mb = fmaxf(mb, ord_dec(bm[j * kMaxBlk + c]));  // running max after block b
        const float p = expf(sc[j * capr + kk] - mb);
        const float f = expf(mb - mfin[j]);
        l[j] = fmaf(p, f, l[j]);
        pw[j] = round_bf16(p) * f;
      }
    }
    const int cnt = min(32, kend - r0);
    for (int i = 0; i < cnt; ++i) {
      const int k = r0 + i;
      float vv[DPL];
      if (DPL == 4) {
        const uint2 u = *(const uint2 *)(Vs + (int64_t)k * D + lane * 4);
        vv[0] = bf16_lo(u.x), vv[1 % DPL] = bf16_hi(u.x), vv[2 % DPL] = bf16_lo(u.y), vv[3 % DPL] = bf16_hi(u.y);
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) vv[e] = bf16_bits_to_f32(Vs[(int64_t)k * D + lane * DPL + e]);
      }
#pragma unroll
      for (int j = 0; j < GRP; ++j) {
        const float pk = __shfl_sync(0xffffffffu, pw[j], i);
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[j][e] = fmaf(pk, vv[e], acc[j][e]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    const float lt = warp_sum(l[j]);
    if (lane == 0) wl[warp * GRP + j] = lt;
#pragma unroll
    for (int e = 0; e < DPL; ++e) wacc[(warp * GRP + j) * D + lane * DPL + e] = acc[j][e];
  }
  csync();
}

// Attention of kv head g for this step, q heads [head0, head0 + GRP) of its group (one CTA; with two CTAs per kv
// head each takes half of the group): those q heads and the new k row from the q|k|v words
// (normalised and rotated by one warp each), the new k and v rows appended to the cache (and to the shared-memory
// copies Ks / Vs when those hold the cache), then attention over keys [0, pos] (attn_smem on the shared-memory
// copies, else the attention core of attention.cu: both the reference GPU kernel's 128-key block walk), and the
// group's output published as LL words.
template <int DPL, int GRP, bool TRACE>
__device__ void attention_ll(const Params &P, const egpt_qwen3_layer &Ly, int g, int head0, int64_t pos,
                             const unsigned long long *qkv_w, uint32_t qkv_tag, unsigned long long *out_w,
                             uint32_t out_tag, float *u, uint16_t *Ks, uint16_t *Vs, int tslot) {
  constexpr int D = DPL * 32;
  AttnScratch<DPL, GRP> &S = *reinterpret_cast<AttnScratch<DPL, GRP> *>(u);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint16_t *kc = (uint16_t *)Ly.k_cache, *vc = (uint16_t *)Ly.v_cache;
  const int64_t kv_base = (int64_t)g * P.cap * D;
  if (warp <= GRP + 1) {
    const int head = warp < GRP ? head0 + warp : warp == GRP ? P.NQ + g : P.NQ + P.NKV + g;
    const int64_t e0 = (int64_t)head * D + lane * DPL;  // first element of this lane
    float v[DPL];
    if (DPL >= 2) {
#pragma unroll
      for (int i = 0; i < DPL; i += 2) {
        const uint32_t w = (uint32_t)ll_wait(qkv_w + (e0 + i) / 2, qkv_tag);
        v[i] = bf16_lo(w);
        v[i + 1] = bf16_hi(w);
      }
    } else {
      const uint32_t w = (uint32_t)ll_wait(qkv_w + e0 / 2, qkv_tag);
      v[0] = (e0 & 1) ? bf16_hi(w) : bf16_lo(w);
    }
    if (warp == GRP + 1) {  // v row: appended as is
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        vc[kv_base + pos * D + lane * DPL + i] = f32_to_bf16_bits(v[i]);
        if (Vs) Vs[pos * D + lane * DPL + i] = f32_to_bf16_bits(v[i]);
      }
    } else {
      const bool isk = warp == GRP;
      const uint16_t *nw = (const uint16_t *)(isk ? Ly.k_norm : Ly.q_norm) + lane * DPL;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) ss = fmaf(v[i], v[i], ss);
      const float inv = rsqrtf(warp_sum(ss) / (float)D + P.eps);
      constexpr int half = D / 2;
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[i] = round_bf16(round_bf16(v[i] * inv) * bf16_bits_to_f32(nw[i]));
#pragma unroll
      for (int i = 0; i < DPL; ++i) {  // element e pairs with e +- D/2, held DPL * 16 elements = 16 lanes away
        const int e = lane * DPL + i, r = e < half ? e : e - half;
        const float cs = bf16_bits_to_f32(P.rope_cos[pos * half + r]), sn = bf16_bits_to_f32(P.rope_sin[pos * half + r]);
        const float other = __shfl_xor_sync(0xffffffffu, v[i], 16);
        const float rot = lane < 16 ? -other : other;
        const float o = round_bf16(round_bf16(v[i] * cs) + round_bf16(rot * sn));
        if (isk) {
          kc[kv_base + pos * D + lane * DPL + i] = f32_to_bf16_bits(o);
          if (Ks) Ks[pos * D + lane * DPL + i] = f32_to_bf16_bits(o);
        } else {
          S.q[warp][lane * DPL + i] = o;
        }
      }
    }
  }
  if (threadIdx.x < GRP) S.mb[threadIdx.x] = -INFINITY;
  if (Ks && threadIdx.x < GRP * kMaxBlk)  // block maxima of the shared-memory attention
    ((int *)((float *)(Vs + P.cap * D) + GRP * ((P.cap + 7) / 8 * 8)))[threadIdx.x] = ord_enc(-INFINITY);
  __threadfence();
  csync();
  if (TRACE && tslot >= 0 && P.trace && threadIdx.x == 0) P.trace[tslot] = globaltimer_ns();
  if (Ks) {  // K and V rows in shared memory
    const int capr = (P.cap + 7) / 8 * 8;
    float *sc = (float *)(Vs + P.cap * D);
    int *bm = (int *)(sc + GRP * capr);
    float *wacc = (float *)(bm + GRP * kMaxBlk), *wl = wacc + kW * GRP * D;
    attn_smem<DPL, GRP>(Ks, Vs, (int)(pos + 1), S.q, P.scale, sc, capr, bm, wacc, wl);
    // merge of the 16 warps' sums in a fixed order: 4 parts of 4 warps each (into the part's first warp's slot),
    // then the 4 parts
    constexpr int NW = GRP * D / 2;  // output words (two dims each)
    for (int t = threadIdx.x; t < 4 * NW; t += kCT) {
      const int idx = t % NW, part = t / NW;
      const int j = (2 * idx) / D, dd = 2 * idx - j * D, w0 = 4 * part;
      float num0 = 0.f, num1 = 0.f;
#pragma unroll
      for (int w = w0; w < w0 + 4; ++w) {
        num0 += wacc[(w * GRP + j) * D + dd];
        num1 += wacc[(w * GRP + j) * D + dd + 1];
      }
      wacc[(w0 * GRP + j) * D + dd] = num0;
      wacc[(w0 * GRP + j) * D + dd + 1] = num1;
    }
    csync();
    for (int idx = threadIdx.x; idx < NW; idx += kCT) {
      const int j = (2 * idx) / D, dd = 2 * idx - j * D;
      float num0 = 0.f, num1 = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) den += wl[w * GRP + j];
#pragma unroll
      for (int w = 0; w < kW; w += 4) {
        num0 += wacc[(w * GRP + j) * D + dd];
        num1 += wacc[(w * GRP + j) * D + dd + 1];
      }
      ll_put(out_w + ((int64_t)head0 * D) / 2 + idx, pack2(num0 / den, num1 / den), out_tag);
    }
    if (TRACE && tslot >= 0 && P.trace) {
      csync();
      if (threadIdx.x == 0) P.trace[tslot + 1] = globaltimer_ns();
    }
    return;
  }
  AttnTask tk;
  tk.K = Ks ? (const void *)Ks : (const void *)(kc + kv_base);
  tk.V = Vs ? (const void *)Vs : (const void *)(vc + kv_base);
  tk.k0 = 0;
  tk.k1 = pos + 1;
  tk.scale = P.scale;
  tk.prefetch_v = Vs ? 0 : 1;  // rows in shared memory: nothing to prefetch
  attn_walk<DPL, GRP, true, kCT, false>(tk, S);
  csync();
  const int64_t ntiles = (tk.k1 - tk.k0 + kKeyTile - 1) / kKeyTile;
  const int busy = (int)min((int64_t)kAttnWarps, ntiles);
  // merge the warps in a fixed order (the arithmetic of attn_finish), two output elements per word
  for (int idx = threadIdx.x; idx < GRP * D / 2; idx += kCT) {
    const int j = (2 * idx) / D, dd = 2 * idx - j * D;
    float M = -INFINITY;
    for (int w = 0; w < busy; ++w) M = fmaxf(M, S.w_m[w][j]);
    float lsum = 0.f, a0 = 0.f, a1 = 0.f;
    for (int w = 0; w < busy; ++w) {
      if (S.w_l[w][j] == 0.f) continue;
      const float f = expf(S.w_m[w][j] - M);
      lsum += S.w_l[w][j] * f;
      a0 += S.w_acc[w][j][dd] * f;
      a1 += S.w_acc[w][j][dd + 1] * f;
    }
    ll_put(out_w + ((int64_t)head0 * D) / 2 + idx, pack2(a0 / lsum, a1 / lsum), out_tag);
  }
  if (TRACE && tslot >= 0 && P.trace) {
    csync();
    if (threadIdx.x == 0) P.trace[tslot + 1] = globaltimer_ns();
  }
}

// L2 prefetch of kv head g's cached K and V rows [0, pos) (attention from global memory).
template <int D>
__device__ __forceinline__ void prefetch_kv(const Params &P, const egpt_qwen3_layer &Ly, int g, int64_t pos) {
  constexpr int lines = D * 2 / 128 > 0 ? D * 2 / 128 : 1;
  const int64_t n = pos * lines;
  const char *kb = (const char *)Ly.k_cache + (int64_t)g * P.cap * D * 2;
  const char *vb = (const char *)Ly.v_cache + (int64_t)g * P.cap * D * 2;
  for (int64_t i = threadIdx.x; i < 2 * n; i += kCT) {
    const char *a = (i < n ? kb : vb) + (i < n ? i : i - n) * 128;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
  }
}

template <bool TRACE>
__device__ __forceinline__ void stamp(const Params &P, int k) {
  if (TRACE && P.trace && threadIdx.x == 0) P.trace[k] = globaltimer_ns();
}

// ------------------------------------------------------------------------------------------------ kernel
template <int DPL, int GRP, bool TRACE>
__global__ void __launch_bounds__(kCT, 1) dataflow_step_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = DPL * 32;
  const int nstages = 4 * P.L + 1;
  const int W = (int)gridDim.x - P.NKV * P.cph;        // GEMV CTAs
  const int attn_a = (int)blockIdx.x - W;               // >= 0: this CTA runs attention
  const int attn_g = attn_a >= 0 ? attn_a / P.cph : -1;  // its kv head
  const int attn_part = attn_a >= 0 ? attn_a % P.cph : 0;  // and which part of the group's q heads
  // layout: scratch 512 B | stage table | barriers | part | union(digit planes, attention scratch) | rings / K, V
  float *redf = (float *)smem;
  double *redd = (double *)smem;  // first 16 doubles overlap redf[0..31]
  int *s_flag = (int *)(smem + 256);
  float *s_bv = (float *)(smem + 320);
  int *s_bi = (int *)(smem + 384);
  DStage *stab = (DStage *)(smem + 512);
  size_t off = 512 + ((size_t)nstages * sizeof(DStage) + 127) / 128 * 128;
  uint64_t *bars = (uint64_t *)(smem + off);             // kW * rw ring barriers, then the K/V barrier
  off += ((size_t)(kW * P.rw + 1) * 8 + 127) / 128 * 128;
  long long *part = (long long *)(smem + off);
  off += P.part_bytes;
  float *u = (float *)(smem + off);
  int8_t *xd = (int8_t *)u;
  off += P.u_bytes;
  uint8_t *big = smem + off;                              // GEMV CTAs: rings; attention CTAs: K and V rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < nstages; i += kCT) {
    DStage d;
    int n, k, kind;
    const void *sp;
    if (i == 4 * P.L) {
      sp = P.s_lm, n = (int)P.V, k = P.H, kind = LMHEAD;
    } else {
      const egpt_qwen3_layer &Ly = P.layers[i >> 2];
      switch (i & 3) {
        case 0: sp = Ly.s_qkv, n = (P.NQ + 2 * P.NKV) * P.D, k = P.H, kind = QKV; break;
        case 1: sp = Ly.s_o, n = P.H, k = P.NQ * P.D, kind = OPROJ; break;
        case 2: sp = Ly.s_gu, n = 2 * P.I, k = P.H, kind = GATEUP; break;
        default: sp = Ly.s_down, n = P.H, k = P.I, kind = DOWN; break;
      }
    }
    const int tiles = n / 16;
    d.map = &P.maps[i];
    d.w = i == 4 * P.L ? P.w_lm
                       : (i & 3) == 0 ? P.layers[i >> 2].w_qkv
                       : (i & 3) == 1 ? P.layers[i >> 2].w_o
                       : (i & 3) == 2 ? P.layers[i >> 2].w_gu : P.layers[i >> 2].w_down;
    d.s = sp;
    d.k = k;
    d.kind = (unsigned char)kind;
    d.nk = (unsigned char)((k + kChunkCols - 1) / kChunkCols);
    d.ntl = (short)(attn_g < 0 && (int)blockIdx.x < tiles ? (tiles - (int)blockIdx.x + W - 1) / W : 0);
    stab[i] = d;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s <= kW * P.rw; ++s) mbar_init(bars + s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  __syncthreads();

  // ---------------------------------------------------------------- step state
  const unsigned epoch = *(volatile unsigned *)P.epoch;
  const int64_t pos = *P.position;
  const int64_t tok = *P.token;
  bool ok = true;
  if (pos < 0 || pos >= P.cap || tok < 0 || tok >= P.V) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    ok = false;
  }
  const uint16_t *emb = P.embed + (ok ? tok : 0) * P.H;
  const LLMap M(P);
  if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 0);

  if (attn_g >= 0) {
    // ------------------------------------------------------------ attention CTA: every layer's kv head attn_g
    uint64_t *kvbar = bars + kW * P.rw;
    uint16_t *Ks = P.kv_smem ? (uint16_t *)big : nullptr;
    uint16_t *Vs = P.kv_smem ? (uint16_t *)big + P.cap * D : nullptr;
    int kv_pending = -1;  // layer whose K/V copy is in flight and not yet waited for
    if (ok && Ks) {
      if (threadIdx.x == 0) kv_load<D>(P, 0, attn_g, pos, Ks, Vs, kvbar);
      kv_pending = 0;
    }
    for (int l = 0; l < P.L; ++l) {
      const egpt_qwen3_layer &Ly = P.layers[l];
      unsigned long long *lw = P.ll + (int64_t)l * M.LW;
      if (ok && !Ks) prefetch_kv<D>(P, Ly, attn_g, pos);
      if (ok && Ks) {
        if (mbar_wait(kvbar, (unsigned)l & 1u))
          kv_pending = -1;
        else
          ok = false;
      }
      if (ok) {
        const int tslot = (TRACE && attn_a == 0) ? 3 + 5 * P.L + 10 * l + 2 : -1;
        if (GRP >= 2 && P.cph == 2)
          attention_ll<DPL, (GRP >= 2 ? GRP / 2 : 1), TRACE>(P, Ly, attn_g, attn_g * GRP + attn_part * (GRP / 2), pos,
                                                         lw + M.o_qkv, tag_of(P, epoch, l, 0), lw + M.o_attn,
                                                         tag_of(P, epoch, l, 1), u, Ks, Vs, tslot);
        else
          attention_ll<DPL, GRP, TRACE>(P, Ly, attn_g, attn_g * GRP, pos, lw + M.o_qkv, tag_of(P, epoch, l, 0),
                                        lw + M.o_attn, tag_of(P, epoch, l, 1), u, Ks, Vs, tslot);
        if (TRACE && attn_a == 0) stamp<TRACE>(P, 2 + 5 * l);
      } else {  // bad position or a failed copy: publish zeros so that no consumer waits for this head
        const int gh = GRP / P.cph;  // this CTA's q heads
        for (int idx = threadIdx.x; idx < gh * D / 2; idx += kCT)
          ll_put(lw + M.o_attn + ((int64_t)(attn_g * GRP + attn_part * gh) * D) / 2 + idx, 0u, tag_of(P, epoch, l, 1));
      }
      csync();  // the copies' rows and the attention scratch are free again
      if (ok && Ks && l + 1 < P.L) {
        if (threadIdx.x == 0) {
          fence_async_smem();
          kv_load<D>(P, l + 1, attn_g, pos, Ks, Vs, kvbar);
        }
        kv_pending = l + 1;
      }
    }
    if (kv_pending >= 0 && threadIdx.x == 0) mbar_drain(kvbar, (unsigned)kv_pending & 1u);  // none in flight at exit
  } else {
    // ------------------------------------------------------------ GEMV CTA
    Ring R;
    R.rw = P.rw;
    R.slots = big + (size_t)warp * P.rw * kItem;
    R.full = bars + warp * P.rw;
    R.n = 0;
    R.slot = 0;
    R.phase = 0u;
    R.issued = 0;
    R.fill.s = 0;
    R.fill.i = 0;
    cur_seek(stab, nstages, R.fill);
    if (lane == 0) {
      for (int k = 0; k < P.rw; ++k) issue_item(P, stab, nstages, W, R, k);
    }
    R.fill.s = __shfl_sync(0xffffffffu, R.fill.s, 0);
    R.fill.i = __shfl_sync(0xffffffffu, R.fill.i, 0);
    R.issued = __shfl_sync(0xffffffffu, R.issued, 0);
    Cursor cur;
    cur.s = 0;
    cur.i = 0;
    cur_seek(stab, nstages, cur);
    NormW nw;
    for (int l = 0; l < P.L; ++l) {
      const egpt_qwen3_layer &Ly = P.layers[l];
      unsigned long long *lw = P.ll + (int64_t)l * M.LW;
      const unsigned long long *h_in = l == 0 ? nullptr : lw;  // layer 0: the embedding row
      // q|k|v = Wqkv . RMSNorm(h)
      if (stab[4 * l].ntl > 0) {
        load_norm((const uint16_t *)Ly.ln_in, P.H, nw);
        const int E = stage_input(h_in, emb, P.H, tag_of(P, epoch, l - 1, 4), &nw, P.eps, xd, redd, redf);
        if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 1 + 5 * l);
        gemv_stage<TRACE>(P, stab, nstages, W, 4 * l, R, cur, xd, E, part, lw + M.o_qkv, tag_of(P, epoch, l, 0),
                          nullptr, nullptr, 0u, blockIdx.x == 0 ? 3 + 5 * P.L + 10 * l + 0 : -1);
      }
      // h_mid = h + Wo . attn
      if (stab[4 * l + 1].ntl > 0) {
        const int E = stage_input(lw + M.o_attn, nullptr, (int64_t)P.NQ * P.D, tag_of(P, epoch, l, 1), nullptr,
                                  P.eps, xd, redd, redf);
        if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 3 + 5 * l);
        gemv_stage<TRACE>(P, stab, nstages, W, 4 * l + 1, R, cur, xd, E, part, lw + M.o_mid, tag_of(P, epoch, l, 2),
                          h_in, emb, tag_of(P, epoch, l - 1, 4), blockIdx.x == 0 ? 3 + 5 * P.L + 10 * l + 4 : -1);
      }
      // act = silu(Wg . RMSNorm(h_mid)) * (Wu . RMSNorm(h_mid))
      if (stab[4 * l + 2].ntl > 0) {
        load_norm((const uint16_t *)Ly.ln_post, P.H, nw);
        const int E = stage_input(lw + M.o_mid, nullptr, P.H, tag_of(P, epoch, l, 2), &nw, P.eps, xd, redd, redf);
        if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 4 + 5 * l);
        gemv_stage<TRACE>(P, stab, nstages, W, 4 * l + 2, R, cur, xd, E, part, lw + M.o_act, tag_of(P, epoch, l, 3),
                          nullptr, nullptr, 0u, blockIdx.x == 0 ? 3 + 5 * P.L + 10 * l + 6 : -1);
      }
      // h_next = h_mid + Wdown . act
      if (stab[4 * l + 3].ntl > 0) {
        const int E = stage_input(lw + M.o_act, nullptr, P.I, tag_of(P, epoch, l, 3), nullptr, P.eps, xd, redd, redf);
        if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 5 + 5 * l);
        gemv_stage<TRACE>(P, stab, nstages, W, 4 * l + 3, R, cur, xd, E, part, lw + M.LW, tag_of(P, epoch, l, 4),
                          lw + M.o_mid, nullptr, tag_of(P, epoch, l, 2),
                          blockIdx.x == 0 ? 3 + 5 * P.L + 10 * l + 8 : -1);
      }
    }
    // token = argmax(lm_head . RMSNorm(h_L))
    Best best{-INFINITY, 0x7fffffff};
    if (stab[4 * P.L].ntl > 0) {
      load_norm(P.final_norm, P.H, nw);
      const int E = stage_input(P.ll + (int64_t)P.L * M.LW, nullptr, P.H, tag_of(P, epoch, P.L - 1, 4), &nw, P.eps,
                                xd, redd, redf);
      if (TRACE && blockIdx.x == 0) stamp<TRACE>(P, 1 + 5 * P.L);
      lm_stage(P, stab, nstages, W, 4 * P.L, R, cur, xd, E, best, part);
    }
    // every issued copy has landed before the CTA exits (normally the warp consumed all of them)
    if (lane == 0) {
      for (int n = max(0, R.issued - R.rw); n < R.issued; ++n) mbar_drain(R.full + n % R.rw, (unsigned)(n / R.rw) & 1u);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
      if (argmax_better(ov, oi, best.v, best.i)) best.v = ov, best.i = oi;
    }
    if (lane == 0) s_bv[warp] = best.v, s_bi[warp] = best.i;
  }
  // ---------------------------------------------------------------- argmax over CTAs, the last one writes the token
  if (attn_g >= 0 && lane == 0) s_bv[warp] = -INFINITY, s_bi[warp] = 0x7fffffff;
  csync();
  if (threadIdx.x == 0) {
    float bv = s_bv[0];
    int bi = s_bi[0];
    for (int w = 1; w < kW; ++w)
      if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
    P.lm_val[blockIdx.x] = bv;
    P.lm_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned prev = atomicAdd(P.lm_cnt, 1u);
    *s_flag = prev == (unsigned)(gridDim.x - 1);
  }
  csync();
  if (*s_flag) {
    __threadfence();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += kCT) {
      const float v = __ldcg(&P.lm_val[b]);
      const int i = __ldcg(&P.lm_idx[b]);
      if (argmax_better(v, i, bv, bi)) bv = v, bi = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (argmax_better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    csync();
    if (lane == 0) s_bv[warp] = bv, s_bi[warp] = bi;
    csync();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kW; ++w)
        if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
      ok = ok && !device_error_set();
      *P.token = ok ? (int64_t)bi : 0;
      *P.position += 1;
      *P.lm_cnt = 0u;
      *P.epoch += 1u;
      __threadfence();
      if (TRACE && P.trace) P.trace[2 + 5 * P.L] = globaltimer_ns();
    }
  }
}

// ------------------------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// Tensor map of an int8 matrix [n, k] (k a multiple of 64) viewed as [k/64][n][64] bytes, box {64, 8, 4}.
static CUresult encode_raw(CUtensorMap *m, const void *ptr, int64_t n, int64_t k) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
  const cuuint32_t estr[3] = {1, 1, 1};
  const cuuint64_t dims[3] = {64, (cuuint64_t)n, (cuuint64_t)(k / 64)};
  const cuuint64_t strides[2] = {(cuuint64_t)k, 64};
  const cuuint32_t box[3] = {64, 8, 4};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
// Whether the driver encodes this view (decided once, on a well-formed probe that nothing dereferences).
static bool maps_ok() {
  static int v = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    CUtensorMap m;
    v = encode_raw(&m, (const void *)(uintptr_t)0x100000, 64, 512) == CUDA_SUCCESS ? 1 : 0;
  });
  return v == 1;
}
static int encode_matrix(CUtensorMap *m, const void *ptr, int64_t n, int64_t k) {
  const CUresult r = encode_raw(m, ptr, n, k);
  if (r != CUDA_SUCCESS) return set_error(EGPT_ERR_ARG, "dataflow: tensor map of a [%lld, %lld] matrix rejected (%d)",
                                          (long long)n, (long long)k, (int)r);
  return EGPT_OK;
}

constexpr size_t kStateBytes = 256;  // step state at the start of the workspace (epoch at +0), then the LL words

// Encoded tensor maps per workspace, re-encoded whenever the plan's weights or shapes differ from the cached ones
// (encoding is host-only work, ~1 us per matrix).
struct MapCache {
  std::vector<uint64_t> key;
  std::vector<CUtensorMap> maps;
};
static std::mutex g_map_mu;
static std::unordered_map<const void *, MapCache> g_maps;

static std::vector<uint64_t> map_key(const egpt_qwen3_plan *Pl) {
  std::vector<uint64_t> k = {(uint64_t)Pl->n_layers, (uint64_t)Pl->hidden, (uint64_t)Pl->intermediate,
                             (uint64_t)Pl->n_q_heads, (uint64_t)Pl->n_kv_heads, (uint64_t)Pl->head_dim,
                             (uint64_t)Pl->vocab, (uint64_t)(uintptr_t)Pl->w_lm};
  for (int l = 0; l < Pl->n_layers; ++l) {
    const egpt_qwen3_layer &Ly = Pl->layers[l];
    k.push_back((uint64_t)(uintptr_t)Ly.w_qkv), k.push_back((uint64_t)(uintptr_t)Ly.w_o);
    k.push_back((uint64_t)(uintptr_t)Ly.w_gu), k.push_back((uint64_t)(uintptr_t)Ly.w_down);
  }
  return k;
}

// The plan's tensor maps into `out` (4 L + 1 entries), from the cache or freshly encoded.
static int plan_maps(const egpt_qwen3_plan *Pl, CUtensorMap *out) {
  const int L = Pl->n_layers, D = Pl->head_dim;
  const size_t n = (size_t)4 * L + 1;
  std::vector<uint64_t> key = map_key(Pl);
  std::lock_guard<std::mutex> lock(g_map_mu);
  MapCache &c = g_maps[Pl->df_ws];
  if (c.key != key || c.maps.size() != n) {
    const int64_t H = Pl->hidden, I = Pl->intermediate, NQD = (int64_t)Pl->n_q_heads * D;
    const int64_t NQKV = (int64_t)(Pl->n_q_heads + 2 * Pl->n_kv_heads) * D;
    std::vector<CUtensorMap> maps(n);
    int r = EGPT_OK;
    for (int l = 0; l < L && r == EGPT_OK; ++l) {
      const egpt_qwen3_layer &Ly = Pl->layers[l];
      r = encode_matrix(&maps[4 * l], Ly.w_qkv, NQKV, H);
      if (r == EGPT_OK) r = encode_matrix(&maps[4 * l + 1], Ly.w_o, H, NQD);
      if (r == EGPT_OK) r = encode_matrix(&maps[4 * l + 2], Ly.w_gu, 2 * I, H);
      if (r == EGPT_OK) r = encode_matrix(&maps[4 * l + 3], Ly.w_down, H, I);
    }
    if (r == EGPT_OK) r = encode_matrix(&maps[4 * L], Pl->w_lm, Pl->vocab, H);
    if (r != EGPT_OK) {
      g_maps.erase(Pl->df_ws);
      return r;
    }
    c.key = std::move(key);
    c.maps = std::move(maps);
  }
  std::copy(c.maps.begin(), c.maps.end(), out);
  return EGPT_OK;
}

// Shared memory of the largest layer stage's per-item row sums on a GEMV CTA: (its tiles per CTA) x chunks x 16 x 8 B.
static size_t part_bytes(const egpt_qwen3_plan *Pl, int W) {
  const int64_t D = Pl->head_dim, H = Pl->hidden, I = Pl->intermediate;
  const int64_t nk[4] = {(H + 255) / 256, (Pl->n_q_heads * D + 255) / 256, (H + 255) / 256, (I + 255) / 256};
  const int64_t n[4] = {(Pl->n_q_heads + 2 * Pl->n_kv_heads) * D, H, 2 * I, H};
  int64_t items = 0;
  for (int i = 0; i < 4; ++i) items = std::max(items, (n[i] / 16 + W - 1) / W * nk[i]);
  return (size_t)(items * 16 * 8 + 127) / 128 * 128;
}

template <int DPL, int GRP>
static size_t attn_bytes() {
  return (sizeof(AttnScratch<DPL, GRP>) + 127) / 128 * 128;
}

struct Layout {
  size_t smem;
  int rw, part, ubytes, kv_smem, cph;
};

static bool layout(const egpt_qwen3_plan *Pl, Layout &lo) {
  // the stage shares are sized for the smaller GEMV grid (two attention CTAs per kv head), enough for either
  const int G = num_sms(), W = G - 2 * Pl->n_kv_heads;
  const int L = Pl->n_layers, D = Pl->head_dim, grp = Pl->n_q_heads / Pl->n_kv_heads;
  const int64_t kmax = std::max<int64_t>({(int64_t)Pl->hidden, (int64_t)Pl->intermediate, (int64_t)Pl->n_q_heads * D});
  const size_t ab = D == 32 ? attn_bytes<1, 2>() : grp == 2 ? attn_bytes<4, 2>() : attn_bytes<4, 4>();
  lo.part = (int)std::max(part_bytes(Pl, W), (kLmPartBytes + 127) / 128 * 128);  // also the lm_head's partial tiles
  lo.ubytes = (int)std::max<size_t>((4 * (size_t)x_stride(kmax) + 127) / 128 * 128, ab);
  const size_t limit = smem_limit();  // the kernel has no static shared memory
  const size_t fixed0 = 512 + ((size_t)(4 * L + 1) * sizeof(DStage) + 127) / 128 * 128 + (size_t)lo.part +
                        (size_t)lo.ubytes;
  // ring slots per warp: as many as fit (at least 1, at most 4), with their barriers
  lo.rw = 0;
  for (int rw = 4; rw >= 1; --rw) {
    const size_t bars = ((size_t)(kW * rw + 1) * 8 + 127) / 128 * 128;
    if (fixed0 + bars + (size_t)kW * rw * kItem <= limit) {
      lo.rw = rw;
      break;
    }
  }
  if (lo.rw == 0) return false;
  const size_t big = (size_t)kW * lo.rw * kItem;
  lo.smem = fixed0 + ((size_t)(kW * lo.rw + 1) * 8 + 127) / 128 * 128 + big;
  const size_t sa = 4 * (size_t)smem_attn_floats(Pl->cap, grp, D);
  // attention CTAs: K and V rows of the whole cache, then the attention scratch
  lo.kv_smem = ((size_t)Pl->cap * D * 2 * 2 + sa <= big && Pl->cap <= kMaxBlk * kRefBlock) ? 1 : 0;
  // two attention CTAs per kv head (half of the group's q heads each) when the rows sit in shared memory: the
  // attention stage is issue-bound on one CTA, and the GEMV stages are bound by their latency chain, not by the
  // 8 CTAs they give up
  lo.cph = (lo.kv_smem && grp >= 2) ? 2 : 1;
  return true;
}

static int validate(const egpt_qwen3_plan *Pl, Layout *lo_out) {
  if (!Pl || !Pl->layers || !Pl->layers_dev || !Pl->embed || !Pl->final_norm || !Pl->w_lm || !Pl->s_lm ||
      !Pl->rope_cos || !Pl->rope_sin || !Pl->token || !Pl->position || !Pl->lm_ws || !Pl->df_ws)
    return set_error(EGPT_ERR_ARG, "dataflow step: null pointer in plan");
  if (Pl->tp_world > 1) return set_error(EGPT_ERR_ARG, "dataflow step: one GPU only (tensor parallelism: the persistent step)");
  const int D = Pl->head_dim, NQ = Pl->n_q_heads, NKV = Pl->n_kv_heads;
  const int64_t H = Pl->hidden, I = Pl->intermediate;
  if (Pl->n_layers < 1 || NQ < 1 || NKV < 1 || NQ % NKV || Pl->vocab < 16 || Pl->cap < 1)
    return set_error(EGPT_ERR_SHAPE, "dataflow step: bad model sizes");
  if (Pl->n_layers > kMaxLayers) return set_error(EGPT_ERR_SHAPE, "dataflow step: at most %d layers", kMaxLayers);
  const int grp = NQ / NKV;
  if (!((D == 128 && (grp == 2 || grp == 4)) || (D == 32 && grp == 2)))
    return set_error(EGPT_ERR_SHAPE, "dataflow step: head_dim %d / group %d not built", D, grp);
  if (H % 64 || I % 64 || ((int64_t)NQ * D) % 64 || Pl->vocab % 16 || H > kMaxK || I > kMaxK || (int64_t)NQ * D > kMaxK)
    return set_error(EGPT_ERR_SHAPE, "dataflow step: hidden, intermediate and nq*d must be multiples of 64 and at most "
                     "%d, vocab a multiple of 16", kMaxK);
  const int G = num_sms();
  if (G > kArgmaxMaxCtas || G <= 2 * NKV) return set_error(EGPT_ERR_SHAPE, "dataflow step: SM count %d unusable", G);
  if (Pl->vocab > 0x7fffffffLL) return set_error(EGPT_ERR_SHAPE, "dataflow step: vocabulary too large");
  if (!maps_ok()) return set_error(EGPT_ERR_LAUNCH, "dataflow step: this driver does not encode the weights' tensor maps");
  bool aligned = (uintptr_t)Pl->w_lm % 16 == 0;
  for (int l = 0; l < Pl->n_layers; ++l) {
    const egpt_qwen3_layer &Ly = Pl->layers[l];
    aligned = aligned && (uintptr_t)Ly.w_qkv % 16 == 0 && (uintptr_t)Ly.w_o % 16 == 0 && (uintptr_t)Ly.w_gu % 16 == 0 &&
              (uintptr_t)Ly.w_down % 16 == 0 && (uintptr_t)Ly.ln_in % 8 == 0 && (uintptr_t)Ly.ln_post % 8 == 0 &&
              (uintptr_t)Ly.k_cache % 16 == 0 && (uintptr_t)Ly.v_cache % 16 == 0;
  }
  if (!aligned || (uintptr_t)Pl->df_ws % 256 || (uintptr_t)Pl->final_norm % 8 || (uintptr_t)Pl->embed % 8)
    return set_error(EGPT_ERR_ALIGN, "dataflow step: weights and caches 16-byte, norms 8-byte, workspace 256-byte "
                     "aligned");
  if (Pl->lm_ws_bytes < egpt_lm_head_ws_bytes(Pl->vocab) || Pl->df_ws_bytes < egpt_dataflow_ws_bytes(Pl))
    return set_error(EGPT_ERR_WORKSPACE, "dataflow step: workspace too small");
  Layout lo;
  if (!layout(Pl, lo)) return set_error(EGPT_ERR_SHAPE, "dataflow step: shared memory too small for this shape");
  *lo_out = lo;
  return EGPT_OK;
}

template <int DPL, int GRP>
static cudaError_t launch(const Params &P, size_t smem, cudaStream_t st, bool trace) {
  auto kern = trace ? dataflow_step_kernel<DPL, GRP, true> : dataflow_step_kernel<DPL, GRP, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kCT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *argv[] = {(void *)&P};
  return cudaLaunchKernelExC(&cfg, (const void *)kern, argv);
}

}  // namespace df
}  // namespace egpt

extern "C" size_t egpt_dataflow_ws_bytes(const egpt_qwen3_plan *Pl) {
  if (!Pl || Pl->n_layers < 1) return 0;
  return egpt::df::kStateBytes +
         (size_t)egpt::df::ll_words(Pl->n_layers, Pl->hidden, Pl->n_q_heads, Pl->n_kv_heads, Pl->head_dim,
                                    Pl->intermediate) * 8;
}

extern "C" int egpt_decode_step_dataflow_check(const egpt_qwen3_plan *Pl) {
  egpt::clear_error();
  egpt::df::Layout lo;
  return egpt::df::validate(Pl, &lo);
}

extern "C" int egpt_dataflow_prepare(const egpt_qwen3_plan *Pl) {
  using namespace egpt;
  clear_error();
  df::Layout lo;
  const int rc = df::validate(Pl, &lo);
  if (rc != EGPT_OK) return rc;
  std::vector<CUtensorMap> maps((size_t)4 * Pl->n_layers + 1);
  return df::plan_maps(Pl, maps.data());
}

extern "C" int egpt_decode_step_dataflow(const egpt_qwen3_plan *Pl, void *stream) {
  using namespace egpt;
  clear_error();
  df::Layout lo;
  const int rc = df::validate(Pl, &lo);
  if (rc != EGPT_OK) return rc;
  const int D = Pl->head_dim, grp = Pl->n_q_heads / Pl->n_kv_heads;
  static thread_local df::Params P;  // 29 KB, mostly tensor maps: kept off the host stack
  P = df::Params{};
  const int mrc = df::plan_maps(Pl, P.maps);
  if (mrc != EGPT_OK) return mrc;
  P.L = Pl->n_layers, P.H = Pl->hidden, P.NQ = Pl->n_q_heads, P.NKV = Pl->n_kv_heads, P.D = D;
  P.I = Pl->intermediate, P.V = Pl->vocab, P.cap = Pl->cap, P.eps = Pl->eps, P.scale = Pl->attn_scale;
  P.scale_bf16 = Pl->scale_dtype == EGPT_BF16;
  P.rw = lo.rw, P.kv_smem = lo.kv_smem, P.cph = lo.cph;
  P.w_lm = Pl->w_lm;
  P.layers = Pl->layers_dev;
  P.embed = (const uint16_t *)Pl->embed, P.final_norm = (const uint16_t *)Pl->final_norm;
  P.rope_cos = (const uint16_t *)Pl->rope_cos, P.rope_sin = (const uint16_t *)Pl->rope_sin;
  P.s_lm = Pl->s_lm;
  P.token = Pl->token, P.position = Pl->position;
  P.logits = (uint16_t *)Pl->logits;
  P.epoch = (unsigned *)Pl->df_ws;
  P.ll = (unsigned long long *)((char *)Pl->df_ws + df::kStateBytes);
  P.lm_val = (float *)Pl->lm_ws;
  P.lm_idx = (int *)((char *)Pl->lm_ws + kArgmaxMaxCtas * 4);
  P.lm_cnt = (unsigned *)((char *)Pl->lm_ws + kArgmaxMaxCtas * 8);
  P.part_bytes = lo.part, P.u_bytes = lo.ubytes;
  P.trace = (unsigned long long *)Pl->trace;
  const cudaStream_t cs = (cudaStream_t)stream;
  const bool tr = P.trace != nullptr;
  cudaError_t e;
  if (D == 32)
    e = df::launch<1, 2>(P, lo.smem, cs, tr);
  else if (grp == 2)
    e = df::launch<4, 2>(P, lo.smem, cs, tr);
  else
    e = df::launch<4, 4>(P, lo.smem, cs, tr);
  return check_launch(e, "dataflow_step_kernel");
}
