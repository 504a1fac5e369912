// Persistent decode step for B200 (sm_100a): one cooperative kernel per token, one CTA per SM.
//
// Replaces the launch sequence of egpt_decode_step (5 kernels per layer + lm_head), whose kernel boundaries
// (launch, ramp-up, tail, activation reload) cost several microseconds each and dominate the 1.7 GB weight
// stream of a Qwen3-1.7B token (~265 us at the measured HBM bandwidth). Inside one kernel:
//   * every GEMV stage (QKV, O, gate/up, down of each layer, then lm_head) is cut into row pairs; pair q of a
//     stage belongs to CTA q % G and, inside the CTA, to warp (q / G) % 16, so at any moment the whole GPU
//     reads a narrow, contiguous window of the matrix (all DRAM channels busy);
//   * each warp walks ONE flattened stream of (stage, pair, 2048-column chunk) items across all stages of
//     the token. Weights do not depend on activations, so each warp keeps kRing items in flight in its own
//     shared-memory ring (cp.async, 8 x 16 B per lane and item, plus the rows' scales) and an L2 prefetch
//     cursor (prefetch.global.L2::evict_last) kAhead items further: HBM keeps streaming the next stages'
//     weights while the warps wait at a barrier or run attention;
//   * the int8 x fp32 math is the exact packed-f32x2 dot product of gemv_i8.cu (same summation order per row);
//   * per stage the CTA stages its input vector in shared memory (fused RMSNorm, or the embedding row for
//     layer 0) and the lanes owning a reduced pair apply the fused epilogue (scale, residual add, SiLU*up,
//     lm_head argmax);
//   * stages that consume a whole vector produced by other CTAs are separated by a grid barrier: a monotonic
//     64-bit arrival counter with release/acquire ordering and a per-step epoch; every wait is bounded and
//     records EGPT_ERR_TIMEOUT instead of hanging;
//   * attention runs as a stage: CTA t < nkv * nsplit takes kv head t / nsplit and key range t % nsplit of
//     whole 128-key blocks (q/k RMSNorm + RoPE + KV append, then the attention core of attention.cu with the
//     reference GPU kernel's softmax rounding; ranges exchange their maxima), the last range of each head
//     combines;
//   * the lm_head stage keeps (max, index) per CTA; the last CTA reduces them, writes the token and advances
//     the position and the step epoch.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace egpt {
namespace ps {

constexpr int kNC = 16;                // warps (all compute)
constexpr int kCT = kNC * 32;          // threads
constexpr int kChunk = 2048;           // columns per stream item: 4 x 16-byte segments per lane and row
#ifndef EGPT_PS_RING
#define EGPT_PS_RING 2
#endif
#ifndef EGPT_PS_AHEAD
#define EGPT_PS_AHEAD 0
#endif
#ifndef EGPT_PS_PF_LAST
#define EGPT_PS_PF_LAST 1
#endif
#ifndef EGPT_PS_HOT_PF
#define EGPT_PS_HOT_PF 0
#endif
constexpr int kRing = EGPT_PS_RING;    // stream items in flight per warp (shared-memory ring filled by cp.async)
constexpr int kSlot = 2 * kChunk + 32; // ring slot: 2 rows x 2048 int8, then the rows' 16-byte scale blocks
constexpr int kAhead = EGPT_PS_AHEAD;  // L2 prefetch distance beyond the ring, in stream items per warp

enum Kind { QKV = 0, OPROJ = 1, GATEUP = 2, DOWN = 3, LMHEAD = 4 };

struct Params {
  int L, H, NQ, NKV, D, I;
  int64_t V, cap;
  float eps, scale;
  int scale_bf16, max_split;
  const egpt_qwen3_layer *layers;  // device array
  const uint16_t *embed, *final_norm, *rope_cos, *rope_sin;
  const int8_t *w_lm;
  const void *s_lm;
  int64_t *token, *position;
  uint16_t *h, *qkv, *attn, *act, *logits;
  float *attn_ws, *attn_xmax;           // split partials, range maxima
  unsigned *attn_cnt, *attn_xcnt, *attn_xgen;  // per kv head: combine / max-exchange arrivals, exchange generation
  float *lm_val;
  int *lm_idx;
  unsigned *lm_cnt;
  unsigned long long *bar;
  unsigned *epoch;
  unsigned long long *trace;  // nullable: per-barrier %globaltimer stamps of CTA 0
};

struct Stage {
  const int8_t *w;
  const void *s;
  int64_t n, k;
  int kind;
};

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory"); }

__device__ __forceinline__ Stage stage_desc(const Params &P, int s) {
  Stage st;
  if (s == 4 * P.L) {
    st.w = P.w_lm, st.s = P.s_lm, st.n = P.V, st.k = P.H, st.kind = LMHEAD;
    return st;
  }
  const egpt_qwen3_layer &Ly = P.layers[s >> 2];
  switch (s & 3) {
    case 0: st.w = Ly.w_qkv, st.s = Ly.s_qkv, st.n = (int64_t)(P.NQ + 2 * P.NKV) * P.D, st.k = P.H, st.kind = QKV; break;
    case 1: st.w = Ly.w_o, st.s = Ly.s_o, st.n = P.H, st.k = (int64_t)P.NQ * P.D, st.kind = OPROJ; break;
    case 2: st.w = Ly.w_gu, st.s = Ly.s_gu, st.n = 2 * (int64_t)P.I, st.k = P.H, st.kind = GATEUP; break;
    default: st.w = Ly.w_down, st.s = Ly.s_down, st.n = P.H, st.k = P.I, st.kind = DOWN; break;
  }
  return st;
}

__device__ __forceinline__ int64_t phys_row(const Stage &st, int64_t lr) {
  if (st.kind != GATEUP) return lr;
  return (lr & 1) ? (st.n >> 1) + (lr >> 1) : (lr >> 1);
}

// ------------------------------------------------------------------------------------------------ stream
// A warp's flattened stream of (stage, pair, chunk) items.
struct Cursor {
  Stage st;
  int s;          // stage index; 4L + 1 = end of the stream
  int c, nk;      // chunk of the current pair, chunks per row
  int64_t q;      // pair index within the stage
};

__device__ __forceinline__ void cur_stage(const Params &P, Cursor &cu, int s) {
  const int64_t step0 = (int64_t)blockIdx.x + (int64_t)gridDim.x * (threadIdx.x >> 5);
  for (; s <= 4 * P.L; ++s) {
    const Stage st = stage_desc(P, s);
    if (step0 < (st.n >> 1)) {
      cu.st = st, cu.s = s, cu.c = 0, cu.nk = (int)((st.k + kChunk - 1) / kChunk), cu.q = step0;
      return;
    }
  }
  cu.s = 4 * P.L + 1;
}
__device__ __forceinline__ void cur_next(const Params &P, Cursor &cu) {
  if (++cu.c < cu.nk) return;
  cu.c = 0;
  cu.q += (int64_t)gridDim.x * kNC;
  if (cu.q >= (cu.st.n >> 1)) cur_stage(P, cu, cu.s + 1);
}
__device__ __forceinline__ bool cur_end(const Params &P, const Cursor &cu) { return cu.s > 4 * P.L; }

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of row pr's scale inside the 16-byte block that holds it.
__device__ __forceinline__ int scale_off(const Params &P, const Stage &st, int64_t pr) {
  return (int)(((uintptr_t)st.s + (uintptr_t)(pr << (P.scale_bf16 ? 1 : 2))) & 15);
}

// Issue the copies of one item into a ring slot: each lane copies segments j * 32 + lane of both rows
// (8 x 16 B; the lane later reads back exactly the bytes it copied, so no cross-lane sync is needed) and
// lanes 0 and 1 copy the 16-byte block holding their row's scale. The caller commits the group.
__device__ __forceinline__ void fill_item(const Params &P, const Cursor &cu, uint8_t *slot) {
  const int lane = threadIdx.x & 31;
  const int64_t col0 = (int64_t)cu.c * kChunk;
  const int cw = (int)min((int64_t)kChunk, cu.st.k - col0);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int8_t *row = cu.st.w + phys_row(cu.st, 2 * cu.q + r) * cu.st.k + col0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sl = j * 32 + lane;
      if (sl * 16 < cw) cp_async16(slot + r * kChunk + sl * 16, row + sl * 16);
    }
  }
  if (lane < 2) {
    const int64_t pr = phys_row(cu.st, 2 * cu.q + lane);
    const uintptr_t a = (uintptr_t)cu.st.s + (uintptr_t)(pr << (P.scale_bf16 ? 1 : 2));
    cp_async16(slot + 2 * kChunk + lane * 16, (const void *)(a & ~(uintptr_t)15));
  }
}

// L2 prefetch of one item: lanes 0-15 take row 0, 16-31 row 1, one 128-byte line each.
__device__ __forceinline__ void prefetch_item(const Cursor &cu) {
  const int lane = threadIdx.x & 31;
  const int64_t col0 = (int64_t)cu.c * kChunk;
  const int cw = (int)min((int64_t)kChunk, cu.st.k - col0);
  const int off = (lane & 15) * 128;
  if (off < cw) {
    const int8_t *p = cu.st.w + phys_row(cu.st, 2 * cu.q + (lane >> 4)) * cu.st.k + col0 + off;
#if EGPT_PS_PF_LAST
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
#else
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
#endif
  }
}

// ------------------------------------------------------------------------------------------------ sync
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier: arrivals accumulate on a monotonic counter; barrier idx (1-based) of the step with epoch
// base completes when the counter reaches (base + idx) * G. Bounded: records EGPT_ERR_TIMEOUT, returns false.
__device__ bool grid_barrier(const Params &P, unsigned long long base, unsigned long long idx, int *s_ok) {
  const unsigned long long target = (base + idx) * gridDim.x;
  csync();
  if (threadIdx.x == 0) {
    const bool tr = P.trace && blockIdx.x == 0;
    if (tr) P.trace[2 * idx - 1] = globaltimer_ns();
    __threadfence();
    atomicAdd(P.bar, 1ull);
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int it = 0; ld_acquire_u64(P.bar) < target; ++it) {
      if ((it & 63) == 63) {
        if (device_error_set()) {
          ok = 0;
          break;
        }
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_device_error(EGPT_ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    if (tr) P.trace[2 * idx] = globaltimer_ns();
    *s_ok = ok;
  }
  csync();
  return *s_ok != 0;
}

// Trace: stamp k (CTA 0, thread 0) of the second trace region: the moment stage k's input is ready (GEMV
// stages: staged and normalised; attention: this CTA's scores done).
__device__ __forceinline__ void stamp(const Params &P, int k) {
  if (P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[4 + 10 * P.L + k] = globaltimer_ns();
}

// Small data read on the step's critical path (norm weights), marked evict_last in L2 so that the weight stream
// (normal priority) does not push it out between steps: one 128-byte line per thread, grid-strided.
__device__ void hot_prefetch(const Params &P) {
  const int64_t gt = (int64_t)blockIdx.x * kCT + threadIdx.x, gs = (int64_t)gridDim.x * kCT;
  const int64_t lh = ((int64_t)P.H * 2 + 127) / 128, ld = ((int64_t)P.D * 2 + 127) / 128;
  const int64_t per_layer = 2 * lh + 2 * ld;
  for (int64_t i = gt; i < per_layer * P.L + lh; i += gs) {
    const char *a;
    if (i >= per_layer * P.L) {
      a = (const char *)P.final_norm + (i - per_layer * P.L) * 128;
    } else {
      const egpt_qwen3_layer &Ly = P.layers[i / per_layer];
      int64_t r = i % per_layer;
      if (r < lh) a = (const char *)Ly.ln_in + r * 128;
      else if ((r -= lh) < lh) a = (const char *)Ly.ln_post + r * 128;
      else if ((r -= lh) < ld) a = (const char *)Ly.q_norm + r * 128;
      else a = (const char *)Ly.k_norm + (r - ld) * 128;
    }
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(a));
  }
}

// CTA-wide sum in a fixed order: per-warp butterfly, then every thread adds the warp partials in order.
__device__ __forceinline__ float csum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  csync();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNC; ++w) t += red[w];
  csync();  // red is reused by the next reduction
  return t;
}

constexpr int kMaxPerThread = 12;  // staged inputs up to 12 * 512 = 6144 elements

// RMSNorm weights of a stage input, loaded into registers BEFORE the grid barrier that precedes the stage
// (they do not depend on the step), so their latency hides behind the barrier instead of adding to it.
struct NormW {
  float w[kMaxPerThread];
};
__device__ __forceinline__ void load_norm(const uint16_t *nw, int64_t k, NormW &n) {
#pragma unroll
  for (int e = 0; e < kMaxPerThread; ++e) {
    const int64_t i = threadIdx.x + (int64_t)e * kCT;
    n.w[e] = i < k ? bf16_bits_to_f32(nw[i]) : 0.f;
  }
}

// Stage an input vector of k bf16 values into xs (fp32, [4][k/16] float4 layout), optionally RMSNorm'd with
// the preloaded weights nw (HF rounding points): one pass over global memory, one CTA reduction. copy_to
// (nullable) receives the raw values (layer 0: h = embedding row).
__device__ void stage_input(const uint16_t *src, int64_t k, const NormW *nw, float eps, float4 *xs, float *red,
                            uint16_t *copy_to) {
  const int t = threadIdx.x;
  float v[kMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < kMaxPerThread; ++e) {
    const int64_t i = t + (int64_t)e * kCT;
    v[e] = 0.f;
    if (i < k) {
      const uint16_t raw = __ldcg(src + i);
      if (copy_to) copy_to[i] = raw;
      v[e] = bf16_bits_to_f32(raw);
    }
    ss = fmaf(v[e], v[e], ss);
  }
  if (nw) {
    const float inv = rsqrtf(csum(ss, red) / (float)k + eps);
#pragma unroll
    for (int e = 0; e < kMaxPerThread; ++e) v[e] = round_bf16(round_bf16(v[e] * inv) * nw->w[e]);
  }
  const int segs = (int)(k >> 4);
  float *xsf = (float *)xs;
#pragma unroll
  for (int e = 0; e < kMaxPerThread; ++e) {
    const int64_t i = t + (int64_t)e * kCT;
    if (i < k) {
      const int sg = (int)(i >> 4), el = (int)(i & 15);
      xsf[((el >> 2) * segs + sg) * 4 + (el & 3)] = v[e];
    }
  }
  csync();
}

// ------------------------------------------------------------------------------------------------ GEMV stage
struct Best {
  float v;
  int i;
};

struct Stream {
  Cursor cur, fill, pf;  // consumption, ring-fill (kRing items ahead of cur) and L2-prefetch cursors
  int lead;              // items pf is ahead of fill
  int slot;              // ring slot holding cur's item
  uint8_t *ring;         // this warp's kRing slots
};

__device__ __forceinline__ void top_up_prefetch(const Params &P, Stream &S) {
  if constexpr (kAhead > 0) {
    while (S.lead < kAhead && !cur_end(P, S.pf)) {
      prefetch_item(S.pf);
      cur_next(P, S.pf);
      ++S.lead;
    }
  }
}

// Start the stream: kRing items in flight (one commit group each, empty past the end), prefetch beyond.
__device__ __forceinline__ void stream_start(const Params &P, Stream &S, uint8_t *ring) {
  S.ring = ring;
  S.slot = 0;
  cur_stage(P, S.cur, 0);
  S.fill = S.cur;
#pragma unroll 1
  for (int i = 0; i < kRing; ++i) {
    if (!cur_end(P, S.fill)) {
      fill_item(P, S.fill, ring + i * kSlot);
      cur_next(P, S.fill);
    }
    cp_async_commit();
  }
  S.pf = S.fill;
  S.lead = 0;
  top_up_prefetch(P, S);
}

// Consume this warp's items of stage s (the stream's cursor is at stage s or later). Each consumed slot is
// refilled at once with the item kRing ahead, whatever stage it belongs to: weights do not depend on the
// activations, so the copies for the next stages run on while this warp waits at a barrier.
__device__ void gemv_stage(const Params &P, int s, Stream &S, const float4 *xs, Best &best) {
  const int lane = threadIdx.x & 31;
  uint64_t acc0 = 0ull, acc1 = 0ull;
  float s_e = 0.f, res_e = 0.f;
  while (S.cur.s == s) {
    const Stage st = S.cur.st;
    const int64_t q = S.cur.q;
    const int c = S.cur.c;
    const bool last = c == S.cur.nk - 1;
    const bool resid = st.kind == OPROJ || st.kind == DOWN;
    if (c == 0) {
      acc0 = acc1 = 0ull;
      if (resid && lane < 2) res_e = bf16_bits_to_f32(__ldcg(P.h + 2 * q + lane));
    }
    cp_async_wait<kRing - 1>();  // this lane's copies of cur's item have landed
    const uint8_t *slot = S.ring + S.slot * kSlot;
    if (last && lane < 2) {  // read the scale before the slot is refilled
      const int64_t pr = phys_row(st, 2 * q + lane);
      const uint8_t *blk = slot + 2 * kChunk + lane * 16 + scale_off(P, st, pr);
      s_e = P.scale_bf16 ? bf16_bits_to_f32(*(const uint16_t *)blk) : *(const float *)blk;
    }
    const int64_t col0 = (int64_t)c * kChunk;
    const int cw = (int)min((int64_t)kChunk, st.k - col0);
    const int xsegs = (int)(st.k >> 4);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sl = j * 32 + lane;
      if (sl * 16 < cw) {
        const ulonglong2 *xb = (const ulonglong2 *)(xs + c * (kChunk / 16) + sl);
        uint64_t x2[8];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const ulonglong2 v = xb[(size_t)g * xsegs];
          x2[2 * g] = v.x;
          x2[2 * g + 1] = v.y;
        }
        acc0 = dot16x2(x2, *(const uint4 *)(slot + sl * 16), acc0);
        acc1 = dot16x2(x2, *(const uint4 *)(slot + kChunk + sl * 16), acc1);
      }
    }
    // refill the slot (the FMAs above consumed its bytes) with the item kRing ahead; top up the L2 prefetch
    if (!cur_end(P, S.fill)) {
      fill_item(P, S.fill, S.ring + S.slot * kSlot);
      cur_next(P, S.fill);
      --S.lead;
    }
    cp_async_commit();
    top_up_prefetch(P, S);
    S.slot = S.slot + 1 == kRing ? 0 : S.slot + 1;
    cur_next(P, S.cur);
    if (!last) continue;
    const float2 a0 = unpack2(acc0), a1 = unpack2(acc1);
    const float t0 = warp_sum(a0.x + a0.y), t1 = warp_sum(a1.x + a1.y);
    const float s_up = __shfl_down_sync(0xffffffffu, s_e, 1);
    if (lane < 2) {
      const float y = round_bf16((lane == 0 ? t0 : t1) * s_e);
      const int64_t lr = 2 * q + lane;
      switch (st.kind) {
        case QKV: P.qkv[lr] = f32_to_bf16_bits(y); break;
        case OPROJ:
        case DOWN: P.h[lr] = f32_to_bf16_bits(round_bf16(res_e + y)); break;
        case GATEUP:
          if (lane == 0) {
            const float up = round_bf16(t1 * s_up);
            P.act[q] = f32_to_bf16_bits(round_bf16(round_bf16(y / (1.0f + expf(-y))) * up));
          }
          break;
        default:
          if (P.logits) P.logits[lr] = f32_to_bf16_bits(y);
          if (argmax_better(y, (int)lr, best.v, best.i)) {
            best.v = y;
            best.i = (int)lr;
          }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ attention
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One (kv head, key range) task on the attention core of attention.cu: the same ranges, tiles and merge
// order as attn_split_kernel, so both paths give the same bits. The q heads of the group and the new k row
// are normalised and rotated by one warp each (warp-level reductions, RoPE partners via a 16-lane shuffle).
// With several ranges, each publishes its maximum score per q head and waits (bounded) for the other ranges
// of its kv head: the maxima of the ranges before it start its running maximum of the reference's block walk
// (the per-kernel path rescores those keys instead).
// Step-invariant inputs of a warp's attention prologue role (q head j < GRP, or the k head): its norm weights
// and the RoPE row of this position, DPL values per lane.
template <int DPL>
struct AttnPre {
  float wn[DPL], cs[DPL], sn[DPL];
};

template <int DPL, int GRP>
__device__ __forceinline__ void attn_preload(const Params &P, const egpt_qwen3_layer &Ly, int task, int nsplit, int bps,
                                             int64_t pos, AttnPre<DPL> &pre) {
  constexpr int D = DPL * 32, half = D / 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp > GRP) return;
  const uint16_t *nw = (const uint16_t *)(warp == GRP ? Ly.k_norm : Ly.q_norm) + lane * DPL;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int e = lane * DPL + i, r = e < half ? e : e - half;
    pre.wn[i] = bf16_bits_to_f32(nw[i]);
    pre.cs[i] = bf16_bits_to_f32(P.rope_cos[pos * half + r]);
    pre.sn[i] = bf16_bits_to_f32(P.rope_sin[pos * half + r]);
  }
}

// L2 prefetch of the cached K and V rows of this task's key range (the rows before this step's position).
template <int DPL, int GRP>
__device__ __forceinline__ void attn_prefetch_kv(const Params &P, const egpt_qwen3_layer &Ly, int task, int nsplit,
                                                 int bps, int64_t pos) {
  constexpr int D = DPL * 32;
  constexpr int lines = D * 2 / 128 > 0 ? D * 2 / 128 : 1;  // 128-byte lines per row
  const int g = task / nsplit, split = task % nsplit;
  const int64_t k0 = (int64_t)split * bps * kRefBlock, k1 = min(pos, k0 + (int64_t)bps * kRefBlock);
  const int64_t n = k1 > k0 ? (k1 - k0) * lines : 0;
  const char *kb = (const char *)Ly.k_cache + ((int64_t)g * P.cap + k0) * D * 2;
  const char *vb = (const char *)Ly.v_cache + ((int64_t)g * P.cap + k0) * D * 2;
  for (int64_t i = threadIdx.x; i < 2 * n; i += kCT) {
    const char *a = (i < n ? kb : vb) + (i < n ? i : i - n) * 128;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
  }
}

template <int DPL, int GRP>
__device__ void attention_task(const Params &P, const egpt_qwen3_layer &Ly, int task, int nsplit, int bps, int64_t pos,
                               float *u, const AttnPre<DPL> &pre, int tslot) {
  constexpr int D = DPL * 32;
  AttnScratch<DPL, GRP> &S = *reinterpret_cast<AttnScratch<DPL, GRP> *>(u);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = task / nsplit, split = task % nsplit;
  const int64_t L = pos + 1;
  const int64_t k0 = (int64_t)split * bps * kRefBlock, k1 = min(L, k0 + (int64_t)bps * kRefBlock);
  const bool own = pos >= k0 && pos < k1;  // this range holds the new slot: write it before reading the range
  uint16_t *kc = (uint16_t *)Ly.k_cache, *vc = (uint16_t *)Ly.v_cache;
  const int64_t kv_base = (int64_t)g * P.cap * D;
  if (warp < GRP || (warp == GRP && own)) {
    const bool isk = warp == GRP;
    const uint16_t *src = P.qkv + (int64_t)(isk ? P.NQ + g : g * GRP + warp) * D + lane * DPL;
    float v[DPL];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      v[i] = bf16_bits_to_f32(__ldcg(src + i));
      ss = fmaf(v[i], v[i], ss);
    }
    const float inv = rsqrtf(warp_sum(ss) / (float)D + P.eps);
#pragma unroll
    for (int i = 0; i < DPL; ++i) v[i] = round_bf16(round_bf16(v[i] * inv) * pre.wn[i]);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {  // element e pairs with e +- D/2, held DPL * 16 elements = 16 lanes away
      const float other = __shfl_xor_sync(0xffffffffu, v[i], 16);
      const float rot = lane < 16 ? -other : other;
      const float o = round_bf16(round_bf16(v[i] * pre.cs[i]) + round_bf16(rot * pre.sn[i]));
      if (isk)
        kc[kv_base + pos * D + lane * DPL + i] = f32_to_bf16_bits(o);
      else
        S.q[warp][lane * DPL + i] = o;
    }
  } else if (warp == GRP + 1 && own) {
    const uint16_t *vs = P.qkv + (int64_t)(P.NQ + P.NKV + g) * D;
    for (int i = lane; i < D; i += 32) vc[kv_base + pos * D + i] = __ldcg(vs + i);
  }
  if (own) __threadfence();
  csync();
  AttnTask t;
  t.K = kc + kv_base;
  t.V = vc + kv_base;
  t.k0 = k0;
  t.k1 = k1;
  t.scale = P.scale;
  attn_pass_a<DPL, GRP, true>(t, S);
  stamp(P, tslot);
  const int ntiles = (int)((k1 - k0 + kKeyTile - 1) / kKeyTile);
  if (nsplit > 1) {
    csync();
    if (threadIdx.x < GRP) {
      float m = -INFINITY;
      for (int tt = 0; tt < ntiles; ++tt) m = fmaxf(m, S.tmax[tt][threadIdx.x]);
      P.attn_xmax[(int64_t)(g * GRP + threadIdx.x) * P.max_split + split] = m;
      __threadfence();
    }
    csync();
    if (threadIdx.x == 0) {
      const unsigned gen = ld_acquire_u32(P.attn_xgen + g);  // read before arriving: it cannot move until then
      const unsigned prev = atomicAdd(P.attn_xcnt + g, 1u);
      if (prev == (unsigned)(nsplit - 1)) {
        P.attn_xcnt[g] = 0u;
        __threadfence();
        st_release_u32(P.attn_xgen + g, gen + 1u);
      } else {
        const uint64_t t0 = globaltimer_ns();
        for (int it = 0; ld_acquire_u32(P.attn_xgen + g) == gen; ++it) {
          if ((it & 63) == 63 && (device_error_set() || globaltimer_ns() - t0 > kWaitLimitNs)) {
            set_device_error(EGPT_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
    csync();
    if (threadIdx.x < GRP) {
      float m = -INFINITY;
      for (int s2 = 0; s2 < split; ++s2)
        m = fmaxf(m, __ldcg(P.attn_xmax + (int64_t)(g * GRP + threadIdx.x) * P.max_split + s2));
      S.mb[threadIdx.x] = m;
    }
  } else if (threadIdx.x < GRP) {
    S.mb[threadIdx.x] = -INFINITY;
  }
  attn_walk<DPL, GRP, true, kCT>(t, S, true);
  AttnOut o;
  o.out = P.attn;
  o.part = P.attn_ws;
  o.cnt = P.attn_cnt + g;
  o.g = g;
  o.split = split;
  o.nsplit = nsplit;
  o.max_split = P.max_split;
  o.busy = min(kAttnWarps, ntiles);
  attn_finish<DPL, GRP, true, kCT>(S, o);
}

// ------------------------------------------------------------------------------------------------ kernel
template <int DPL, int GRP>
__global__ void __launch_bounds__(kCT, 1) decode_step_kernel(const Params P) {
  extern __shared__ __align__(128) uint8_t smem[];
  float *red = (float *)smem;                    // 64 floats
  uint8_t *ring = smem + 256;                    // kNC x kRing weight slots
  float *u = (float *)(ring + kNC * kRing * kSlot);  // union: staged input (float4) / attention scratch
  float4 *xs = (float4 *)u;
  __shared__ int s_flag;
  __shared__ float s_bv[kNC];
  __shared__ int s_bi[kNC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Start the weight stream immediately: it does not depend on the token, the position or the activations.
  Stream S;
  stream_start(P, S, ring + (size_t)warp * kRing * kSlot);
#if EGPT_PS_HOT_PF
  hot_prefetch(P);
#endif

  const unsigned long long nb = 5ull * (unsigned long long)P.L;  // grid barriers per step
  const unsigned long long base = (unsigned long long)(*(volatile unsigned *)P.epoch) * nb;
  unsigned long long bidx = 0;
  bool ok = true;
  Best best{-INFINITY, 0x7fffffff};
  const int64_t pos = *P.position;
  const int64_t tok = *P.token;
  if (pos < 0 || pos >= P.cap || tok < 0 || tok >= P.V) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    ok = false;
  }
  const int bps = split_blocks(pos + 1, P.max_split);  // attention: ranges of bps 128-key blocks
  const int nsplit = split_count(pos + 1, bps);
  if (bps * kRefBlock > AttnScratch<DPL, GRP>::KS) {  // excluded on the host for positions < cap
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    ok = false;
  }
  if (P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[0] = globaltimer_ns();

  // Everything a stage reads that does not depend on the step (norm weights, the attention prologue's norm
  // weights and RoPE row, the KV ranges) is requested before the barrier that precedes the stage.
  const bool attn_cta = (int)blockIdx.x < P.NKV * nsplit;
  NormW nw;
  load_norm((const uint16_t *)P.layers[0].ln_in, P.H, nw);
  for (int l = 0; l < P.L; ++l) {
    const egpt_qwen3_layer &Ly = P.layers[l];
    if (attn_cta) attn_prefetch_kv<DPL, GRP>(P, Ly, blockIdx.x, nsplit, bps, pos);
    // ---- q|k|v = Wqkv . RMSNorm(h)  (layer 0: h = embed[token], CTA 0 stores it)
    const uint16_t *hin = l == 0 ? P.embed + (ok ? tok : 0) * P.H : P.h;
    stage_input(hin, P.H, &nw, P.eps, xs, red, (l == 0 && blockIdx.x == 0) ? P.h : nullptr);
    stamp(P, 5 * l);
    gemv_stage(P, 4 * l, S, xs, best);
    AttnPre<DPL> pre;
    if (attn_cta) attn_preload<DPL, GRP>(P, Ly, blockIdx.x, nsplit, bps, pos, pre);
    ok = grid_barrier(P, base, ++bidx, &s_flag) && ok;
    // ---- attention (q/k norm + RoPE + KV append + split-K softmax . V + combine)
    if (ok && attn_cta) attention_task<DPL, GRP>(P, Ly, blockIdx.x, nsplit, bps, pos, u, pre, 5 * l + 1);
    ok = grid_barrier(P, base, ++bidx, &s_flag) && ok;
    // ---- h += Wo . attn
    stage_input(P.attn, (int64_t)P.NQ * P.D, nullptr, 0.f, xs, red, nullptr);
    stamp(P, 5 * l + 2);
    gemv_stage(P, 4 * l + 1, S, xs, best);
    load_norm((const uint16_t *)Ly.ln_post, P.H, nw);
    ok = grid_barrier(P, base, ++bidx, &s_flag) && ok;
    // ---- act = silu(Wg . RMSNorm(h)) * (Wu . RMSNorm(h))
    stage_input(P.h, P.H, &nw, P.eps, xs, red, nullptr);
    stamp(P, 5 * l + 3);
    gemv_stage(P, 4 * l + 2, S, xs, best);
    ok = grid_barrier(P, base, ++bidx, &s_flag) && ok;
    // ---- h += Wdown . act
    stage_input(P.act, P.I, nullptr, 0.f, xs, red, nullptr);
    stamp(P, 5 * l + 4);
    gemv_stage(P, 4 * l + 3, S, xs, best);
    load_norm(l + 1 < P.L ? (const uint16_t *)P.layers[l + 1].ln_in : P.final_norm, P.H, nw);
    ok = grid_barrier(P, base, ++bidx, &s_flag) && ok;
  }
  // ---- token = argmax(lm_head . RMSNorm(h)); the last CTA also advances position and the step epoch
  stage_input(P.h, P.H, &nw, P.eps, xs, red, nullptr);
  stamp(P, 5 * P.L);
  gemv_stage(P, 4 * P.L, S, xs, best);
  if (P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[1 + 10 * P.L] = globaltimer_ns();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
    if (argmax_better(ov, oi, best.v, best.i)) best.v = ov, best.i = oi;
  }
  if (lane == 0) s_bv[warp] = best.v, s_bi[warp] = best.i;
  csync();
  if (threadIdx.x == 0) {
    float bv = s_bv[0];
    int bi = s_bi[0];
    for (int w = 1; w < kNC; ++w)
      if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
    P.lm_val[blockIdx.x] = bv;
    P.lm_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned prev = atomicAdd(P.lm_cnt, 1u);
    s_flag = prev == (unsigned)(gridDim.x - 1);
  }
  csync();
  if (s_flag) {
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
      for (int w = 1; w < kNC; ++w)
        if (argmax_better(s_bv[w], s_bi[w], bv, bi)) bv = s_bv[w], bi = s_bi[w];
      *P.token = ok ? (int64_t)bi : 0;
      *P.position += 1;
      *P.lm_cnt = 0u;
      *P.epoch += 1u;
      __threadfence();
      if (P.trace) P.trace[2 + 10 * P.L] = globaltimer_ns();
    }
  }
}

template <int DPL, int GRP>
static cudaError_t launch(const Params &P, size_t smem, cudaStream_t st) {
  auto kern = decode_step_kernel<DPL, GRP>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
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

}  // namespace ps
}  // namespace egpt

using namespace egpt;

extern "C" size_t egpt_step_sync_ws_bytes(void) { return 64; }

// Host-side checks of a plan for the persistent kernel; on success *smem is its dynamic shared memory.
static int persistent_validate(const egpt_qwen3_plan *Pl, size_t *smem_out) {
  if (!Pl || !Pl->layers || !Pl->layers_dev || !Pl->sync_ws || !Pl->embed || !Pl->final_norm || !Pl->w_lm ||
      !Pl->s_lm || !Pl->rope_cos || !Pl->rope_sin || !Pl->token || !Pl->position || !Pl->h || !Pl->qkv ||
      !Pl->attn || !Pl->act || !Pl->lm_ws || !Pl->attn_ws)
    return set_error(EGPT_ERR_ARG, "decode_step_persistent: null pointer in plan");
  const int D = Pl->head_dim, NQ = Pl->n_q_heads, NKV = Pl->n_kv_heads;
  const int64_t H = Pl->hidden, I = Pl->intermediate;
  if (Pl->n_layers < 1 || H < 16 || I < 16 || NQ < 1 || NKV < 1 || NQ % NKV || Pl->vocab < 2 || Pl->cap < 1)
    return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: bad model sizes");
  const int grp = NQ / NKV;
  const bool shape_ok = (D == 128 && (grp == 2 || grp == 4)) || (D == 32 && grp == 2);
  if (!shape_ok) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: head_dim %d / group %d not built", D, grp);
  if (H % 16 || I % 16 || ((int64_t)NQ * D) % 16 || Pl->vocab % 2 ||
      std::max<int64_t>({H, I, (int64_t)NQ * D}) > (int64_t)ps::kMaxPerThread * ps::kCT)
    return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: sizes must be multiples of 16 (vocab even)");
  const int G = num_sms();
  if (G > kArgmaxMaxCtas) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: too many SMs");
  // weights are copied in 16-byte pieces; a scale is read from the 16-byte block that holds it
  const size_t sal = Pl->scale_dtype == EGPT_BF16 ? 2 : 4;
  bool aligned = (uintptr_t)Pl->w_lm % 16 == 0 && (uintptr_t)Pl->s_lm % sal == 0;
  for (int l = 0; l < Pl->n_layers; ++l) {
    const egpt_qwen3_layer &Ly = Pl->layers[l];
    aligned = aligned && (uintptr_t)Ly.w_qkv % 16 == 0 && (uintptr_t)Ly.w_o % 16 == 0 &&
              (uintptr_t)Ly.w_gu % 16 == 0 && (uintptr_t)Ly.w_down % 16 == 0 && (uintptr_t)Ly.s_qkv % sal == 0 &&
              (uintptr_t)Ly.s_o % sal == 0 && (uintptr_t)Ly.s_gu % sal == 0 && (uintptr_t)Ly.s_down % sal == 0;
  }
  if (!aligned)
    return set_error(EGPT_ERR_ALIGN, "decode_step_persistent: weights must be 16-byte aligned, scales element aligned");
  if (Pl->attn_ws_bytes < egpt_attn_ws_bytes(1, NQ, NKV, D, Pl->attn_max_split) ||
      Pl->lm_ws_bytes < egpt_lm_head_ws_bytes(Pl->vocab))
    return set_error(EGPT_ERR_WORKSPACE, "decode_step_persistent: workspace too small");
  // shared memory: reduction scratch + weight ring + union(staged input, attention scratch)
  const int64_t kmax = std::max<int64_t>({H, I, (int64_t)NQ * D});
  const size_t attn_bytes = D == 32 ? sizeof(AttnScratch<1, 2>) : grp == 2 ? sizeof(AttnScratch<4, 2>) : sizeof(AttnScratch<4, 4>);
  const size_t smem = 256 + (size_t)ps::kNC * ps::kRing * ps::kSlot + std::max<size_t>((size_t)kmax * 4, (attn_bytes + 15) / 16 * 16);
  const int max_split = std::max(1, std::min(Pl->attn_max_split, G / NKV));
  if ((int64_t)split_blocks(Pl->cap, max_split) * kRefBlock > split_keys_max(grp))
    return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: cap %lld needs more than %d attention ranges per kv head",
                     (long long)Pl->cap, max_split);
  if (smem > smem_limit() - 1024)
    return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: activations (%lld) too large for shared memory",
                     (long long)kmax);
  *smem_out = smem;
  return EGPT_OK;
}

extern "C" int egpt_decode_step_persistent_check(const egpt_qwen3_plan *Pl) {
  clear_error();
  size_t smem = 0;
  return persistent_validate(Pl, &smem);
}

extern "C" int egpt_decode_step_persistent(const egpt_qwen3_plan *Pl, void *stream) {
  clear_error();
  size_t smem = 0;
  const int rc = persistent_validate(Pl, &smem);
  if (rc != EGPT_OK) return rc;
  const int D = Pl->head_dim, NQ = Pl->n_q_heads, NKV = Pl->n_kv_heads;
  const int64_t H = Pl->hidden, I = Pl->intermediate;
  const int grp = NQ / NKV;
  const int max_split = std::max(1, std::min(Pl->attn_max_split, num_sms() / NKV));

  ps::Params P{};
  P.L = Pl->n_layers, P.H = (int)H, P.NQ = NQ, P.NKV = NKV, P.D = D, P.I = (int)I;
  P.V = Pl->vocab, P.cap = Pl->cap, P.eps = Pl->eps, P.scale = Pl->attn_scale;
  P.scale_bf16 = Pl->scale_dtype == EGPT_BF16, P.max_split = max_split;
  P.layers = Pl->layers_dev;
  P.embed = (const uint16_t *)Pl->embed, P.final_norm = (const uint16_t *)Pl->final_norm;
  P.rope_cos = (const uint16_t *)Pl->rope_cos, P.rope_sin = (const uint16_t *)Pl->rope_sin;
  P.w_lm = Pl->w_lm, P.s_lm = Pl->s_lm;
  P.token = Pl->token, P.position = Pl->position;
  P.h = (uint16_t *)Pl->h, P.qkv = (uint16_t *)Pl->qkv, P.attn = (uint16_t *)Pl->attn, P.act = (uint16_t *)Pl->act;
  P.logits = (uint16_t *)Pl->logits;
  P.attn_ws = (float *)Pl->attn_ws;
  P.attn_xmax = P.attn_ws + (size_t)NQ * Pl->attn_max_split * (D + 2);
  P.attn_cnt = (unsigned *)((char *)Pl->attn_ws + attn_ws_float_bytes(1, NQ, D, Pl->attn_max_split));
  P.attn_xcnt = P.attn_cnt + NKV;
  P.attn_xgen = P.attn_cnt + 2 * NKV;
  P.lm_val = (float *)Pl->lm_ws;
  P.lm_idx = (int *)((char *)Pl->lm_ws + kArgmaxMaxCtas * 4);
  P.lm_cnt = (unsigned *)((char *)Pl->lm_ws + kArgmaxMaxCtas * 8);
  P.bar = (unsigned long long *)Pl->sync_ws;
  P.epoch = (unsigned *)((char *)Pl->sync_ws + 8);
  P.trace = (unsigned long long *)Pl->trace;
  cudaError_t e;
  if (D == 128 && grp == 2)
    e = ps::launch<4, 2>(P, smem, (cudaStream_t)stream);
  else if (D == 128)
    e = ps::launch<4, 4>(P, smem, (cudaStream_t)stream);
  else
    e = ps::launch<1, 2>(P, smem, (cudaStream_t)stream);
  return check_launch(e, "decode_step_kernel");
}
