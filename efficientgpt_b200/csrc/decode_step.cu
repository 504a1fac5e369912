// Persistent decode step for B200 (sm_100a): one cooperative kernel per token, one CTA per SM.
//
// Replaces the launch sequence of egpt_decode_step (5 kernels per layer + lm_head), whose kernel boundaries
// (launch, ramp-up, tail, activation reload) cost several microseconds each and dominate the 1.7 GB weight
// stream of a Qwen3-1.7B token (~265 us at the measured HBM bandwidth). Inside one kernel:
//   * every GEMV stage (q|k|v, o, gate|up, down of each layer, then lm_head) is cut into 16-row tiles (tile t
//     belongs to CTA t % G) and 256-column items of 4 KB;
//   * each warp walks ONE flattened stream of (stage, tile, chunk) items across all stages of the token. Weights
//     do not depend on activations, so each warp keeps kRing items in flight in its own shared-memory ring
//     (cp.async, XOR-swizzled rows): HBM keeps streaming the next stages' weights while the warps wait at a
//     barrier or run attention;
//   * the GEMVs are exact: the stage input is staged once per CTA as fixed point (four int8 digit planes),
//     mma.sync.m16n8k32.s8 gives exact int32 per item, the planes fold into exact int64 row sums, and each row is
//     rounded once, then scaled and rounded at the reference's bf16 points (fused RMSNorm prologue; residual,
//     SiLU*up, lm_head argmax epilogues);
//   * three grid barriers per layer (after o_proj, gate|up and down_proj: a monotonic 64-bit arrival counter with
//     release/acquire ordering and a per-step epoch); after q|k|v and attention, dependency counters (q|k|v tiles
//     per kv group, kv heads done) replace them. Every wait is bounded and records EGPT_ERR_TIMEOUT instead of
//     hanging;
//   * attention runs as a stage: CTA t < nkv * nsplit takes kv head t / nsplit and key range t % nsplit of
//     whole 128-key blocks (q/k RMSNorm + RoPE + KV append, then the attention core of attention.cu with the
//     reference GPU kernel's softmax rounding; ranges exchange their maxima), the last range of each head
//     combines;
//   * the lm_head stage keeps (max, index) per CTA; the last CTA reduces them, writes the token and advances
//     the position and the step epoch;
//   * tensor parallelism (TP instantiation, 2/4/8 GPUs, one process each): the stage sizes are this rank's
//     shard; o_proj and down_proj CTAs store their rows' exact fp64 partial sums into every rank's exchange
//     region over NVLink as sequence-tagged LL slots, and the next stage on every rank waits for the slots it
//     reads and adds the g partials in rank order before the residual add and RMSNorm; those two stages need
//     no grid barrier. The lm_head's per-rank (logit, index) keys are exchanged the same way. The collective
//     lives inside the step kernel: no extra launch, no library call, no fence or flag round trip.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace egpt {
namespace ps {

constexpr int kNC = 16;                // warps (all compute)
constexpr int kCT = kNC * 32;          // threads
constexpr int kTileRows = 16;          // rows per tensor-core tile (mma m16n8k32)
constexpr int kChunkCols = 256;        // columns per stream item: 16 rows x 256 int8 = 4 KB
constexpr int kItemBytes = kTileRows * kChunkCols;
#ifndef EGPT_PS_RING
#define EGPT_PS_RING 2
#endif
constexpr int kRing = EGPT_PS_RING;    // stream items in flight per warp (shared-memory ring filled by cp.async)
constexpr int kSlot = kItemBytes + 64; // ring slot: the item, then its tile's 16 scales (up to 64 bytes)
constexpr int kXPad = 64;              // bytes between the digit planes of the staged input (bank spread)

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
  unsigned long long *qcnt;  // one-GPU step: q|k|v tiles written, per kv group (monotonic over steps and layers)
  unsigned long long *acnt;  // one-GPU step: kv heads whose attention output is written (monotonic)
  int part_bytes;            // shared memory for the layer stages' per-item row sums
  unsigned long long *trace;  // nullable: per-barrier %globaltimer stamps of CTA 0
  // tensor parallelism (TP instantiation only)
  int tp_rank, tp_world;
  int64_t v_embed;            // embedding rows (the whole vocabulary; V above is this rank's lm_head rows)
  char *xchg[8];              // exchange regions of all ranks, mapped in this process
  uint16_t *h2;               // second residual buffer
};

// A GEMV stage: n logical rows in tiles of 16 (GATEUP: tile t = gate rows 8t..8t+7 then up rows 8t..8t+7),
// k columns in chunks of 256; tile t belongs to CTA t % G. Layer stages split a tile's chunks over the CTA's
// warps (item i of the CTA's list -> warp i % 16) and reduce the exact partial sums through shared memory;
// the lm_head gives whole tiles to warps (tile t -> warp (t / G) % 16), so its argmax epilogue stays in the warp.
struct Stage {
  const int8_t *w;
  const void *s;
  int64_t n, k, tiles;
  int kind, nk;
  int ntl;  // tiles of this stage that belong to this CTA
};

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory"); }

// Stage table in shared memory (built once per launch from the device layer array): a stage's weights and
// scales are then found without a global load on the stream's critical path.
struct StageT {
  const int8_t *w;
  const void *s;
  int64_t n, k;
  int kind, ntl;  // ntl: this CTA's tiles of the stage (computed once per launch)
};
constexpr int kStabOffset = 256;  // after the 64-float reduction scratch

__device__ __forceinline__ StageT stage_from_layers(const Params &P, int s) {
  StageT st;
  st.ntl = 0;
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

__device__ __forceinline__ StageT *stage_table() {
  extern __shared__ __align__(128) uint8_t smem[];
  return (StageT *)(smem + kStabOffset);
}

__device__ __forceinline__ Stage stage_desc(const Params &P, int s) {
  const StageT &t = stage_table()[s];
  Stage st;
  st.w = t.w, st.s = t.s, st.n = t.n, st.k = t.k, st.kind = t.kind;
  st.tiles = st.n / kTileRows;
  st.nk = (int)((st.k + kChunkCols - 1) / kChunkCols);
  st.ntl = t.ntl;
  return st;
}

// Tiles of a stage that belong to this CTA (tile t belongs to CTA t % G; counted once per launch).
__device__ __forceinline__ int cta_tiles(const Stage &st) { return st.ntl; }

// Physical weight row of row r (< 16) of tile t.
__device__ __forceinline__ int64_t tile_row(const Stage &st, int64_t t, int r) {
  if (st.kind != GATEUP) return t * kTileRows + r;
  return r < 8 ? t * 8 + r : (st.n >> 1) + t * 8 + (r - 8);
}
// Byte offset of row r's scale in the slot's scale block (lm_head items carry their tile's scales).
__device__ __forceinline__ int scale_pos(int r, int esz) { return r * esz; }

// ------------------------------------------------------------------------------------------------ stream
// A warp's flattened stream of (stage, tile, chunk) items across all stages of the step (32-bit arithmetic,
// no divisions: this runs once per item on the stage's critical path).
struct Cursor {
  Stage st;
  int s;          // stage index; 4L + 1 = end of the stream
  int c;          // chunk
  int tile;       // tile index within the stage
  int tl, ntl;    // layer stages: tile-local index in this CTA's list, tiles of this CTA
  int item;       // layer stages: item index in the CTA's list (tl * nk + c)
};

__device__ __forceinline__ void cur_stage(const Params &P, Cursor &cu, int s) {
  const int w = threadIdx.x >> 5;
  for (; s <= 4 * P.L; ++s) {
    const Stage st = stage_desc(P, s);
    if (st.kind == LMHEAD) {
      const int t0 = (int)blockIdx.x + (int)gridDim.x * w;
      if (t0 < st.tiles) {
        cu.st = st, cu.s = s, cu.c = 0, cu.tile = t0, cu.tl = cu.ntl = cu.item = 0;
        return;
      }
    } else {
      const int ntl = (int)cta_tiles(st);
      if (w < ntl * st.nk) {
        cu.st = st, cu.s = s, cu.item = w, cu.ntl = ntl;
        cu.tl = 0, cu.c = w;
        while (cu.c >= st.nk) cu.c -= st.nk, ++cu.tl;
        cu.tile = (int)blockIdx.x + (int)gridDim.x * cu.tl;
        return;
      }
    }
  }
  cu.s = 4 * P.L + 1;
}
__device__ __forceinline__ void cur_next(const Params &P, Cursor &cu) {
  if (cu.st.kind == LMHEAD) {
    if (++cu.c < cu.st.nk) return;
    cu.c = 0;
    cu.tile += (int)gridDim.x * kNC;
    if (cu.tile >= cu.st.tiles) cur_stage(P, cu, cu.s + 1);
    return;
  }
  cu.item += kNC;
  cu.c += kNC;
  while (cu.c >= cu.st.nk) cu.c -= cu.st.nk, ++cu.tl;
  if (cu.tl >= cu.ntl) {
    cur_stage(P, cu, cu.s + 1);
    return;
  }
  cu.tile = (int)blockIdx.x + (int)gridDim.x * cu.tl;
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

// Copy one item into a ring slot: piece p (16 bytes) of tile row r lands at r * 256 + 16 * (p ^ 4 (r & 1)),
// which spreads the MMA fragment reads of rows g and g + 8 over all banks; for the lm_head, lanes 0..3 also
// copy the tile's scales. Pieces past the end of the row are not copied (their x digits are zero). The caller
// commits.
__device__ __forceinline__ void fill_item(const Params &P, const Cursor &cu, uint8_t *slot) {
  // piece id = 32 i + lane: row r = 2 i + (lane >> 4), piece pc = lane & 15 for every i, so a lane walks its rows
  // with one add per piece (rows 0-7 and 8-15 of a gate|up tile are two separate blocks)
  const int lane = threadIdx.x & 31, hi = lane >> 4, pc = lane & 15;
  const Stage &st = cu.st;
  const int64_t col0 = (int64_t)cu.c * kChunkCols;
  if (pc * 16 < st.k - col0) {
    const int8_t *g0 = st.w + tile_row(st, cu.tile, hi) * st.k + col0 + pc * 16;
    const int8_t *g1 = st.w + tile_row(st, cu.tile, 8 + hi) * st.k + col0 + pc * 16;
    uint8_t *d = slot + hi * kChunkCols + 16 * (pc ^ (hi << 2));
#pragma unroll
    for (int i = 0; i < 4; ++i) cp_async16(d + i * 2 * kChunkCols, g0 + (int64_t)i * 2 * st.k);
#pragma unroll
    for (int i = 0; i < 4; ++i) cp_async16(d + (8 + i * 2) * kChunkCols, g1 + (int64_t)i * 2 * st.k);
  }
  const int esz = P.scale_bf16 ? 2 : 4;
  if (st.kind == LMHEAD && lane * 16 < kTileRows * esz)
    cp_async16(slot + kItemBytes + lane * 16, (const char *)st.s + cu.tile * kTileRows * esz + lane * 16);
}

// ------------------------------------------------------------------------------------------------ sync
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier: arrivals accumulate on a monotonic counter; barrier idx (1-based) of the step with epoch
// base completes when the counter reaches (base + idx) * G. Bounded: records EGPT_ERR_TIMEOUT, returns false.
// Split in two so that work can go between arriving and waiting: grid_arrive publishes this CTA's writes and
// counts it in (thread 0: one release reduction); grid_wait spins (thread 0) until every CTA arrived.
template <bool TRACE>
__device__ __forceinline__ void grid_arrive(const Params &P, unsigned long long idx) {
  csync();
  if (threadIdx.x == 0) {
    if (TRACE && P.trace && blockIdx.x == 0) P.trace[2 * idx - 1] = globaltimer_ns();
    // release: the CTA's writes (ordered before by the CTA barrier) are visible before the count
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(P.bar) : "memory");
  }
}
template <bool TRACE>
__device__ bool grid_wait(const Params &P, unsigned long long base, unsigned long long idx, int *s_ok) {
  const unsigned long long target = (base + idx) * gridDim.x;
  if (threadIdx.x == 0) {
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
    if (TRACE && P.trace && blockIdx.x == 0) P.trace[2 * idx] = globaltimer_ns();
    *s_ok = ok;
  }
  csync();
  return *s_ok != 0;
}

// ------------------------------------------------------------------------------------------------ TP exchange
// Exchange region of a rank: LL slots of 16 bytes, each carrying a 64-bit payload as two 8-byte words
// (sequence number << 32 | 32 payload bits). Every 8-byte word is written and read in one piece, so a reader that
// finds the expected sequence number in both words has the payload of that exchange site: data and flag travel
// together, with no fence, flag or barrier between producer and consumer. Layout: lm_head keys [8] at 0,
// partial sums [2 = o_proj, down_proj][8 source ranks][H] at 4096.
constexpr int kXDataOff = 4096;
__device__ __forceinline__ char *xkey(char *x, int src) { return x + 16 * src; }
__device__ __forceinline__ char *xpart(char *x, int kind, int src, int H) {
  return x + kXDataOff + (((int64_t)kind * 8 + src) * H) * 16;
}
__device__ __forceinline__ void ll_store(char *p, unsigned long long v, unsigned seq) {
  const unsigned long long hi = (unsigned long long)seq << 32;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(hi | (v & 0xFFFFFFFFull)), "l"(hi | (v >> 32))
               : "memory");
}
__device__ __forceinline__ bool ll_load(const char *p, unsigned seq, unsigned long long &v) {
  unsigned long long w0, w1;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
  v = (w0 & 0xFFFFFFFFull) | (w1 << 32);
  return (unsigned)(w0 >> 32) == seq && (unsigned)(w1 >> 32) == seq;
}
// Sequence number of exchange site `site` (o_proj of layer l: 2l, down_proj: 2l + 1, lm_head: 2L) of step `epoch`,
// never 0 (the value of a zero-filled region).
__device__ __forceinline__ unsigned tp_seq(const Params &P, unsigned epoch, int site) {
  const unsigned long long n = (unsigned long long)epoch * (2ull * (unsigned long long)P.L + 1ull) + (unsigned)site;
  return (unsigned)(n % 0xFFFFFFFFull) + 1u;
}
// Bounded spin until slot p carries sequence number seq; on timeout (or another wait's error) records the error
// and returns whatever the slot holds.
__device__ __forceinline__ unsigned long long ll_wait(const char *p, unsigned seq, uint64_t t0) {
  unsigned long long v;
  for (int it = 0; !ll_load(p, seq, v); ++it) {
    if ((it & 63) == 63) {
      if (device_error_set()) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_device_error(EGPT_ERR_TIMEOUT);
        break;
      }
    }
  }
  return v;
}
// lm_head key of a rank's best (logit, global index): larger key = larger logit, then lower index (NaN above
// everything, -0 == +0), the order of argmax_better.
__device__ __forceinline__ unsigned long long argmax_key(float v, long long idx) {
  unsigned u = __float_as_uint(v);
  if (v != v) u = 0xFFFFFFFFu;
  else if (v == 0.f) u = 0x80000000u;
  else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}
// 2^e as a double (e within the normal range, which every staged-input exponent is).
__device__ __forceinline__ double pow2_f64(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

// Dependency wait (one-GPU step): thread 0 spins (bounded) until the monotonic counter c reaches target, then
// the CTA proceeds; replaces a grid barrier where only some producers matter (q|k|v tiles of one kv group before
// its attention, the kv heads' outputs before o_proj).
__device__ bool dep_wait(const unsigned long long *c, unsigned long long target, int *s_ok) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int it = 0; ld_acquire_u64(c) < target; ++it) {
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
    *s_ok = ok;
  }
  csync();
  return *s_ok != 0;
}

// Trace: stamp k (CTA 0, thread 0) of the second trace region: the moment stage k's input is ready (GEMV
// stages: staged and normalised; attention: this CTA's scores done).
template <bool TRACE>
__device__ __forceinline__ void stamp(const Params &P, int k) {
  if (TRACE && P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[4 + 10 * P.L + k] = globaltimer_ns();
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
constexpr int kGroups = kMaxPerThread / 4;  // a thread stages groups of 4 consecutive elements

// RMSNorm weights of a stage input, loaded into registers BEFORE the grid barrier that precedes the stage
// (they do not depend on the step), so their latency hides behind the barrier instead of adding to it.
// Thread t holds elements 4 (t + 512 j) .. + 3, j < kGroups.
// The weights stay as the loaded bf16 pairs and are widened where they are used: an instruction that consumed the
// loads here would stall the thread on their latency right away.
struct NormW {
  uint2 u[kGroups];
  __device__ __forceinline__ float w(int e) const {
    const uint32_t x = (e & 2) ? u[e >> 2].y : u[e >> 2].x;
    return (e & 1) ? bf16_hi(x) : bf16_lo(x);
  }
};
__device__ __forceinline__ void load_norm(const uint16_t *nw, int64_t k, NormW &n) {
#pragma unroll
  for (int j = 0; j < kGroups; ++j) {
    const int64_t i = 4 * ((int64_t)threadIdx.x + (int64_t)j * kCT);
    n.u[j] = make_uint2(0u, 0u);
    if (i < k) n.u[j] = *(const uint2 *)(nw + i);
  }
}

// y * 2^e for any e the staged inputs produce (exact unless the result underflows).
__device__ __forceinline__ float mul_pow2(float y, int e) {
  if (e < -126) {
    y *= __int_as_float((e + 100 + 127) << 23);
    e = -100;
  } else if (e > 127) {
    y *= __int_as_float((127 + 127) << 23);
    e -= 127;
  }
  return y * __int_as_float((e + 127) << 23);
}

// Padded stride of the digit planes for an input of k values.
__host__ __device__ __forceinline__ int x_stride(int64_t k) {
  return (int)((k + kChunkCols - 1) / kChunkCols * kChunkCols) + kXPad;
}

// Balanced base-256 digit d (0..3) of X, |X| < 2^30: X = sum_d digit_d 256^d with every digit in [-128, 127].
__device__ __forceinline__ void digits4(int X, int (&d)[4]) {
  d[0] = (int)(int8_t)(X & 0xFF);
  X = (X - d[0]) >> 8;
  d[1] = (int)(int8_t)(X & 0xFF);
  X = (X - d[1]) >> 8;
  d[2] = (int)(int8_t)(X & 0xFF);
  d[3] = (X - d[2]) >> 8;
}

// Stage an input vector of k bf16 values (k a multiple of 4; optionally RMSNorm'd with the preloaded weights
// nw, HF rounding points) as exact fixed point: x[i] = X[i] * 2^E with |X| < 2^30, E from a bound on the largest
// |x[i]| (values far below it round to the fixed-point grid), and X split into four balanced base-256 digit
// planes xd[d][i] in [-128, 127], zero-padded to whole 256-column chunks. One CTA reduction gives both the sum
// of squares and the bound (max |x w| * rsqrt(...) * (1 + 2^-8)^2 covers the two bf16 roundings of the norm).
// copy_to (nullable) receives the raw values (layer 0: h = embedding row). Returns E.
// TP (tin non-null): the input is the residual sum h' = bf16(src + bf16(fp32(sum_r part_r) * s)) of the previous
// o_proj / down_proj, from its np ranks' exact partials (added in rank order) and row scales; copy_to gets h'.
struct TpIn {
  const char *parts;  // LL slots of rank r's partials at parts + 16 (r k + i)
  const void *s;      // row scales of the stage that produced them
  int np, s_bf16;
  unsigned seq;       // sequence number of the exchange site
};
template <bool TP>
__device__ int stage_input(const uint16_t *src, int64_t k, const NormW *nw, float eps, int8_t *xd, float *red,
                           uint16_t *copy_to, const TpIn *tin) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float v[kMaxPerThread];
  double ss = 0.0;  // the bf16 squares are exact in fp32; their fp64 sum is exact in practice and order-free
  float mx = 0.f;
  if (TP && tin) {
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (i < k) {
        const uint2 u = __ldcg((const uint2 *)(src + i));
        float sc[4];
        if (tin->s_bf16) {
          const uint2 su = *(const uint2 *)((const uint16_t *)tin->s + i);
          sc[0] = bf16_lo(su.x), sc[1] = bf16_hi(su.x), sc[2] = bf16_lo(su.y), sc[3] = bf16_hi(su.y);
        } else {
          const float4 sf = *(const float4 *)((const float *)tin->s + i);
          sc[0] = sf.x, sc[1] = sf.y, sc[2] = sf.z, sc[3] = sf.w;
        }
        // partials of two ranks per pass: eight slot loads in flight before the first check
        double a[4] = {0.0, 0.0, 0.0, 0.0};
        const uint64_t t0 = globaltimer_ns();
        for (int r = 0; r < tin->np; r += 2) {
          const char *p0 = tin->parts + ((int64_t)r * k + i) * 16;
          const char *p1 = p0 + k * 16;
          const bool two = r + 1 < tin->np;
          unsigned long long v[8];
          bool ok = true;
#pragma unroll
          for (int q = 0; q < 4; ++q) ok = ll_load(p0 + 16 * q, tin->seq, v[q]) && ok;
          if (two) {
#pragma unroll
            for (int q = 0; q < 4; ++q) ok = ll_load(p1 + 16 * q, tin->seq, v[4 + q]) && ok;
          }
          if (!ok) {  // not all there yet: wait slot by slot
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = ll_wait(p0 + 16 * q, tin->seq, t0);
            if (two) {
#pragma unroll
              for (int q = 0; q < 4; ++q) v[4 + q] = ll_wait(p1 + 16 * q, tin->seq, t0);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) a[q] += __longlong_as_double((long long)v[q]);
          if (two) {
#pragma unroll
            for (int q = 0; q < 4; ++q) a[q] += __longlong_as_double((long long)v[4 + q]);
          }
        }
        const float hs[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = round_bf16(hs[q] + round_bf16(__double2float_rn(a[q]) * sc[q]));
        if (copy_to)
          *(uint2 *)(copy_to + i) = make_uint2((uint32_t)f32_to_bf16_bits(o[0]) | ((uint32_t)f32_to_bf16_bits(o[1]) << 16),
                                               (uint32_t)f32_to_bf16_bits(o[2]) | ((uint32_t)f32_to_bf16_bits(o[3]) << 16));
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) v[4 * j + q] = o[q];
    }
  } else {
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
      uint2 u = make_uint2(0u, 0u);
      if (i < k) {
        u = __ldcg((const uint2 *)(src + i));
        if (copy_to) *(uint2 *)(copy_to + i) = u;
      }
      v[4 * j] = bf16_lo(u.x), v[4 * j + 1] = bf16_hi(u.x), v[4 * j + 2] = bf16_lo(u.y), v[4 * j + 3] = bf16_hi(u.y);
    }
  }
#pragma unroll
  for (int e = 0; e < kMaxPerThread; ++e) {
    ss += (double)(v[e] * v[e]);
    mx = fmaxf(mx, fabsf(nw ? v[e] * nw->w(e) : v[e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  mx = warp_max(mx);
  double *redd = (double *)red;  // red: 16 doubles (bytes 0-127), then the maxima at red[32..47]
  if (lane == 0) redd[warp] = ss, red[32 + warp] = mx;
  csync();
  double tot = 0.0;
  float bound = red[32];
#pragma unroll
  for (int w = 0; w < kNC; ++w) tot += redd[w];
#pragma unroll
  for (int w = 1; w < kNC; ++w) bound = fmaxf(bound, red[32 + w]);
  if (nw) {
    const float inv = rsqrtf((float)tot / (float)k + eps);
#pragma unroll
    for (int e = 0; e < kMaxPerThread; ++e) v[e] = round_bf16(round_bf16(v[e] * inv) * nw->w(e));
    bound = bound * inv * 1.0079f;
  }
  const int ex = bound > 0.f ? ((__float_as_int(bound) >> 23) & 0xFF) - 127 : 0;  // floor(log2 bound)
  const int E = ex - 29;
  const int xs = x_stride(k);
  const int64_t kpad = xs - kXPad;
#pragma unroll
  for (int j = 0; j < kGroups; ++j) {
    const int64_t i = 4 * ((int64_t)t + (int64_t)j * kCT);
    if (i < kpad) {
      uint32_t word[4] = {0u, 0u, 0u, 0u};
      if (i < k) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          int d[4];
          digits4(__float2int_rn(mul_pow2(v[4 * j + q], -E)), d);
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

// Inputs wider than kMaxPerThread * kCT values (no norm, no residual: the down_proj input of a 12288-wide MLP):
// the same fixed point as stage_input in two passes over the vector, one for the bound and one (L2 hits) for the
// digit planes, so no thread holds more than four values.
__device__ int stage_input_wide(const uint16_t *src, int64_t k, int8_t *xd, float *red) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float mx = 0.f;
  for (int64_t i = 4 * (int64_t)t; i < k; i += 4 * kCT) {
    const uint2 u = __ldcg((const uint2 *)(src + i));
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(bf16_lo(u.x)), fabsf(bf16_hi(u.x))), fmaxf(fabsf(bf16_lo(u.y)), fabsf(bf16_hi(u.y)))));
  }
  mx = warp_max(mx);
  if (lane == 0) red[kNC + warp] = mx;
  csync();
  float bound = red[kNC];
#pragma unroll
  for (int w = 1; w < kNC; ++w) bound = fmaxf(bound, red[kNC + w]);
  const int ex = bound > 0.f ? ((__float_as_int(bound) >> 23) & 0xFF) - 127 : 0;  // floor(log2 bound)
  const int E = ex - 29;
  const int xs = x_stride(k);
  const int64_t kpad = xs - kXPad;
  for (int64_t i = 4 * (int64_t)t; i < kpad; i += 4 * kCT) {
    uint32_t word[4] = {0u, 0u, 0u, 0u};
    if (i < k) {
      const uint2 u = __ldcg((const uint2 *)(src + i));
      const float v[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        int d[4];
        digits4(__float2int_rn(mul_pow2(v[q], -E)), d);
#pragma unroll
        for (int p = 0; p < 4; ++p) word[p] |= ((uint32_t)d[p] & 0xFFu) << (8 * q);
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) *(uint32_t *)(xd + (int64_t)p * xs + i) = word[p];
  }
  csync();
  return E;
}

// ------------------------------------------------------------------------------------------------ GEMV stage
struct Best {
  float v;
  int i;
};

struct Stream {
  Cursor cur, fill;  // consumption and ring-fill (kRing items ahead of cur) cursors
  int slot;          // ring slot holding cur's item
  uint8_t *ring;     // this warp's kRing slots
};

// Start the stream: kRing items in flight (one commit group each, empty past the end).
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
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float load_scale(const Params &P, const void *s, int64_t row) {
  return P.scale_bf16 ? bf16_bits_to_f32(((const uint16_t *)s)[row]) : ((const float *)s)[row];
}

// Epilogue inputs of a layer stage for thread e (< this CTA's tiles x 16, or x 8 for gate/up pairs): its rows'
// scales and (o, down) the residual row, requested when the stage starts and consumed after its items.
// Raw bits as loaded (bf16 in the low half, or fp32 scales), widened in the epilogue: converting at the load would
// stall the thread on the load's latency at the start of the stage.
struct EpiIn {
  uint32_t s0, s1, res;
};
__device__ __forceinline__ uint32_t raw_scale(const Params &P, const void *s, int64_t row) {
  return P.scale_bf16 ? (uint32_t)((const uint16_t *)s)[row] : __float_as_uint(((const float *)s)[row]);
}
__device__ __forceinline__ float scale_of(const Params &P, uint32_t raw) {
  return P.scale_bf16 ? __uint_as_float(raw << 16) : __uint_as_float(raw);
}
template <bool TP>
__device__ __forceinline__ void load_epi(const Params &P, int gs, EpiIn &in) {
  const Stage sd = stage_desc(P, gs);
  in.s0 = in.s1 = in.res = 0u;
  if (sd.kind == LMHEAD) return;
  const int per_tile = sd.kind == GATEUP ? 8 : kTileRows;
  const int e = threadIdx.x;
  if (e >= cta_tiles(sd) * per_tile) return;
  const int sh = per_tile == 8 ? 3 : 4;
  const int64_t tile = blockIdx.x + (int64_t)gridDim.x * (e >> sh);
  const int r = e & (per_tile - 1);
  in.s0 = raw_scale(P, sd.s, tile_row(sd, tile, r));
  if (sd.kind == GATEUP) in.s1 = raw_scale(P, sd.s, tile_row(sd, tile, r + 8));
  if (!TP && (sd.kind == OPROJ || sd.kind == DOWN)) in.res = (uint32_t)__ldcg(P.h + tile * kTileRows + r);
}

// Consume this warp's items of stage s (the stream's cursor is at stage s or later). Per item and lane (g =
// lane / 4, t = lane % 4): 16 bytes of tile rows g and g + 8 and (g < 4) 16 bytes of digit plane g for each of
// four 64-column steps feed two int8 tensor-core MMAs; column d of the accumulator is row . plane d, exact in
// int32, and lane t = 0 folds the planes into the exact int64 row sums. Every consumed slot is refilled at once
// with the item kRing ahead, whatever stage it belongs to. Layer stages leave each item's sums in `part` and,
// after a CTA barrier, threads e < (CTA tiles) x 16 (x 8 for gate/up pairs) add a row's items in order and
// apply the epilogue; their scales and residuals are fetched before the items stream. The lm_head epilogue
// (bf16 logits, argmax) runs in the warp that owns the tile.
// TP: o_proj / down_proj rows store their exact partial sum (fp64, before the scale) into every rank's region,
// tagged with the exchange site's sequence number tseq.
template <bool TP>
__device__ void gemv_stage(const Params &P, int s, Stream &S, const int8_t *xd, int E, long long *part,
                           const EpiIn &ein, Best &best, unsigned tseq) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const Stage sd = stage_desc(P, s);
  const bool lm = sd.kind == LMHEAD;
  const int per_tile = sd.kind == GATEUP ? 8 : kTileRows;
  const int e = threadIdx.x;
  const bool epi = !lm && e < cta_tiles(sd) * per_tile;
  const int esh = per_tile == 8 ? 3 : 4;
  const int64_t etile = blockIdx.x + (int64_t)gridDim.x * (e >> esh);
  const int er = e & (per_tile - 1);
  const EpiIn er_raw = ein;  // widened after the items (scale_of, bf16 residual)
  const int xs = x_stride(sd.k);
  int c4[4] = {0, 0, 0, 0};
  while (S.cur.s == s) {
    const int c = S.cur.c;
    const int64_t tile = S.cur.tile, item = S.cur.item;
    const bool last = c == sd.nk - 1;
    if (!lm || c == 0) c4[0] = c4[1] = c4[2] = c4[3] = 0;
    cp_async_wait<kRing - 1>();  // this lane's copies of the item have landed
    __syncwarp();                // ... and every other lane's
    const uint8_t *slot = S.ring + S.slot * kSlot;
    const int8_t *xb = xd + (int64_t)c * kChunkCols + g * xs + 16 * t;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sw = 16 * ((4 * j + t) ^ ((g & 1) << 2));
      const uint4 wa = *(const uint4 *)(slot + g * kChunkCols + sw);
      const uint4 wb = *(const uint4 *)(slot + (g + 8) * kChunkCols + sw);
      uint4 xv = make_uint4(0u, 0u, 0u, 0u);
      if (g < 4) xv = *(const uint4 *)(xb + 64 * j);
      mma_s8(c4, wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
      mma_s8(c4, wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
    }
    float s0 = 0.f, s1 = 0.f;
    if (lm && last && t == 0) {
      const uint8_t *sb = slot + kItemBytes;
      if (P.scale_bf16) {
        s0 = bf16_bits_to_f32(*(const uint16_t *)(sb + scale_pos(g, 2)));
        s1 = bf16_bits_to_f32(*(const uint16_t *)(sb + scale_pos(g + 8, 2)));
      } else {
        s0 = *(const float *)(sb + scale_pos(g, 4));
        s1 = *(const float *)(sb + scale_pos(g + 8, 4));
      }
    }
    __syncwarp();  // every lane's reads of the slot are done before any lane refills it
    if (!cur_end(P, S.fill)) {
      fill_item(P, S.fill, S.ring + S.slot * kSlot);
      cur_next(P, S.fill);
    }
    cp_async_commit();
    S.slot = S.slot + 1 == kRing ? 0 : S.slot + 1;
    cur_next(P, S.cur);
    if (lm && !last) continue;
    // digit planes 2t, 2t+1 of rows g, g + 8 sit in lane t: lane t = 0 gathers planes 2, 3 from lane t = 1
    const int o0 = __shfl_down_sync(0xffffffffu, c4[0], 1), o1 = __shfl_down_sync(0xffffffffu, c4[1], 1);
    const int o2 = __shfl_down_sync(0xffffffffu, c4[2], 1), o3 = __shfl_down_sync(0xffffffffu, c4[3], 1);
    if (t != 0) continue;
    const long long T0 = (long long)c4[0] + ((long long)c4[1] << 8) + ((long long)o0 << 16) + ((long long)o1 << 24);
    const long long T1 = (long long)c4[2] + ((long long)c4[3] << 8) + ((long long)o2 << 16) + ((long long)o3 << 24);
    if (!lm) {
      part[item * kTileRows + g] = T0;
      part[item * kTileRows + g + 8] = T1;
      continue;
    }
    const int64_t r0 = tile * kTileRows + g, r1 = r0 + 8;
    const float l0 = round_bf16(mul_pow2(__ll2float_rn(T0), E) * s0), l1 = round_bf16(mul_pow2(__ll2float_rn(T1), E) * s1);
    if (P.logits) {
      P.logits[r0] = f32_to_bf16_bits(l0);
      P.logits[r1] = f32_to_bf16_bits(l1);
    }
    if (argmax_better(l0, (int)r0, best.v, best.i)) best.v = l0, best.i = (int)r0;
    if (argmax_better(l1, (int)r1, best.v, best.i)) best.v = l1, best.i = (int)r1;
  }
  if (lm) return;
  csync();  // all items' sums are in `part`
  if (!epi) return;
  const int64_t tl = e >> esh;
  long long T0 = 0, T1 = 0;
  for (int c = 0; c < sd.nk; ++c) {
    T0 += part[(tl * sd.nk + c) * kTileRows + er];
    if (sd.kind == GATEUP) T1 += part[(tl * sd.nk + c) * kTileRows + er + 8];
  }
  const float y0 = mul_pow2(__ll2float_rn(T0), E);
  switch (sd.kind) {
    case QKV: P.qkv[etile * kTileRows + er] = f32_to_bf16_bits(y0 * scale_of(P, er_raw.s0)); break;
    case OPROJ:
    case DOWN:
      if (TP) {
        const double y = __ll2double_rn(T0) * pow2_f64(E);  // exact: |T0| < 2^53
        const int64_t row = etile * kTileRows + er;
        const unsigned long long bits = (unsigned long long)__double_as_longlong(y);
        for (int q = 0; q < P.tp_world; ++q)
          ll_store(xpart(P.xchg[q], sd.kind == OPROJ ? 0 : 1, P.tp_rank, P.H) + row * 16, bits, tseq);
      } else {
        P.h[etile * kTileRows + er] =
            f32_to_bf16_bits(__uint_as_float(er_raw.res << 16) + round_bf16(y0 * scale_of(P, er_raw.s0)));
      }
      break;
    default: {  // GATEUP: act = bf16(bf16(silu(gate)) * up)
      const float gt = round_bf16(y0 * scale_of(P, er_raw.s0)),
                  up = round_bf16(mul_pow2(__ll2float_rn(T1), E) * scale_of(P, er_raw.s1));
      P.act[etile * 8 + er] = f32_to_bf16_bits(round_bf16(gt / (1.0f + expf(-gt))) * up);
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

template <int DPL, int GRP, bool TRACE>
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
  t.prefetch_v = 1;
  attn_pass_a<DPL, GRP, true>(t, S);
  stamp<TRACE>(P, tslot);
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
  attn_walk<DPL, GRP, true, kCT, true>(t, S);
  AttnOut o;
  o.out = P.attn;
  o.part = P.attn_ws;
  o.cnt = P.attn_cnt + g;
  o.g = g;
  o.split = split;
  o.nsplit = nsplit;
  o.max_split = P.max_split;
  o.busy = min(kAttnWarps, ntiles);
  o.done = P.acnt;  // read by the one-GPU step's o_proj; the tensor-parallel step keeps a grid barrier instead
  attn_finish<DPL, GRP, true, kCT>(S, o);
}

// ------------------------------------------------------------------------------------------------ kernel
template <int DPL, int GRP, bool TP, bool WIDE, bool TRACE>
__global__ void __launch_bounds__(kCT, 1) decode_step_kernel(const Params P) {
  extern __shared__ __align__(128) uint8_t smem[];
  float *red = (float *)smem;                    // 64 floats
  // stage table (4L + 1 entries) and a copy of the layer array, then the weight rings
  const int stab_bytes = ((4 * P.L + 1) * (int)sizeof(StageT) + 127) / 128 * 128;
  const int lay_bytes = (P.L * (int)sizeof(egpt_qwen3_layer) + 127) / 128 * 128;
  egpt_qwen3_layer *layers = (egpt_qwen3_layer *)(smem + kStabOffset + stab_bytes);
  for (int i = threadIdx.x; i <= 4 * P.L; i += kCT) {
    StageT t = stage_from_layers(P, i);
    const int tiles = (int)(t.n / kTileRows), b = blockIdx.x;
    t.ntl = b < tiles ? (tiles - b + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    stage_table()[i] = t;
  }
  for (int i = threadIdx.x; i < P.L; i += kCT) layers[i] = P.layers[i];
  csync();
  uint8_t *ring = smem + kStabOffset + stab_bytes + lay_bytes;  // kNC x kRing weight slots
  long long *part = (long long *)(ring + kNC * kRing * kSlot);  // layer stages: per-item exact row sums
  float *u = (float *)((uint8_t *)part + P.part_bytes);  // union: staged input digit planes / attention scratch
  int8_t *xd = (int8_t *)u;
  __shared__ int s_flag;
  __shared__ float s_bv[kNC];
  __shared__ int s_bi[kNC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Start the weight stream immediately: it does not depend on the token, the position or the activations.
  Stream S;
  stream_start(P, S, ring + (size_t)warp * kRing * kSlot);

  const unsigned long long nb = 3ull * (unsigned long long)P.L;  // grid barriers per step
  const unsigned epoch = *(volatile unsigned *)P.epoch;
  const unsigned long long base = (unsigned long long)epoch * nb;
  unsigned long long bidx = 0;
  bool ok = true;
  Best best{-INFINITY, 0x7fffffff};
  const int64_t pos = *P.position;
  const int64_t tok = *P.token;
  if (pos < 0 || pos >= P.cap || tok < 0 || tok >= P.v_embed) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    ok = false;
  }
  const int bps = split_blocks(pos + 1, P.max_split);  // attention: ranges of bps 128-key blocks
  const int nsplit = split_count(pos + 1, bps);
  if (bps * kRefBlock > AttnScratch<DPL, GRP>::KS) {  // excluded on the host for positions < cap
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    ok = false;
  }
  if (TRACE && P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[0] = globaltimer_ns();

  // Everything a stage reads that does not depend on the step (norm weights, the attention prologue's norm
  // weights and RoPE row, the KV ranges) is requested before the barrier that precedes the stage.
  const bool attn_cta = (int)blockIdx.x < P.NKV * nsplit;
  NormW nw;
  AttnPre<DPL> pre;
  EpiIn ein;
  // One pass per stage: 5 per layer (q|k|v, attention, o, gate|up, down), then the lm_head. Every stage body and
  // every request helper has ONE site in the code: the kernel's executed instruction footprint decides how fast a
  // stage that runs once per layer executes. Pass st = -1 only issues the requests of stage 0.
  for (int st = -1; st <= 5 * P.L; ++st) {
    if (st >= 0) {
      const int l = st / 5, ph = st == 5 * P.L ? 5 : st % 5;
      const egpt_qwen3_layer &Ly = layers[l < P.L ? l : P.L - 1];
      if (ph == 1) {
        // ---- attention (q/k norm + RoPE + KV append + split-K softmax . V + combine); one GPU: starts once the
        //      q|k|v tiles of its kv group are written (no grid barrier after q|k|v)
        if (!TP && attn_cta)
          ok = dep_wait(P.qcnt + blockIdx.x / nsplit,
                        ((unsigned long long)epoch * P.L + l + 1) * (unsigned long long)((GRP + 2) * DPL * 32 / kTileRows),
                        &s_flag) && ok;
        if (ok && attn_cta) attention_task<DPL, GRP, TRACE>(P, Ly, blockIdx.x, nsplit, bps, pos, u, pre, st);
      } else {
        // one GPU: o_proj starts once every kv head's attention output is written (no grid barrier after attention)
        if (!TP && ph == 2)
          ok = dep_wait(P.acnt, ((unsigned long long)epoch * P.L + l + 1) * (unsigned long long)P.NKV, &s_flag) && ok;
        // ---- GEMV stages: q|k|v = Wqkv . RMSNorm(h) (layer 0: h = embed[token], CTA 0 stores it);
        //      h += Wo . attn;  act = silu(Wg . RMSNorm(h)) * (Wu . RMSNorm(h));  h += Wdown . act;
        //      token = argmax(lm_head . RMSNorm(h))
        const uint16_t *src = ph == 2 ? P.attn : ph == 4 ? P.act : (ph == 0 && l == 0) ? P.embed + (ok ? tok : 0) * P.H : P.h;
        const int64_t k = ph == 2 ? (int64_t)P.NQ * P.D : ph == 4 ? P.I : P.H;
        const bool norm = ph == 0 || ph == 3 || ph == 5;
        uint16_t *copy_to = (st == 0 && blockIdx.x == 0) ? P.h : nullptr;
        TpIn tin;
        const TpIn *tinp = nullptr;
        if (TP && ((ph == 0 && l > 0) || ph == 3 || ph == 5)) {
          // residual sums: q|k|v and lm_head read h2 + down_proj partials (q|k|v: CTA 0 stores the sum in h),
          // gate|up reads h + o_proj partials (CTA 0 stores the sum in h2)
          const bool after_o = ph == 3;
          src = after_o ? P.h : P.h2;
          tin.parts = xpart(P.xchg[P.tp_rank], after_o ? 0 : 1, 0, P.H);
          tin.s = after_o ? Ly.s_o : layers[l - 1].s_down;
          tin.np = P.tp_world;
          tin.s_bf16 = P.scale_bf16;
          tin.seq = tp_seq(P, epoch, after_o ? 2 * l : 2 * (l - 1) + 1);
          tinp = &tin;
          copy_to = blockIdx.x != 0 || ph == 5 ? nullptr : after_o ? P.h2 : P.h;
        }
        const int gs = ph == 5 ? 4 * P.L : 4 * l + (ph == 0 ? 0 : ph - 1);
        // TP shards leave some CTAs without tiles in a stage: those skip it (and its partial-sum reads); CTA 0
        // always has tile 0 and stores the residual sum
        if (!TP || ph == 5 || cta_tiles(stage_desc(P, gs)) > 0) {
          const int E = (WIDE && k > kMaxPerThread * kCT)
                            ? stage_input_wide(src, k, xd, red)
                            : stage_input<TP>(src, k, norm ? &nw : nullptr, P.eps, xd, red, copy_to, tinp);
          stamp<TRACE>(P, st);
          load_epi<TP>(P, gs, ein);  // consumed after the items
          gemv_stage<TP>(P, gs, S, xd, E, part, ein, best,
                         (TP && (ph == 2 || ph == 4)) ? tp_seq(P, epoch, 2 * l + (ph == 4)) : 0u);
          if (!TP && ph == 0) {  // count this CTA's q|k|v tiles in, per kv group, once their rows are written
            csync();
            if (threadIdx.x == 0) {
              constexpr int kTilesPerHead = DPL * 32 / kTileRows;
              const int tiles = (P.NQ + 2 * P.NKV) * kTilesPerHead;
              for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                const int hd = t / kTilesPerHead;
                const int g = hd < P.NQ ? hd / GRP : hd < P.NQ + P.NKV ? hd - P.NQ : hd - P.NQ - P.NKV;
                red_release_add_u64(P.qcnt + g, 1ull);
              }
            }
          }
        }
      }
    }
    if (st < 5 * P.L) {
      // TP: no barrier after o_proj and down_proj: the next stage waits for the sequence-tagged partial sums of
      // every rank (which every CTA of every rank stored), and that wait orders everything the barrier did
      // one GPU: no barrier after q|k|v and attention either: dependency counters order those stages
      const bool bar = TP ? !(st >= 0 && (st % 5 == 2 || st % 5 == 4)) : !(st >= 0 && (st % 5 == 0 || st % 5 == 1));
      // step-invariant inputs of stage st + 1, requested between arriving at the barrier that precedes it and
      // waiting there (after the arrival's fence, which would otherwise wait for them): norm weights, the
      // attention prologue's weights and RoPE row, KV ranges
      if (st >= 0 && bar) grid_arrive<TRACE>(P, bidx + 1);
      const int n = st + 1, ln = n / 5, pn = n == 5 * P.L ? 5 : n % 5;
      const egpt_qwen3_layer &Ln = layers[ln < P.L ? ln : P.L - 1];
      if (pn == 0 || pn == 3 || pn == 5)
        load_norm(pn == 5 ? P.final_norm : (const uint16_t *)(pn == 0 ? Ln.ln_in : Ln.ln_post), P.H, nw);
      if (pn == 1 && attn_cta) attn_preload<DPL, GRP>(P, Ln, blockIdx.x, nsplit, bps, pos, pre);
      if (pn == 0 && attn_cta) attn_prefetch_kv<DPL, GRP>(P, Ln, blockIdx.x, nsplit, bps, pos);
      if (st >= 0 && bar) ok = grid_wait<TRACE>(P, base, ++bidx, &s_flag) && ok;
    }
  }
  if (TRACE && P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[1 + 10 * P.L] = globaltimer_ns();
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
      int64_t next = bi;
      if (TP) {  // every rank's best key to every rank, then the same maximum everywhere
        const unsigned seq = tp_seq(P, epoch, 2 * P.L);
        const unsigned long long key = argmax_key(bv, (long long)bi + (long long)P.tp_rank * P.V);
        for (int q = 0; q < P.tp_world; ++q) ll_store(xkey(P.xchg[q], P.tp_rank), key, seq);
        const uint64_t t0 = globaltimer_ns();
        unsigned long long bk = 0ull;
        for (int r = 0; r < P.tp_world; ++r) {
          const unsigned long long kr = ll_wait(xkey(P.xchg[P.tp_rank], r), seq, t0);
          bk = kr > bk ? kr : bk;
        }
        if (device_error_set()) ok = false;
        next = (int64_t)(0xFFFFFFFFu - (unsigned)(bk & 0xFFFFFFFFull));
      }
      *P.token = ok ? next : 0;
      *P.position += 1;
      *P.lm_cnt = 0u;
      *P.epoch += 1u;
      __threadfence();
      if (TRACE && P.trace) P.trace[2 + 10 * P.L] = globaltimer_ns();
    }
  }
}

// Shared memory for the per-item row sums of the largest layer stage: (its tiles per CTA) x chunks x 16 x 8 B.
static size_t part_bytes(const egpt_qwen3_plan *Pl, int G) {
  const int64_t D = Pl->head_dim, H = Pl->hidden, I = Pl->intermediate;
  const int64_t nk[4] = {(H + kChunkCols - 1) / kChunkCols, (Pl->n_q_heads * D + kChunkCols - 1) / kChunkCols,
                         (H + kChunkCols - 1) / kChunkCols, (I + kChunkCols - 1) / kChunkCols};
  const int64_t n[4] = {(Pl->n_q_heads + 2 * Pl->n_kv_heads) * D, H, 2 * I, H};
  int64_t items = 0;
  for (int i = 0; i < 4; ++i) items = std::max(items, (n[i] / kTileRows + G - 1) / G * nk[i]);
  return (size_t)items * kTileRows * 8;
}

// The %globaltimer stamps of plan->trace live in their own instantiation: the production kernel carries no
// trace code (its instruction footprint is on the critical path of every stage).
template <int DPL, int GRP, bool TP, bool WIDE = false>
static cudaError_t launch(const Params &P, size_t smem, cudaStream_t st) {
  auto kern = P.trace ? decode_step_kernel<DPL, GRP, TP, WIDE, true> : decode_step_kernel<DPL, GRP, TP, WIDE, false>;
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

// Step synchronisation words: u64 barrier counter at 0, u32 epoch at 8, u64 attention-done counter at 64, u64
// q|k|v-tile counters per kv group from 72.
constexpr int kMaxSyncGroups = 240;
extern "C" size_t egpt_step_sync_ws_bytes(void) { return 72 + 8 * kMaxSyncGroups; }

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
  if (NKV > kMaxSyncGroups) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: more than %d kv heads", kMaxSyncGroups);
  const bool shape_ok = (D == 128 && (grp == 2 || grp == 4)) || (D == 32 && grp == 2);
  if (!shape_ok) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: head_dim %d / group %d not built", D, grp);
  // inputs staged in registers: hidden and nq*d up to kMaxPerThread * kCT; the intermediate (down_proj input,
  // no norm) up to twice that on the one-GPU head_dim-128 / group-4 instantiation (two-pass staging)
  const int64_t reg_max = (int64_t)ps::kMaxPerThread * ps::kCT;
  const bool wide_ok = D == 128 && grp == 4 && Pl->tp_world <= 1;
  if (H % 16 || I % 16 || ((int64_t)NQ * D) % 16 || Pl->vocab % 16 || std::max<int64_t>(H, (int64_t)NQ * D) > reg_max ||
      I > (wide_ok ? 2 * reg_max : reg_max))
    return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: hidden, intermediate, nq*d and vocab must be multiples "
                     "of 16, hidden and nq*d at most %lld, intermediate at most %lld", (long long)reg_max,
                     (long long)(wide_ok ? 2 * reg_max : reg_max));
  const int G = num_sms();
  if (G > kArgmaxMaxCtas) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: too many SMs");
  if (Pl->tp_world > 1) {
    const int g = Pl->tp_world;
    if (g != 2 && g != 4 && g != 8) return set_error(EGPT_ERR_ARG, "decode_step_persistent: tp_world must be 2, 4 or 8");
    if (Pl->tp_rank < 0 || Pl->tp_rank >= g) return set_error(EGPT_ERR_ARG, "decode_step_persistent: tp_rank out of range");
    if (!Pl->h2) return set_error(EGPT_ERR_ARG, "decode_step_persistent: tensor parallelism needs h2");
    for (int r = 0; r < g; ++r)
      if (!Pl->tp_xchg[r] || (uintptr_t)Pl->tp_xchg[r] % 256)
        return set_error(EGPT_ERR_ARG, "decode_step_persistent: exchange region of rank %d missing or not 256-byte aligned", r);
    if (Pl->vocab * g > 0x7fffffffLL) return set_error(EGPT_ERR_SHAPE, "decode_step_persistent: vocabulary too large");
  } else if (Pl->tp_world < 0) {
    return set_error(EGPT_ERR_ARG, "decode_step_persistent: negative tp_world");
  }
  // weights and each tile's scales are copied in 16-byte pieces
  const size_t sal = 16;
  bool aligned = (uintptr_t)Pl->w_lm % 16 == 0 && (uintptr_t)Pl->s_lm % sal == 0;
  for (int l = 0; l < Pl->n_layers; ++l) {
    const egpt_qwen3_layer &Ly = Pl->layers[l];
    aligned = aligned && (uintptr_t)Ly.w_qkv % 16 == 0 && (uintptr_t)Ly.w_o % 16 == 0 &&
              (uintptr_t)Ly.w_gu % 16 == 0 && (uintptr_t)Ly.w_down % 16 == 0 && (uintptr_t)Ly.s_qkv % sal == 0 &&
              (uintptr_t)Ly.s_o % sal == 0 && (uintptr_t)Ly.s_gu % sal == 0 && (uintptr_t)Ly.s_down % sal == 0;
  }
  if (!aligned)
    return set_error(EGPT_ERR_ALIGN, "decode_step_persistent: weights and scales must be 16-byte aligned");
  if (Pl->attn_ws_bytes < egpt_attn_ws_bytes(1, NQ, NKV, D, Pl->attn_max_split) ||
      Pl->lm_ws_bytes < egpt_lm_head_ws_bytes(Pl->vocab))
    return set_error(EGPT_ERR_WORKSPACE, "decode_step_persistent: workspace too small");
  // shared memory: reduction scratch + weight ring + union(staged input digit planes, attention scratch)
  const int64_t kmax = std::max<int64_t>({H, I, (int64_t)NQ * D});
  const size_t attn_bytes = D == 32 ? sizeof(AttnScratch<1, 2>) : grp == 2 ? sizeof(AttnScratch<4, 2>) : sizeof(AttnScratch<4, 4>);
  const size_t stab = ((size_t)(4 * Pl->n_layers + 1) * sizeof(ps::StageT) + 127) / 128 * 128 +
                      ((size_t)Pl->n_layers * sizeof(egpt_qwen3_layer) + 127) / 128 * 128;
  const size_t smem = ps::kStabOffset + stab + (size_t)ps::kNC * ps::kRing * ps::kSlot + ps::part_bytes(Pl, G) +
                      std::max<size_t>(4 * (size_t)ps::x_stride(kmax), (attn_bytes + 15) / 16 * 16);
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
  P.acnt = (unsigned long long *)((char *)Pl->sync_ws + 64);
  P.qcnt = (unsigned long long *)((char *)Pl->sync_ws + 72);
  P.part_bytes = (int)ps::part_bytes(Pl, num_sms());
  P.trace = (unsigned long long *)Pl->trace;
  P.v_embed = Pl->vocab;
  const bool tp = Pl->tp_world > 1;
  if (tp) {
    P.tp_rank = Pl->tp_rank, P.tp_world = Pl->tp_world;
    P.v_embed = Pl->vocab * Pl->tp_world;
    for (int r = 0; r < Pl->tp_world; ++r) P.xchg[r] = (char *)Pl->tp_xchg[r];
    P.h2 = (uint16_t *)Pl->h2;
  }
  cudaError_t e;
  const cudaStream_t cs = (cudaStream_t)stream;
  if (D == 128 && grp == 2)
    e = tp ? ps::launch<4, 2, true>(P, smem, cs) : ps::launch<4, 2, false>(P, smem, cs);
  else if (D == 128 && !tp && I > ps::kMaxPerThread * ps::kCT)
    e = ps::launch<4, 4, false, true>(P, smem, cs);  // the 12288-wide MLP of the 8B shape on one GPU
  else if (D == 128)
    e = tp ? ps::launch<4, 4, true>(P, smem, cs) : ps::launch<4, 4, false>(P, smem, cs);
  else
    e = tp ? ps::launch<1, 2, true>(P, smem, cs) : ps::launch<1, 2, false>(P, smem, cs);
  return check_launch(e, "decode_step_kernel");
}
