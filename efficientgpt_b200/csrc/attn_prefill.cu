// Causal attention over a prompt (prefill) on the 5th-generation tensor cores (tcgen05, sm_100a):
//
//   out[i, h] = softmax(scale * q[i, h] . K[0 .. pos0 + i]) V[0 .. pos0 + i]     for rows i < m
//
// q bf16 [m rows][ldq] (head h at columns h*128 ..), K and V the bf16 cache of one layer, [nkv][cap][128], GQA
// head h reading kv head h / (nq / nkv); out bf16 [m rows][ldo]. head_dim 128.
//
// One CTA per (q head, 128 query rows), the longest query blocks first, 576 threads:
//   warp 0   lane 0 issues TMA loads (this GPU's memory, no multicast): the Q tile once (two 64-column halves,
//            128-byte swizzle), then K blocks of 128 keys into a 3-slot ring and V blocks into a 2-slot ring (a K
//            slot frees once its scores are computed, a V slot once its P.V has run); the K/V tensor maps end at
//            key pos0 + m, so rows past the prompt arrive as zeros (stale cache rows are never read);
//   warp 1   allocates TMEM (two 128-column score buffers S, the 128-column output accumulator O, two 64-column
//            buffers P; lane = query row) and, lane 0, issues tcgen05.mma.kind::f16: S_j = Q K_j^T (both K-major
//            in shared memory) two blocks ahead, and O += P_j V_j with P_j read from TMEM as the A operand and V
//            MN-major straight from its TMA tile;
//   warps 2-17 run the softmax: four warps per TMEM lane quarter (the rows they may read), each taking 32 of a
//            row's 128 columns. Per block: load the thread's 32 scores of S_j, mask keys past the row's position,
//            exchange the partial row maxima within the quarter (shared memory, named barrier), store
//            P_j = bf16(2^(scale log2(e) s - m)) into TMEM (two values per column) and keep a partial sum. The
//            running maximum m moves only when a block's maximum exceeds it by more than 2^8 (then O's columns
//            are rescaled in TMEM, the one step that waits for the previous P.V): probabilities stay below 2^8, and
//            O and the sum use the same m, so the result is the same softmax with fewer rescales. After the last
//            block: bf16(O / sum of the partial sums).
// Rounding: probabilities enter P.V as bf16 (relative to the maximum in use), fp32 accumulation, one bf16 rounding
// of the normalised output (the flash-attention scheme of the SDPA kernels the reference's prefill runs on).
// Every mbarrier wait is bounded (EGPT_ERR_TIMEOUT through egpt_device_error); before the CTA exits the issued TMA
// loads and MMAs are drained (bounded) and TMEM is freed.
#include "internal.h"
#include "common.cuh"

namespace egpt {
namespace apf {

constexpr int kD = 128;                // head dim
constexpr int kBQ = 128;               // query rows per CTA (TMEM lanes)
constexpr int kBK = 128;               // keys per block
constexpr int kHalf = 128 * 128;       // bytes: 128 rows x 64 bf16, one 128-byte swizzle column of a tile
constexpr int kTile = 2 * kHalf;       // 32 KB: 128 rows x 128 bf16
constexpr int kKStages = 3;            // K ring (a slot frees once its scores are computed)
constexpr int kVStages = 2;            // V ring (a slot frees once its P.V has run)
constexpr int kSplit = 4;              // softmax warps per TMEM lane quarter
constexpr int kCols = kBK / kSplit;    // 32 columns of S (and of O) per softmax thread
constexpr int kSmThreads = 128 * kSplit;
constexpr int kThreads = 64 + kSmThreads;  // TMA warp, MMA warp, 16 softmax warps
constexpr float kStale = 8.f;          // the running maximum moves when a block's exceeds it by more (log2 units)
constexpr uint32_t kTmemCols = 512;    // S0 | S1 | O | P0 | P1 (128 + 128 + 128 + 64 + 64 columns)
constexpr uint32_t kOCol = 2 * kBK;
constexpr uint32_t kPCol = 3 * kBK;    // P_j: 128 bf16 per row packed two per column, buffer j % 2
constexpr size_t kRedBytes = 2 * kSplit * kBQ * 4;  // partial row maxima (and sums), two blocks in flight
constexpr size_t kSmem = 1024 /* alignment slack */ + (size_t)kTile /* Q */ +
                         (size_t)(kKStages + kVStages) * kTile /* K, V */ + kRedBytes + 256 /* barriers, TMEM address */;

struct Args {
  CUtensorMap qmap;  // q bf16 [m][ldq], box {64, 128}, 128-byte swizzle
  CUtensorMap kmap;  // K bf16 [nkv][pos0 + m][128] (row stride 256 B, head stride cap rows), box {64, 128, 1}
  CUtensorMap vmap;  // V, same view
  uint16_t *out;
  int64_t ldo, m, pos0;
  int nq, nkv, nqb;
  float scale_log2;  // softmax scale * log2(e)
};

// Instruction descriptors: D fp32, A and B bf16, M 128, N 128; A and B K-major for S = Q K^T, B MN-major
// (transposed) for O = P V.
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescO = kIdescS | (1u << 16);

// MN-major operand [K rows of 128 bytes][two 64-element column groups kHalf bytes apart], 128-byte swizzle:
// leading byte offset = the next 64 columns, stride byte offset = the next 8 K rows.
__device__ __forceinline__ uint64_t sw128_mn_desc(const void *tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr >> 4) & 0x3FFFull) | ((uint64_t)(kHalf >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D (TMEM) += A (TMEM: row i in lane i, K elements packed two per 32-bit column) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t *v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Barrier of the kSplit softmax warps that share a TMEM lane quarter (ids 1-4; 0 is __syncthreads).
__device__ __forceinline__ void quarter_sync(int quarter) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "n"(32 * kSplit) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded wait by every lane of a warp; true only if all of them saw the phase complete (the tcgen05.ld/st that
// follow are warp-collective, so the warp stays together). Measured against one polling lane and a warp barrier:
// 204 vs 214 us per launch at p = 4096.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, unsigned parity) {
  return __all_sync(0xffffffffu, gtc::mbar_wait(bar, parity));
}
// Two fp32 lanes at once (packed f32x2 instructions of sm_100).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__global__ void __launch_bounds__(kThreads, 1) attn_prefill_kernel(const __grid_constant__ Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);  // 1024-aligned operand tiles
  uint8_t *sq = smem;                                 // Q: two [128 rows][128 B] halves
  uint8_t *sk = sq + kTile;                           // K slots, each two [128 keys][128 B] halves
  uint8_t *sv = sk + (size_t)kKStages * kTile;        // V slots, the same layout
  float *red = (float *)(sv + (size_t)kVStages * kTile);  // [2][kSplit][128] partial row maxima / sums
  uint64_t *bars = (uint64_t *)((uint8_t *)red + kRedBytes);
  uint64_t *q_full = bars, *k_full = bars + 1, *k_empty = k_full + kKStages, *v_full = k_empty + kKStages;
  uint64_t *v_empty = v_full + kVStages, *s_full = v_empty + kVStages;
  uint64_t *p_full = s_full + 2, *o_done = p_full + 1, *mma_done = o_done + 1;
  uint32_t *tmem_slot = (uint32_t *)(mma_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int h = (int)(blockIdx.x % (unsigned)A.nq);
  const int qb = A.nqb - 1 - (int)(blockIdx.x / (unsigned)A.nq);  // longest query blocks first
  const int kvh = h / (A.nq / A.nkv);
  const int64_t r0 = (int64_t)qb * kBQ;
  const int64_t rows = min((int64_t)kBQ, A.m - r0);
  const int nkb = (int)((A.pos0 + r0 + rows - 1) / kBK) + 1;  // key blocks any row of the tile sees

  if (threadIdx.x == 0) {
    gtc::mbar_init(q_full, 1);
    for (int s = 0; s < kKStages; ++s) {
      gtc::mbar_init(k_full + s, 1);
      gtc::mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      gtc::mbar_init(v_full + s, 1);
      gtc::mbar_init(v_empty + s, 1);
    }
    gtc::mbar_init(s_full, 1);
    gtc::mbar_init(s_full + 1, 1);
    gtc::mbar_init(p_full, kSmThreads);
    gtc::mbar_init(o_done, 1);
    gtc::mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  gtc::tc_fence_before();
  __syncthreads();
  gtc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      gtc::mbar_arrive_tx(q_full, kTile);
      gtc::tma_load_2d(sq, &A.qmap, h * kD, (int)r0, q_full);
      gtc::tma_load_2d(sq + kHalf, &A.qmap, h * kD + 64, (int)r0, q_full);
      int nk = 0, nv = 0;  // K and V blocks issued; K runs one block ahead of V (scores come first)
      auto load_k = [&](int b) -> bool {
        const int ks = b % kKStages;
        if (b >= kKStages && !gtc::mbar_wait(k_empty + ks, (unsigned)((b / kKStages) - 1) & 1u)) return false;
        uint8_t *k = sk + (size_t)ks * kTile;
        gtc::mbar_arrive_tx(k_full + ks, kTile);
        tma_load_3d(k, &A.kmap, 0, b * kBK, kvh, k_full + ks);
        tma_load_3d(k + kHalf, &A.kmap, 64, b * kBK, kvh, k_full + ks);
        ++nk;
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !load_k(j + 1)) break;
        const int vs = j % kVStages;
        if (j >= kVStages && !gtc::mbar_wait(v_empty + vs, (unsigned)((j / kVStages) - 1) & 1u)) break;
        uint8_t *v = sv + (size_t)vs * kTile;
        gtc::mbar_arrive_tx(v_full + vs, kTile);
        tma_load_3d(v, &A.vmap, 0, j * kBK, kvh, v_full + vs);
        tma_load_3d(v + kHalf, &A.vmap, 64, j * kBK, kvh, v_full + vs);
        ++nv;
      }
      // none of this CTA's copies may still be landing when it exits
      gtc::mbar_drain(q_full, 0);
      for (int b = max(0, nk - kKStages); b < nk; ++b) gtc::mbar_drain(k_full + b % kKStages, (unsigned)(b / kKStages) & 1u);
      for (int b = max(0, nv - kVStages); b < nv; ++b) gtc::mbar_drain(v_full + b % kVStages, (unsigned)(b / kVStages) & 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // S_j = Q K_j^T into score buffer j % 2: eight K = 16 steps, 32 bytes apart inside a 128-byte swizzled row.
      // Its commit also completes once every MMA issued before it has (P.V of block j - 2 included).
      auto issue_scores = [&](int j) -> bool {
        const int s = j % kKStages;
        if (!gtc::mbar_wait(k_full + s, (unsigned)(j / kKStages) & 1u)) return false;
        gtc::tc_fence_after();
        const uint8_t *k = sk + (size_t)s * kTile;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const int half = kk >> 2;
          const uint64_t off = (uint64_t)(2 * (kk & 3));
          umma(tmem + (uint32_t)((j & 1) * kBK), gtc::sw128_desc(sq + half * kHalf) + off,
               gtc::sw128_desc(k + half * kHalf) + off, kIdescS, kk > 0 ? 1u : 0u);
        }
        gtc::umma_commit(k_empty + s);  // the K slot is free once these MMAs have read it
        gtc::umma_commit(s_full + (j & 1));
        return true;
      };
      bool ok = gtc::mbar_wait(q_full, 0) && issue_scores(0) && (nkb < 2 || issue_scores(1));
      for (int j = 0; j < nkb && ok; ++j) {
        const int vs = j % kVStages;
        if (!gtc::mbar_wait(p_full, (unsigned)j & 1u) || !gtc::mbar_wait(v_full + vs, (unsigned)(j / kVStages) & 1u))
          break;
        gtc::tc_fence_after();
        const uint8_t *v = sv + (size_t)vs * kTile;
        const uint32_t pa = tmem + kPCol + (uint32_t)((j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)  // 16 keys per step: 8 columns of P, 16 rows of 128 bytes of V
          umma_ts(tmem + kOCol, pa + (uint32_t)(8 * kk), sw128_mn_desc(v + (size_t)kk * 16 * 128), kIdescO,
                  (j > 0 || kk > 0) ? 1u : 0u);
        gtc::umma_commit(v_empty + vs);  // the V slot is free once these MMAs have read it
        gtc::umma_commit(o_done);
        if (j + 2 < nkb && !issue_scores(j + 2)) break;  // block j + 2's scores overlap the softmax of j + 1
      }
      gtc::umma_commit(mma_done);  // completes once every MMA issued above has finished
      gtc::mbar_drain(mma_done, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax: 32 columns of one row per thread
    // Every warp of a quarter takes every named barrier, whatever its waits returned (a warp whose wait gave up
    // skips its TMEM accesses and arrivals, not the barriers), so no barrier is left waiting.
    const int quarter = warp & 3;         // TMEM lanes this warp may access: 32 (warp % 4) ..
    const int part = (warp - 2) >> 2;    // its column part
    const int row = 32 * quarter + lane;
    const int c0 = part * kCols;
    const int64_t qrow = r0 + row;
    const int64_t qpos = A.pos0 + qrow;                   // the last key this row sees
    const int64_t mask_from = A.pos0 + r0;                // blocks ending past it need the causal mask
    const uint32_t taddr = tmem + ((uint32_t)(32 * quarter) << 16);
    float m_run = -INFINITY, l_part = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      ok = ok && warp_wait(s_full + (j & 1), (unsigned)(j >> 1) & 1u);
      uint32_t sc[kCols];
      float mx = -INFINITY;
      if (ok) {
        gtc::tc_fence_after();
        tmem_ld32(taddr + (uint32_t)((j & 1) * kBK + c0), sc);
        tmem_wait_ld();
        // columns past `lim` are keys after the row's position (lim >= kCols - 1: none)
        const int lim = (int64_t)j * kBK + kBK - 1 > mask_from
                            ? (int)max(min(qpos - ((int64_t)j * kBK + c0), (int64_t)kCols), (int64_t)-1)
                            : kCols;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          float x = __uint_as_float(sc[c]);
          if (c > lim) x = -INFINITY;
          sc[c] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      }
      float *rb = red + (j & 1) * kSplit * kBQ;
      rb[part * kBQ + row] = mx;
      quarter_sync(quarter);
      float bm = rb[row];
#pragma unroll
      for (int q = 1; q < kSplit; ++q) bm = fmaxf(bm, rb[q * kBQ + row]);
      bm *= A.scale_log2;  // the row's block maximum in log2 units (scale > 0)
      float alpha = 1.f;
      if (bm > m_run + kStale) {  // the same decision in every thread of the row: same partials, same order
        alpha = ex2(m_run - bm);  // 0 on the first block (m_run = -inf)
        m_run = bm;
      }
      // p = 2^(s scale log2(e) - m): the exponent argument two at a time, sums in two fp32 lanes
      const uint64_t sc2 = f2_pack(A.scale_log2, A.scale_log2), nm2 = f2_pack(-m_run, -m_run);
      uint64_t sum2 = f2_pack(0.f, 0.f);
      uint32_t pk[kCols / 2];
#pragma unroll
      for (int c = 0; c < kCols; c += 2) {
        const float2 e = f2_unpack(f2_fma(f2_pack(__uint_as_float(sc[c]), __uint_as_float(sc[c + 1])), sc2, nm2));
        const float p0 = ex2(e.x), p1 = ex2(e.y);
        sum2 = f2_add(sum2, f2_pack(p0, p1));
        pk[c / 2] = gtc::pack_bf16x2(p0, p1);
      }
      const float2 sum = f2_unpack(sum2);
      l_part = l_part * alpha + (sum.x + sum.y);
      if (ok && j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // rescale O once the previous P.V has finished (O then holds every block before this one)
        ok = warp_wait(o_done, (unsigned)(j - 1) & 1u);
        if (ok) {
          gtc::tc_fence_after();
          uint32_t o[kCols];
          tmem_ld32(taddr + kOCol + (uint32_t)c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < kCols; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(taddr + kOCol + (uint32_t)c0, o);
          tmem_wait_st();
        }
      }
      if (ok) {
        // P_j, keys c0 .. c0 + 31 of the row as 16 packed columns, into TMEM buffer j % 2: the P.V of block j - 2
        // has finished reading it (S_j's commit completes after that MMA)
        tmem_st16(taddr + kPCol + (uint32_t)((j & 1) * 64 + c0 / 2), pk);
        tmem_wait_st();
        gtc::tc_fence_before();
        gtc::mbar_arrive(p_full);
      }
    }
    // the row's sum: the parts in a fixed order (the buffer the last block did not use is free)
    float *rb = red + (nkb & 1) * kSplit * kBQ;
    rb[part * kBQ + row] = l_part;
    quarter_sync(quarter);
    float l = 0.f;
#pragma unroll
    for (int q = 0; q < kSplit; ++q) l += rb[q * kBQ + row];
    if (ok && warp_wait(o_done, (unsigned)(nkb - 1) & 1u)) {
      gtc::tc_fence_after();
      const float inv = 1.f / l;
      uint32_t o[kCols];
      tmem_ld32(taddr + kOCol + (uint32_t)c0, o);
      tmem_wait_ld();
      uint32_t w[kCols / 2];
#pragma unroll
      for (int e = 0; e < kCols / 2; ++e)
        w[e] = (uint32_t)f32_to_bf16_bits(__uint_as_float(o[2 * e]) * inv) |
               ((uint32_t)f32_to_bf16_bits(__uint_as_float(o[2 * e + 1]) * inv) << 16);
      if (qrow < A.m) {
        uint16_t *dst = A.out + qrow * A.ldo + (int64_t)h * kD + c0;
#pragma unroll
        for (int e = 0; e < kCols / 8; ++e) ((uint4 *)dst)[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
      }
    }
  }
  gtc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    gtc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace apf
}  // namespace egpt

using namespace egpt;

extern "C" int egpt_attn_prefill(void *out, int64_t ldo, const void *q, int64_t ldq, const void *k_cache,
                                 const void *v_cache, int64_t cap, int64_t pos0, int64_t m, int nq, int nkv, int d,
                                 float scale, void *stream) {
  clear_error();
  if (!out || !q || !k_cache || !v_cache) return set_error(EGPT_ERR_ARG, "attn_prefill: null pointer");
  if (d != apf::kD) return set_error(EGPT_ERR_SHAPE, "attn_prefill: head_dim must be 128");
  if (m < 1 || pos0 < 0 || nq < 1 || nkv < 1 || nq % nkv || cap < pos0 + m || cap > ((int64_t)1 << 31) ||
      m > ((int64_t)1 << 31) || ldq < (int64_t)nq * d || ldo < (int64_t)nq * d ||
      (int64_t)nq * ((m + apf::kBQ - 1) / apf::kBQ) > ((int64_t)1 << 31) - 1)
    return set_error(EGPT_ERR_SHAPE, "attn_prefill: bad shape (nq a multiple of nkv, pos0 + m <= cap)");
  if (!(scale > 0.f)) return set_error(EGPT_ERR_ARG, "attn_prefill: scale must be positive");
  if ((uintptr_t)out % 16 || (uintptr_t)q % 16 || (uintptr_t)k_cache % 16 || (uintptr_t)v_cache % 16 || ldq % 8 ||
      ldo % 8)
    return set_error(EGPT_ERR_ALIGN, "attn_prefill: pointers 16-byte aligned, leading dimensions multiples of 8");
  auto fn = df::encode_fn();
  if (!fn) return set_error(EGPT_ERR_LAUNCH, "attn_prefill: this driver does not encode tensor maps");
  apf::Args A{};
  const cuuint32_t es2[2] = {1, 1}, es3[3] = {1, 1, 1};
  const cuuint64_t qdims[2] = {(cuuint64_t)nq * d, (cuuint64_t)m};
  const cuuint64_t qstrides[1] = {(cuuint64_t)ldq * 2};
  const cuuint32_t qbox[2] = {64, apf::kBQ};
  if (fn(&A.qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(q), qdims, qstrides, qbox, es2,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return set_error(EGPT_ERR_ALIGN, "attn_prefill: tensor map of q rejected");
  // keys past pos0 + m lie outside the map: TMA fills them with zeros
  const cuuint64_t kdims[3] = {(cuuint64_t)d, (cuuint64_t)(pos0 + m), (cuuint64_t)nkv};
  const cuuint64_t kstrides[2] = {(cuuint64_t)d * 2, (cuuint64_t)cap * d * 2};
  const cuuint32_t kbox[3] = {64, apf::kBK, 1};
  if (fn(&A.kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(k_cache), kdims, kstrides, kbox, es3,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      fn(&A.vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(v_cache), kdims, kstrides, kbox, es3,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return set_error(EGPT_ERR_ALIGN, "attn_prefill: tensor map of the cache rejected");
  A.out = (uint16_t *)out, A.ldo = ldo, A.m = m, A.pos0 = pos0, A.nq = nq, A.nkv = nkv;
  A.nqb = (int)((m + apf::kBQ - 1) / apf::kBQ);
  A.scale_log2 = scale * 1.4426950408889634f;
  static int configured[64] = {0};  // the shared-memory opt-in, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(apf::attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)apf::kSmem);
    if (e != cudaSuccess) return check_launch(e, "attn_prefill (shared memory attribute)");
    configured[dev] = 1;
  }
  const unsigned grid = (unsigned)((int64_t)nq * A.nqb);
  apf::attn_prefill_kernel<<<grid, apf::kThreads, apf::kSmem, (cudaStream_t)stream>>>(A);
  return check_launch(cudaGetLastError(), "attn_prefill_kernel");
}
