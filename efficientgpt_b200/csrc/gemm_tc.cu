// int8-weight GEMM for long-prompt prefill on the 5th-generation tensor cores (tcgen05, sm_100a):
//
//   Y[m, n] = bf16( bf16( sum_k X[m, k] * bf16(Q[n, k]) ) * s[n] )        (double rounding: the reference's
//                                                                          >16-row branch, int8_linear.py:96-97)
//   or, without EGPT_FLAG_DOUBLE_ROUND, bf16(fp32 sum * s[n]).
//
// X bf16 [M, K] (row stride ldx), Q int8 [N, K] (row-major, the model's own buffer), s bf16 or fp32 [N]. The
// reference materialises bf16(Q) in HBM on every call; here the int8 rows are converted to bf16 in shared memory
// on their way to the tensor cores, so HBM sees the int8 bytes once per output tile column.
//
// One CTA per 128 x 256 output tile, 320 threads:
//   warp 0   lane 0 issues the TMA loads of X (box 64 columns x 128 rows, 128-byte swizzle) and of the int8 Q tile
//            (box 64 columns x 256 rows, 64-byte swizzle), this GPU's memory, no multicast, into a ring of kStages
//            slots;
//   warp 1   allocates 256 TMEM columns (the fp32 accumulator, lane = row) and, lane 0, issues
//            tcgen05.mma.cta_group::1.kind::f16 (M 128, N 256, K 16; both operands bf16, K-major, 128-byte
//            swizzled shared-memory descriptors), four per 64-column k block, then tcgen05.commit to the slot's
//            "empty" barrier and, after the last block, to the accumulator barrier;
//   warps 2-9 convert Q: each thread reads one row's 64 int8 of the k block from the slot (the 64-byte swizzle
//            makes the 16-byte reads of 8 consecutive rows hit 32 distinct banks), widens them to bf16 (exact:
//            |q| <= 127) and stores them in the operand's swizzled layout (row r at 128 r bytes, 16-byte chunk c at
//            (c ^ (r & 7)) * 16), then fence.proxy.async and an arrival on the slot's "B full" barrier; the slot is
//            reused once the MMAs that read it have committed; after the last block the same warps read the accumulator
//            with tcgen05.ld (warp w owns TMEM lanes 32 (w % 4) .., two warps per lane quarter split the columns),
//            scale, round and store Y. The widening needs no int-to-float conversion (byte_val).
// Every mbarrier wait is bounded (EGPT_ERR_TIMEOUT through egpt_device_error); a role that gives up skips its
// remaining work, and before the CTA exits the issued TMA loads and MMAs are drained (bounded) and TMEM is freed.
#include "internal.h"
#include "common.cuh"

namespace egpt {
namespace gtc {

constexpr int kBM = 128, kBN = 256, kBK = 64;  // output tile and k block (64 bf16 = one 128-byte swizzle row)
constexpr int kStages = 5;   // TMA ring: X and int8 Q tiles (latency cover)
constexpr int kBStages = 2;  // widened Q tiles between the converters and the MMAs
constexpr int kEpiWarps = 4;          // warps 10-13
constexpr int kThreads = 320 + 32 * kEpiWarps;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB: X tile, bf16
constexpr int kRBytes = kBN * kBK;      // 16 KB: Q tile as loaded, int8
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB: Q tile widened to bf16
constexpr int kConvThreads = 256;       // warps 2-9: one Q row each
constexpr size_t kSmem = 1024 /* alignment slack */ + (size_t)kStages * (kABytes + kRBytes) + (size_t)kBStages * kBBytes + 256;
static_assert(kThreads == 448, "roles: TMA, MMA, 8 widening warps, 4 epilogue warps");

struct Args {
  CUtensorMap xmap;  // X bf16 [M, K], box {64, 128}, 128-byte swizzle
  CUtensorMap qmap;  // Q int8 [N, K], box {64, 256}, 64-byte swizzle
  const int8_t *q;
  const void *s;
  int s_bf16;
  uint16_t *y;
  int64_t M, N, K, ldy;
  int double_round;
  int add_out;    // y holds the residual on entry: y = bf16(y + result)
  int ksplit;     // k ranges per output tile (work unit = tile x range); > 1: fp32 partials into ws, then reduce
  float *ws;      // [ksplit][M][N] fp32 partial sums (ksplit > 1)
};

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok)
               : "r"(smem_u32(bar)), "r"(parity)
               : "memory");
  return ok != 0;
}
// Bounded wait; false after a timeout or once another wait of the grid has reported an error.
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
// Bounded by time only (whatever the error state): used to drain work in flight before the CTA exits.
__device__ void mbar_drain(uint64_t *bar, unsigned parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(EGPT_ERR_TIMEOUT);
      return;
    }
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile whose rows are 128 bytes, 8-row groups 1024 bytes
// apart, 128-byte swizzle (start address 1024-aligned; the k offset inside the row is added to the start field).
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr >> 4) & 0x3FFFull)          // start address
         | (1ull << 16)                     // leading byte offset (unused with swizzling): 16 bytes
         | ((uint64_t)(1024 >> 4) << 32)    // stride byte offset: 8 rows x 128 bytes
         | (1ull << 46)                     // descriptor version (sm100)
         | (2ull << 61);                    // 128-byte swizzle
}
// Instruction descriptor: D fp32, A and B bf16, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Two fp32 values (exact integers) -> packed bf16x2, a in the low half (exact).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// Byte i of w (already XORed with 0x80: v + 128 as an unsigned byte) as the fp32 value v, without an int-to-float
// conversion: the bits 0x4B0000uu are the float 2^23 + uu, and subtracting 2^23 + 128 leaves v exactly.
__device__ __forceinline__ float byte_val(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + (uint32_t)i)) - 8388736.0f;
}
// 16 int8 (a uint4) -> 16 bf16 (two uint4), element order kept.
__device__ __forceinline__ void widen16(const uint4 v, uint4 &lo, uint4 &hi) {
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = pack_bf16x2(byte_val(w[i], 0), byte_val(w[i], 1));
    o[2 * i + 1] = pack_bf16x2(byte_val(w[i], 2), byte_val(w[i], 3));
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ void tile_of(const Args &A, int64_t t, int64_t mt, int64_t &m0, int64_t &n0) {
  // consecutive tiles share a weight tile (one N column of tiles, all M tiles): the CTAs running together read
  // each weight tile once from HBM and the x tiles from L2
  n0 = (t / mt) * kBN;
  m0 = (t % mt) * kBM;
}

__global__ void __launch_bounds__(kThreads, 1) gemm_i8_tc_kernel(const __grid_constant__ Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);  // 1024-aligned operand tiles
  uint8_t *sa = smem;                                      // kStages x [128 rows][128 B], bf16, 128-byte swizzle
  uint8_t *sb = smem + (size_t)kStages * kABytes;          // kBStages x [256 rows][128 B], bf16, 128-byte swizzle
  uint8_t *sr = sb + (size_t)kBStages * kBBytes;           // kStages x [256 rows][64 B], int8, 64-byte swizzle
  uint64_t *bars = (uint64_t *)(sr + (size_t)kStages * kRBytes);
  uint64_t *full_a = bars, *empty = bars + kStages;                    // TMA ring
  uint64_t *full_b = bars + 2 * kStages, *bempty = full_b + kBStages;  // widened-Q ring
  uint64_t *acc_full = bempty + kBStages, *acc_empty = acc_full + 2;   // two TMEM accumulators
  uint32_t *tmem_slot = (uint32_t *)(acc_empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (int)(A.K / kBK);
  const int64_t mt = (A.M + kBM - 1) / kBM, tiles = mt * ((A.N + kBN - 1) / kBN);
  const int S = A.ksplit;
  const int64_t units = tiles * S;
  // work unit u: tile u / S, k blocks [kb_lo(u), kb_lo(u) + kb_n(u))
  auto kb_lo = [&](int64_t u) { return (int)((int64_t)(u % S) * nkb / S); };
  auto kb_n = [&](int64_t u) { return (int)((int64_t)(u % S + 1) * nkb / S) - kb_lo(u); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_a + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(full_b + s, kConvThreads);
      mbar_init(bempty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(acc_full + s, 1);
      mbar_init(acc_empty + s, kEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: two accumulators of 256 fp32 columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer: X and int8 Q tiles
    if (lane == 0) {
      int64_t kg = 0;  // k blocks issued by this CTA over all its tiles
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int64_t m0, n0;
        tile_of(A, u / S, mt, m0, n0);
        for (int kb = kb_lo(u), ke = kb_lo(u) + kb_n(u); kb < ke; ++kb, ++kg) {
          const int s = (int)(kg % kStages);
          if (kg >= kStages && !mbar_wait(empty + s, (unsigned)((kg / kStages) - 1) & 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_tx(full_a + s, kABytes + kRBytes);
          tma_load_2d(sa + (size_t)s * kABytes, &A.xmap, kb * kBK, (int)m0, full_a + s);
          tma_load_2d(sr + (size_t)s * kRBytes, &A.qmap, kb * kBK, (int)n0, full_a + s);
        }
      }
      // none of this CTA's copies may still be landing when it exits
      for (int64_t k = max((int64_t)0, kg - kStages); k < kg; ++k)
        mbar_drain(full_a + k % kStages, (unsigned)(k / kStages) & 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int64_t kg = 0, i = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
        const int buf = (int)(i & 1);
        if (i >= 2 && !mbar_wait(acc_empty + buf, (unsigned)((i >> 1) - 1) & 1u)) break;  // epilogue drained it
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * kBN);
        const int kb0 = kb_lo(u);
        for (int kb = kb0, ke = kb0 + kb_n(u); kb < ke; ++kb, ++kg) {
          const int s = (int)(kg % kStages), sbi = (int)(kg % kBStages);
          if (!mbar_wait(full_a + s, (unsigned)(kg / kStages) & 1u) ||
              !mbar_wait(full_b + sbi, (unsigned)(kg / kBStages) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(sa + (size_t)s * kABytes), bd = sw128_desc(sb + (size_t)sbi * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // 16 bf16 = 32 bytes per step inside the swizzled row
            umma_f16(acc, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), (kb != kb0 || k != 0) ? 1u : 0u);
          umma_commit(empty + s);     // the TMA slot is free once these MMAs have read it
          umma_commit(bempty + sbi);  // and so is the widened-Q slot
        }
        umma_commit(acc_full + buf);  // completes when every MMA issued above has finished
      }
    }
  } else if (warp < 2 + kConvThreads / 32) {
    // ---------------------------------------------------------------- Q converters
    const int r = threadIdx.x - 64;  // the Q row (of the 256-row tile) this thread widens
    int64_t kg = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      for (int kb = 0, ke = kb_n(u); kb < ke; ++kb, ++kg) {
        const int s = (int)(kg % kStages), sbi = (int)(kg % kBStages);
        if (!mbar_wait(full_a + s, (unsigned)(kg / kStages) & 1u) ||
            (kg >= kBStages && !mbar_wait(bempty + sbi, (unsigned)((kg / kBStages) - 1) & 1u))) {
          ok = false;
          break;
        }
        const uint8_t *rrow = sr + (size_t)s * kRBytes + (size_t)r * 64;  // chunk c at (c ^ ((r >> 1) & 3)) * 16
        uint8_t *row = sb + (size_t)sbi * kBBytes + (size_t)r * 128;
        uint4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = *(const uint4 *)(rrow + ((c ^ ((r >> 1) & 3)) << 4));
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 16 int8 -> chunks 2c, 2c + 1 (8 bf16 each) of the 128-byte swizzle
          uint4 lo, hi;
          widen16(v[c], lo, hi);
          *(uint4 *)(row + (((2 * c) ^ (r & 7)) << 4)) = lo;
          *(uint4 *)(row + (((2 * c + 1) ^ (r & 7)) << 4)) = hi;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> the tensor cores' reads
        mbar_arrive(full_b + sbi);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue: TMEM -> scale -> bf16 -> Y
    const int quarter = warp & 3;  // TMEM lanes a warp may access: 32 (warp % 4) ..
    int64_t i = 0;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x, ++i) {
      const int buf = (int)(i & 1);
      if (!mbar_wait(acc_full + buf, (unsigned)(i >> 1) & 1u)) break;
      tc_fence_after();
      int64_t m0, n0;
      tile_of(A, u / S, mt, m0, n0);
      const int64_t m = m0 + 32 * quarter + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(buf * kBN + c0);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
              "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
              "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (S > 1) {  // k range partial: the raw fp32 sums, reduced (and scaled) by gemm_reduce_kernel
          if (m < A.M) {
            float *dst = A.ws + ((int64_t)(u % S) * A.M + m) * A.N + n0 + c0;
            if (n0 + c0 + 32 <= A.N) {
#pragma unroll
              for (int j = 0; j < 8; ++j) ((uint4 *)dst)[j] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
              for (int j = 0; j < 32 && n0 + c0 + j < A.N; ++j) dst[j] = __uint_as_float(v[j]);
            }
          }
        } else if (m < A.M) {
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float y2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int64_t n = n0 + c0 + j + e;
              float acc_v = __uint_as_float(v[j + e]);
              if (A.double_round) acc_v = round_bf16(acc_v);
              const float sc = n < A.N ? (A.s_bf16 ? bf16_bits_to_f32(((const uint16_t *)A.s)[n]) : ((const float *)A.s)[n])
                                       : 0.f;
              y2[e] = acc_v * sc;
            }
            packed[j / 2] = (uint32_t)f32_to_bf16_bits(y2[0]) | ((uint32_t)f32_to_bf16_bits(y2[1]) << 16);
          }
          uint16_t *dst = A.y + m * A.ldy + n0 + c0;
          if (A.add_out) {  // y = bf16(residual + bf16(result)), the residual read from y itself
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int64_t n = n0 + c0 + 2 * j;
              const uint32_t r = n + 1 < A.N ? *(const uint32_t *)(dst + 2 * j) : (n < A.N ? (uint32_t)dst[2 * j] : 0u);
              packed[j] = (uint32_t)f32_to_bf16_bits(bf16_lo(r) + bf16_lo(packed[j])) |
                          ((uint32_t)f32_to_bf16_bits(bf16_hi(r) + bf16_hi(packed[j])) << 16);
            }
          }
          if (n0 + c0 + 32 <= A.N) {
#pragma unroll
            for (int j = 0; j < 4; ++j) ((uint4 *)dst)[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
          } else {
            for (int j = 0; j < 32 && n0 + c0 + j < A.N; ++j) dst[j] = (uint16_t)(packed[j / 2] >> (16 * (j & 1)));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + buf);  // the MMAs of tile i + 2 may overwrite this accumulator
    }
  }
  // every MMA this CTA issued has completed before TMEM is freed: the epilogue waited for each accumulator it
  // read; on an early stop, wait here (bounded) for the last commit of each buffer that was used
  if (warp == 1 && lane == 0) {
    int64_t used = 0;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) ++used;
    for (int64_t i = max((int64_t)0, used - 2); i < used; ++i) mbar_drain(acc_full + (i & 1), (unsigned)(i >> 1) & 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kBN) : "memory");
  }
}

// y[m, n] = bf16(bf16(sum_s ws[s][m][n]) * s[n]) (double rounding) or bf16(sum * s[n]); the k ranges in order.
__global__ void __launch_bounds__(256) gemm_reduce_kernel(const __grid_constant__ Args A) {
  const int64_t pairs = A.M * (A.N / 2);
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * 256) {
    const int64_t m = i / (A.N / 2), n = 2 * (i - m * (A.N / 2));
    float acc0 = 0.f, acc1 = 0.f;
    for (int s = 0; s < A.ksplit; ++s) {
      const float2 v = *(const float2 *)(A.ws + ((int64_t)s * A.M + m) * A.N + n);
      acc0 += v.x;
      acc1 += v.y;
    }
    if (A.double_round) acc0 = round_bf16(acc0), acc1 = round_bf16(acc1);
    const float s0 = A.s_bf16 ? bf16_bits_to_f32(((const uint16_t *)A.s)[n]) : ((const float *)A.s)[n];
    const float s1 = A.s_bf16 ? bf16_bits_to_f32(((const uint16_t *)A.s)[n + 1]) : ((const float *)A.s)[n + 1];
    uint32_t *dst = (uint32_t *)(A.y + m * A.ldy + n);
    float y0 = acc0 * s0, y1 = acc1 * s1;
    if (A.add_out) {  // y = bf16(residual + bf16(result)), the residual read from y itself
      const uint32_t r = *dst;
      y0 = bf16_lo(r) + round_bf16(y0), y1 = bf16_hi(r) + round_bf16(y1);
    }
    *dst = (uint32_t)f32_to_bf16_bits(y0) | ((uint32_t)f32_to_bf16_bits(y1) << 16);
  }
}

// k ranges per tile so that the work units fill about one wave of the GPU, each range at least 4 k blocks.
inline int choose_ksplit(int64_t M, int64_t N, int64_t K, int sms) {
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int64_t nkb = K / kBK;
  int64_t s = (sms + tiles - 1) / tiles;
  s = std::min<int64_t>(s, std::max<int64_t>(1, nkb / 4));
  return (int)std::max<int64_t>(1, std::min<int64_t>(s, 16));
}

}  // namespace gtc
}  // namespace egpt

using namespace egpt;

extern "C" size_t egpt_gemm_i8_tc_ws_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < gtc::kBK) return 0;
  const int S = gtc::choose_ksplit(M, N, K, num_sms());
  return S > 1 ? (size_t)S * M * N * 4 : 0;
}

extern "C" int egpt_gemm_i8_tc(void *y, int64_t ldy, const void *x, int64_t ldx, int64_t M, const int8_t *q,
                               const void *s, int s_dtype, int64_t N, int64_t K, unsigned flags, void *ws,
                               size_t ws_bytes, void *stream) {
  clear_error();
  if (!y || !x || !q || !s) return set_error(EGPT_ERR_ARG, "gemm_i8_tc: null pointer");
  if (s_dtype != EGPT_BF16 && s_dtype != EGPT_F32) return set_error(EGPT_ERR_DTYPE, "gemm_i8_tc: scale dtype");
  if (M < 1 || N < 1 || K < gtc::kBK || K % gtc::kBK || ldx < K || ldy < N || M > ((int64_t)1 << 31) ||
      N > ((int64_t)1 << 30) || K > ((int64_t)1 << 20))
    return set_error(EGPT_ERR_SHAPE, "gemm_i8_tc: bad shape (K a multiple of 64)");
  if ((uintptr_t)x % 16 || (uintptr_t)y % 16 || (uintptr_t)q % 16 || ldx % 8 || ldy % 8)
    return set_error(EGPT_ERR_ALIGN, "gemm_i8_tc: x, y, q 16-byte aligned and leading dimensions multiples of 8");
  auto fn = df::encode_fn();
  if (!fn) return set_error(EGPT_ERR_LAUNCH, "gemm_i8_tc: this driver does not encode tensor maps");
  gtc::Args A{};
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t box[2] = {gtc::kBK, gtc::kBM}, es[2] = {1, 1};
  if (fn(&A.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return set_error(EGPT_ERR_ALIGN, "gemm_i8_tc: tensor map of x rejected");
  const cuuint64_t qdims[2] = {(cuuint64_t)K, (cuuint64_t)N};
  const cuuint64_t qstrides[1] = {(cuuint64_t)K};
  const cuuint32_t qbox[2] = {gtc::kBK, gtc::kBN};
  if (fn(&A.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(q), qdims, qstrides, qbox, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return set_error(EGPT_ERR_ALIGN, "gemm_i8_tc: tensor map of q rejected");
  A.q = q, A.s = s, A.s_bf16 = s_dtype == EGPT_BF16, A.y = (uint16_t *)y;
  A.M = M, A.N = N, A.K = K, A.ldy = ldy, A.double_round = (flags & EGPT_FLAG_DOUBLE_ROUND) ? 1 : 0;
  A.add_out = (flags & EGPT_FLAG_ADD_OUT) ? 1 : 0;
  // split K over several CTAs per output tile when the tiles alone leave SMs idle (few rows: decode batches,
  // short prompts), given the workspace for the fp32 partials; else one range per tile
  A.ksplit = 1;
  const int S = gtc::choose_ksplit(M, N, K, num_sms());
  if (S > 1 && ws && ws_bytes >= (size_t)S * M * N * 4 && (uintptr_t)ws % 16 == 0 && N % 2 == 0)
    A.ksplit = S, A.ws = (float *)ws;
  static int configured[64] = {0};  // the shared-memory opt-in, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(gtc::gemm_i8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)gtc::kSmem);
    if (e != cudaSuccess) return check_launch(e, "gemm_i8_tc (shared memory attribute)");
    configured[dev] = 1;
  }
  const int64_t units = ((N + gtc::kBN - 1) / gtc::kBN) * ((M + gtc::kBM - 1) / gtc::kBM) * A.ksplit;
  const unsigned grid = (unsigned)std::min<int64_t>(units, (int64_t)num_sms());  // persistent: one CTA per SM
  gtc::gemm_i8_tc_kernel<<<grid, gtc::kThreads, gtc::kSmem, (cudaStream_t)stream>>>(A);
  int rc = check_launch(cudaGetLastError(), "gemm_i8_tc_kernel");
  if (rc != EGPT_OK || A.ksplit == 1) return rc;
  const int64_t pairs = M * (N / 2);
  const unsigned rgrid = (unsigned)std::min<int64_t>((pairs + 255) / 256, (int64_t)num_sms() * 8);
  gtc::gemm_reduce_kernel<<<rgrid, 256, 0, (cudaStream_t)stream>>>(A);
  return check_launch(cudaGetLastError(), "gemm_reduce_kernel");
}
