// Split-K decode attention for one query row over a long bf16 cache, streamed through shared memory with bulk
// copies (sm_100a): egpt_attn_decode's kernel for m = 1, bf16, head_dim 128, without EGPT_FLAG_APPEND,
// EGPT_FLAG_RAGGED or EGPT_FLAG_REF_SOFTMAX (the other cases run attn_split_kernel of attention.cu).
//
//   out[h] = softmax(scale q_h . K[0 .. L)) V[0 .. L),  L = *position + 1, q head h reading kv head h / GRP.
//
// Grid (nkv, ranges): a CTA owns one kv head, its GRP q heads and one range of whole 128-key blocks (ranges sized
// from L on the device, so a captured graph follows the position). A kv head's K rows (and V rows) are one
// contiguous stream, so a block of 128 keys is one 32 KB bulk copy (cp.async.bulk, this GPU's memory, no
// multicast): warp 8 keeps K and V blocks in flight through a 3-stage ring (192 KB), completion by transaction
// count on the stage's mbarrier; two stages load while the eight compute warps work on the third. Warp w takes
// keys 16 w .. 16 w + 15 of every block: lanes l and l + 16 score key l over the two halves of the row for every q
// head (16-byte pieces rotated by the key so that a shared-memory phase reads different bank groups; q from
// shared memory), the warp keeps its own running maximum, sum and P.V accumulator per q head (lane l: dims
// 4l .. 4l + 3; probabilities enter P.V rounded to bf16, the sums use the fp32 values), and releases the stage.
// The warps merge in a fixed order; one range writes the output, several write partials (maximum, sum,
// unnormalised output, base-2 exponents) and the last range of the kv head to arrive combines them. Every wait
// is bounded (EGPT_ERR_TIMEOUT); the producer drains its copies before the CTA exits.
#include "internal.h"
#include "common.cuh"

namespace egpt {
namespace ast {

constexpr int kD = 128;
constexpr int kBlock = 128;                 // keys per bulk copy (one softmax block of the reference kernel)
constexpr int kStages = 3;
constexpr int kRowBytes = kD * 2;           // bf16 row: 256 bytes
constexpr int kBlockBytes = kBlock * kRowBytes;
constexpr int kWarps = 8;                   // compute warps, 16 keys of every block each
constexpr int kThreads = (kWarps + 1) * 32; // + the copy warp

template <int GRP>
struct Smem {
  uint8_t ring[kStages][2][kBlockBytes];  // [stage][K | V][128 rows of 256 bytes]
  float q[GRP][kD];                       // q heads, pre-scaled by scale log2(e)
  float w_m[kWarps][GRP], w_l[kWarps][GRP];
  float w_acc[kWarps][GRP][kD];
  uint64_t full[kStages], empty[kStages];
  int flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Ranges of whole blocks per kv head: at most `cap` of them (the launch's grid), each `bps` blocks but the last.
__device__ __forceinline__ void range_of(int64_t L, int cap, int split, int64_t &k0, int64_t &k1, int &nsplit) {
  const int64_t nb = (L + kBlock - 1) / kBlock;
  const int64_t bps = (nb + cap - 1) / cap;
  nsplit = (int)((nb + bps - 1) / bps);
  k0 = (int64_t)split * bps * kBlock;
  k1 = min(L, k0 + bps * kBlock);
}

template <int GRP>
__global__ void __launch_bounds__(kThreads, 1) attn_stream_kernel(AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem<GRP> &S = *(Smem<GRP> *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, split = blockIdx.y;
  const int64_t pos = *p.position;
  const int64_t L = pos + 1;
  if (L > p.cap || pos < 0) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return;
  }
  int64_t k0, k1;
  int nsplit;
  range_of(L, p.split_cap, split, k0, k1, nsplit);
  if (split >= nsplit) return;
  const int nblk = (int)((k1 - k0 + kBlock - 1) / kBlock);
  const uint8_t *Kg = (const uint8_t *)p.k_cache + ((int64_t)g * p.cap + k0) * kRowBytes;
  const uint8_t *Vg = (const uint8_t *)p.v_cache + ((int64_t)g * p.cap + k0) * kRowBytes;
  const float sl2 = p.scale * 1.4426950408889634f;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      gtc::mbar_init(S.full + s, 1);
      gtc::mbar_init(S.empty + s, kWarps);  // every compute warp releases every block
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < GRP * kD; i += kThreads) {
    const int j = i / kD, d = i - j * kD;
    S.q[j][d] = bf16_bits_to_f32(((const uint16_t *)p.q)[(int64_t)(g * GRP + j) * kD + d]) * sl2;
  }
  __syncthreads();

  if (warp == kWarps) {
    // ---------------------------------------------------------------- copy warp
    if (lane == 0) {
      int issued = 0;
      for (int b = 0; b < nblk; ++b) {
        const int s = b % kStages;
        if (b >= kStages && !gtc::mbar_wait(S.empty + s, (unsigned)((b / kStages) - 1) & 1u)) break;
        const unsigned bytes = (unsigned)(min((int64_t)kBlock, k1 - k0 - (int64_t)b * kBlock) * kRowBytes);
        gtc::mbar_arrive_tx(S.full + s, 2 * bytes);
        df::bulk_copy(S.ring[s][0], Kg + (int64_t)b * kBlockBytes, bytes, S.full + s);
        df::bulk_copy(S.ring[s][1], Vg + (int64_t)b * kBlockBytes, bytes, S.full + s);
        ++issued;
      }
      for (int b = max(0, issued - kStages); b < issued; ++b)  // nothing may still be landing at exit
        gtc::mbar_drain(S.full + b % kStages, (unsigned)(b / kStages) & 1u);
    }
  } else {
    // ---------------------------------------------------------------- compute warps
    // every block: warp w takes keys 16 w .. 16 w + 15; lane l scores key l % 16 over dims 64 (l / 16) .. + 63
    const int slice = 16 * warp, kl = lane & 15, half = lane >> 4;
    float m_run[GRP], l_run[GRP], acc[GRP][4];
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      m_run[j] = -INFINITY;
      l_run[j] = 0.f;
      acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    }
    for (int b = 0; b < nblk; ++b) {
      const int s = b % kStages;
      if (!__all_sync(0xffffffffu, gtc::mbar_wait(S.full + s, (unsigned)(b / kStages) & 1u))) break;
      const int nvalid = (int)min((int64_t)16, k1 - k0 - (int64_t)b * kBlock - slice);  // keys of this slice
      if (nvalid > 0) {
        const uint8_t *Ks = S.ring[s][0] + (size_t)slice * kRowBytes;
        const uint8_t *Vs = S.ring[s][1] + (size_t)slice * kRowBytes;
        // scores (base-2 exponent units): half a row per lane, 16-byte pieces rotated by the key so that the
        // lanes of a shared-memory phase read different bank groups
        float a[GRP][2];
#pragma unroll
        for (int j = 0; j < GRP; ++j) a[j][0] = a[j][1] = 0.f;
        if (kl < nvalid) {
          const uint4 *row = (const uint4 *)(Ks + (size_t)kl * kRowBytes);
          const int rot = kl & 7;
#pragma unroll 4
          for (int u = 0; u < 8; ++u) {
            const int pc = 8 * half + ((u + rot) & 7);
            const uint4 w = row[pc];
            const float kv[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                                 bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
#pragma unroll
            for (int j = 0; j < GRP; ++j) {
              const float4 q0 = *(const float4 *)&S.q[j][8 * pc], q1 = *(const float4 *)&S.q[j][8 * pc + 4];
              a[j][0] = fmaf(q0.x, kv[0], a[j][0]);
              a[j][1] = fmaf(q0.y, kv[1], a[j][1]);
              a[j][0] = fmaf(q0.z, kv[2], a[j][0]);
              a[j][1] = fmaf(q0.w, kv[3], a[j][1]);
              a[j][0] = fmaf(q1.x, kv[4], a[j][0]);
              a[j][1] = fmaf(q1.y, kv[5], a[j][1]);
              a[j][0] = fmaf(q1.z, kv[6], a[j][0]);
              a[j][1] = fmaf(q1.w, kv[7], a[j][1]);
            }
          }
        }
        float pr[GRP];
#pragma unroll
        for (int j = 0; j < GRP; ++j) {
          const float part = a[j][0] + a[j][1];
          const float sc = part + __shfl_xor_sync(0xffffffffu, part, 16);  // both halves of the row
          const float x = kl < nvalid ? sc : -INFINITY;
          const float m_new = fmaxf(m_run[j], warp_max(x));  // finite: the slice has a valid key
          const float alpha = ex2(m_run[j] - m_new);         // 0 while m_run = -inf
          const float pv = kl < nvalid ? ex2(x - m_new) : 0.f;
          l_run[j] = l_run[j] * alpha + warp_sum(half == 0 ? pv : 0.f);  // each key once
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] *= alpha;
          m_run[j] = m_new;
          pr[j] = round_bf16(pv);  // P.V takes the bf16 probability
        }
        // P.V: lane l accumulates dims 4l .. 4l + 3 over the slice's valid keys (key k's p sits in lane k)
#pragma unroll 4
        for (int k = 0; k < nvalid; ++k) {
          const uint2 v = *(const uint2 *)(Vs + (size_t)k * kRowBytes + 8 * lane);
          const float v0 = bf16_lo(v.x), v1 = bf16_hi(v.x), v2 = bf16_lo(v.y), v3 = bf16_hi(v.y);
#pragma unroll
          for (int j = 0; j < GRP; ++j) {
            const float pk = __shfl_sync(0xffffffffu, pr[j], k);
            acc[j][0] = fmaf(pk, v0, acc[j][0]);
            acc[j][1] = fmaf(pk, v1, acc[j][1]);
            acc[j][2] = fmaf(pk, v2, acc[j][2]);
            acc[j][3] = fmaf(pk, v3, acc[j][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) gtc::mbar_arrive(S.empty + s);  // this warp is done with the stage
    }
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      if (lane == 0) S.w_m[warp][j] = m_run[j], S.w_l[warp][j] = l_run[j];
      *(float4 *)&S.w_acc[warp][j][4 * lane] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- merge the warps (fixed order), then ranges
  float *part = p.ws_f;  // [nq][max_split][D + 2] for row 0
  for (int i = threadIdx.x; i < GRP * kD; i += kThreads) {
    const int j = i / kD, d = i - j * kD;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.w_m[w][j]);
    float lsum = 0.f, a = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      if (S.w_l[w][j] == 0.f) continue;
      const float f = ex2(S.w_m[w][j] - M);
      lsum += S.w_l[w][j] * f;
      a += S.w_acc[w][j][d] * f;
    }
    const int h = g * GRP + j;
    if (nsplit == 1) {
      ((uint16_t *)p.out)[(int64_t)h * kD + d] = f32_to_bf16_bits(a / lsum);
    } else {
      float *slot = part + ((int64_t)h * p.max_split + split) * (kD + 2);
      slot[2 + d] = a;
      if (d == 0) slot[0] = M, slot[1] = lsum;
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *cnt = p.ws_cnt + g;
    const unsigned prev = atomicAdd(cnt, 1u);
    S.flag = prev == (unsigned)(nsplit - 1);
    if (S.flag) *cnt = 0u;
  }
  __syncthreads();
  if (!S.flag) return;
  __threadfence();
  for (int i = threadIdx.x; i < GRP * kD; i += kThreads) {
    const int j = i / kD, d = i - j * kD;
    const int h = g * GRP + j;
    const float *base = part + (int64_t)h * p.max_split * (kD + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(base + s * (kD + 2)));
    float lsum = 0.f, a = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ls = __ldcg(base + s * (kD + 2) + 1);
      if (ls == 0.f) continue;
      const float f = ex2(__ldcg(base + s * (kD + 2)) - M);
      lsum += ls * f;
      a += __ldcg(base + s * (kD + 2) + 2 + d) * f;
    }
    ((uint16_t *)p.out)[(int64_t)h * kD + d] = f32_to_bf16_bits(a / lsum);
  }
}

template <int GRP>
cudaError_t launch_grp(const AttnParams &p, cudaStream_t st, bool pdl) {
  static bool attr = false;
  const size_t smem = sizeof(Smem<GRP>) + 128;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(attn_stream_kernel<GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  return launch_kernel((const void *)attn_stream_kernel<GRP>, dim3(p.nkv, p.split_cap), dim3(kThreads), smem, st, pdl, p);
}

}  // namespace ast

// Whether egpt_attn_decode takes the streamed kernel for this call.
bool attn_stream_applies(int64_t m, int d, int dtype, unsigned flags, int grp) {
  return m == 1 && d == ast::kD && dtype == EGPT_BF16 && (grp == 1 || grp == 2 || grp == 4) &&
         !(flags & (EGPT_FLAG_APPEND | EGPT_FLAG_RAGGED | EGPT_FLAG_REF_SOFTMAX));
}

// Launch with p.split_cap = ranges per kv head (at most max_split, about one CTA per SM over the grid).
cudaError_t attn_stream_launch(AttnParams p, cudaStream_t st, bool pdl) {
  p.split_cap = std::max(1, std::min(p.max_split, std::max(1, num_sms() / p.nkv)));
  if (p.split_cap > 1 && (!p.ws_f || !p.ws_cnt)) p.split_cap = 1;
  switch (p.group) {
    case 1: return ast::launch_grp<1>(p, st, pdl);
    case 2: return ast::launch_grp<2>(p, st, pdl);
    default: return ast::launch_grp<4>(p, st, pdl);
  }
}

}  // namespace egpt
