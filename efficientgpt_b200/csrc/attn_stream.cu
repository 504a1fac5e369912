// Split-K decode attention for one query row over a long bf16 cache, streamed through shared memory with bulk
// copies (sm_100a): egpt_attn_decode's kernel for m = 1, bf16, head_dim 128, without EGPT_FLAG_APPEND,
// EGPT_FLAG_RAGGED or EGPT_FLAG_REF_SOFTMAX (the other cases run attn_split_kernel of attention.cu).
//
//   out[h] = softmax(scale q_h . K[0 .. L)) V[0 .. L),  L = *position + 1, q head h reading kv head h / GRP.
//
// Grid (nkv, ranges): a CTA owns one kv head, its GRP q heads and one range of whole 128-key blocks (ranges sized
// from L on the device, so a captured graph follows the position). A kv head's K rows (and V rows) are one
// contiguous stream, so a block of 128 keys is 32 KB of consecutive bytes, copied as eight 4 KB bulk copies
// (cp.async.bulk, this GPU's memory, no multicast): warp 8 keeps K and V blocks in flight through a 3-stage
// ring (192 KB), completion by transaction count on the stage's mbarrier; two stages load while the eight compute
// warps work on the third. Warp w takes keys 16 w .. 16 w + 15 of every block: lane l reads dims 4l .. 4l + 3 of
// each key row (q's same dims in registers) and one reduce-scatter of the partial dot products leaves every
// score in one lane; the warp keeps a running maximum, sum and P.V accumulator per q head (lane l: dims
// 4l .. 4l + 3; probabilities enter P.V rounded to bf16, the sums use the fp32 values) and releases the stage.
// The warps merge in a fixed order; one range writes the output, several write partials (maximum, sum,
// unnormalised output, base-2 exponents) and the last range of the kv head to arrive combines them. Every wait
// is bounded (EGPT_ERR_TIMEOUT); the producer drains its copies before the CTA exits.
#include "internal.h"
#include "common.cuh"

namespace egpt {
namespace ast {

constexpr int kD = 128;
constexpr int kBlock = 128;                 // keys per ring stage
constexpr int kStages = 3;
constexpr int kRowBytes = kD * 2;           // bf16 row: 256 bytes
constexpr int kBlockBytes = kBlock * kRowBytes;
constexpr unsigned kPiece = 16 * kRowBytes; // bytes per bulk copy: 4 KB
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
        for (unsigned o = 0; o < bytes; o += kPiece) {  // pieces of 16 rows: more copies in flight at once
          const unsigned n = min(kPiece, bytes - o);
          df::bulk_copy(S.ring[s][0] + o, Kg + (int64_t)b * kBlockBytes + o, n, S.full + s);
          df::bulk_copy(S.ring[s][1] + o, Vg + (int64_t)b * kBlockBytes + o, n, S.full + s);
        }
        ++issued;
      }
      for (int b = max(0, issued - kStages); b < issued; ++b)  // nothing may still be landing at exit
        gtc::mbar_drain(S.full + b % kStages, (unsigned)(b / kStages) & 1u);
    }
  } else {
    // ---------------------------------------------------------------- compute warps
    // every block: warp w takes keys 16 w .. 16 w + 15. Lane l holds q's dims 4l .. 4l + 3 of every head and forms
    // the partial dot products of those dims with each key (index 16 j + k for head j, key k); one reduce-scatter
    // leaves every total in one lane (GRP 1: key l / 2 in lanes l, two copies; GRP 2: index l; GRP 4: indices 2l,
    // 2l + 1).
    constexpr int NV = 16 * GRP, NS = NV > 32 ? NV / 32 : 1;  // values held per lane after the reduce-scatter
    constexpr int HL = 32 / GRP;                              // lanes per head after it
    const int slice = 16 * warp;
    float qr[GRP][4];
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      const float4 t = *(const float4 *)&S.q[j][4 * lane];
      qr[j][0] = t.x, qr[j][1] = t.y, qr[j][2] = t.z, qr[j][3] = t.w;
    }
    const int head = lane / HL;  // the head of this lane's totals
    float m_run = -INFINITY;     // running maximum of that head (the same in all its lanes)
    float l_lane = 0.f;          // this lane's share of that head's sum
    float acc[GRP][4];
#pragma unroll
    for (int j = 0; j < GRP; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int b = 0; b < nblk; ++b) {
      const int s = b % kStages;
      if (!__all_sync(0xffffffffu, gtc::mbar_wait(S.full + s, (unsigned)(b / kStages) & 1u))) break;
      const int nvalid = (int)min((int64_t)16, k1 - k0 - (int64_t)b * kBlock - slice);  // keys of this slice
      if (nvalid > 0) {
        const uint8_t *Ks = S.ring[s][0] + (size_t)slice * kRowBytes;
        const uint8_t *Vs = S.ring[s][1] + (size_t)slice * kRowBytes;
        float v[NV];
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // rows past nvalid give totals that are masked below
          const uint2 w = *(const uint2 *)(Ks + (size_t)k * kRowBytes + 8 * lane);
          const float k0v = bf16_lo(w.x), k1v = bf16_hi(w.x), k2v = bf16_lo(w.y), k3v = bf16_hi(w.y);
#pragma unroll
          for (int j = 0; j < GRP; ++j)
            v[16 * j + k] = fmaf(qr[j][0], k0v, qr[j][1] * k1v) + fmaf(qr[j][2], k2v, qr[j][3] * k3v);
        }
        // reduce-scatter: at offset o the lane keeps the upper half of its values if (lane & o), else the lower
        int cnt = NV;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          if (cnt > 1) {
            const int hv = cnt / 2;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
              if (i < hv) {
                const float send = up ? v[i] : v[i + hv];
                const float keep = up ? v[i + hv] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
              }
            }
            cnt = hv;
          } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
          }
        }
        // this lane's keys and the block maximum of its head (scores are in base-2 exponent units)
        float x[NS];
        float bm = -INFINITY;
#pragma unroll
        for (int t = 0; t < NS; ++t) {
          const int key = GRP == 1 ? lane >> 1 : (GRP == 2 ? lane & 15 : ((2 * lane + t) & 15));
          x[t] = key < nvalid ? v[t] : -INFINITY;
          bm = fmaxf(bm, x[t]);
        }
#pragma unroll
        for (int o = HL / 2; o >= 1; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float m_new = fmaxf(m_run, bm);  // finite: the slice has a valid key
        const float alpha = ex2(m_run - m_new);  // 0 while m_run = -inf
        m_run = m_new;
        float pr[NS];
        float psum = 0.f;
#pragma unroll
        for (int t = 0; t < NS; ++t) {
          const float pv = x[t] == -INFINITY ? 0.f : ex2(x[t] - m_new);
          psum += pv;
          pr[t] = round_bf16(pv);  // P.V takes the bf16 probability
        }
        if (GRP == 1 && (lane & 1)) psum = 0.f;  // the odd lane of a pair holds a second copy
        l_lane = l_lane * alpha + psum;
        // P.V: lane l accumulates dims 4l .. 4l + 3; head j's alpha and probabilities come from the lanes that hold
        // them
#pragma unroll
        for (int j = 0; j < GRP; ++j) {
          const float aj = __shfl_sync(0xffffffffu, alpha, j * HL);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] *= aj;
        }
#pragma unroll 4
        for (int k = 0; k < nvalid; ++k) {
          const uint2 w = *(const uint2 *)(Vs + (size_t)k * kRowBytes + 8 * lane);
          const float v0 = bf16_lo(w.x), v1 = bf16_hi(w.x), v2 = bf16_lo(w.y), v3 = bf16_hi(w.y);
#pragma unroll
          for (int j = 0; j < GRP; ++j) {
            float pk;
            if (GRP == 1) pk = __shfl_sync(0xffffffffu, pr[0], 2 * k);
            else if (GRP == 2) pk = __shfl_sync(0xffffffffu, pr[0], 16 * j + k);
            else pk = __shfl_sync(0xffffffffu, (k & 1) ? pr[NS - 1] : pr[0], (16 * j + k) >> 1);
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
    // each head's sum over its lanes
    float l_head = l_lane;
#pragma unroll
    for (int o = HL / 2; o >= 1; o >>= 1) l_head += __shfl_xor_sync(0xffffffffu, l_head, o);
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      const float mj = __shfl_sync(0xffffffffu, m_run, j * HL), lj = __shfl_sync(0xffffffffu, l_head, j * HL);
      if (lane == 0) S.w_m[warp][j] = mj, S.w_l[warp][j] = lj;
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
