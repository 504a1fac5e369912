// Split-K decode attention for one query row over a long bf16 cache, streamed through shared memory with bulk
// copies (sm_100a): egpt_attn_decode's kernels for m = 1, bf16, head_dim 128, without EGPT_FLAG_APPEND or
// EGPT_FLAG_RAGGED (the other cases run attn_split_kernel of attention.cu). With EGPT_FLAG_REF_SOFTMAX (the
// reference GPU kernel's rounding: the probabilities of 128-key block j rounded to bf16 relative to the maximum
// score of blocks 0 .. j) a first pass (attn_block_max_kernel) streams K alone and writes every block's maximum to
// the workspace slots past the ranges in use; the attention pass then starts each range from the maxima of the
// blocks before it and moves its running maximum block by block as the reference kernel does. A call whose
// workspace cannot hold the maxima of `cap` keys takes attn_split_kernel.
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
// unnormalised output; base-2 exponents, or natural ones with the reference rounding) and the last range of the kv
// head to arrive combines them. Every wait is bounded (EGPT_ERR_TIMEOUT); the copy warp drains its copies before
// the CTA exits, and the block-maximum pass's compute warps take every named barrier whatever their waits returned.
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
  float q[GRP][kD];                       // q heads (pre-scaled by scale log2(e) without the reference rounding)
  float w_m[kWarps][GRP], w_l[kWarps][GRP];
  float w_acc[kWarps][GRP][kD];           // (the block-maximum pass keeps its per-warp maxima here)
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

// The reduce-scatter of one warp's 16-key slice: lane l forms the partial dot products of q's dims 4l .. 4l + 3
// (qr) with each key row (index 16 j + k for head j, key k), and one reduce-scatter leaves every total in one lane:
// GRP 1: key l / 2 in lanes l (two copies); GRP 2: index l; GRP 4: indices 2l, 2l + 1 in v[0], v[1]. Rows past
// the valid keys give totals that the caller masks.
template <int GRP>
__device__ __forceinline__ void slice_scores(const uint8_t *Ks, const float (&qr)[GRP][4], float (&v)[16 * GRP]) {
  constexpr int NV = 16 * GRP;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint2 w = *(const uint2 *)(Ks + (size_t)k * kRowBytes + 8 * lane);
    const float k0v = bf16_lo(w.x), k1v = bf16_hi(w.x), k2v = bf16_lo(w.y), k3v = bf16_hi(w.y);
#pragma unroll
    for (int j = 0; j < GRP; ++j)
      v[16 * j + k] = fmaf(qr[j][0], k0v, qr[j][1] * k1v) + fmaf(qr[j][2], k2v, qr[j][3] * k3v);
  }
  // at offset o the lane keeps the upper half of its values if (lane & o), else the lower
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
}
// The key (within the slice) of total t of this lane.
template <int GRP>
__device__ __forceinline__ int slice_key(int lane, int t) {
  return GRP == 1 ? lane >> 1 : (GRP == 2 ? lane & 15 : ((2 * lane + t) & 15));
}
// Block maxima of the reference rounding: head h's slots past the ranges in use (h max_split + split_cap ..) of
// the workspace's partial slots, one float per 128-key block.
__device__ __forceinline__ float *block_max_base(const AttnParams &p, int h) {
  return p.ws_f + ((int64_t)h * p.max_split + p.split_cap) * (kD + 2);
}

// Common set-up of both kernels: the range of this CTA (false: nothing to do).
struct Range {
  int64_t k0, k1;
  int nsplit, nblk;
};
__device__ __forceinline__ bool range_setup(const AttnParams &p, Range &r) {
  const int64_t pos = *p.position;
  const int64_t L = pos + 1;
  if (L > p.cap || pos < 0) {
    if (threadIdx.x == 0) set_device_error(EGPT_ERR_SHAPE);
    return false;
  }
  range_of(L, p.split_cap, blockIdx.y, r.k0, r.k1, r.nsplit);
  if ((int)blockIdx.y >= r.nsplit) return false;
  r.nblk = (int)((r.k1 - r.k0 + kBlock - 1) / kBlock);
  return true;
}
// The copy warp's loop: blocks of K (and V unless K_ONLY) into the ring, then a bounded drain.
template <int GRP, bool K_ONLY>
__device__ __forceinline__ void copy_loop(Smem<GRP> &S, const uint8_t *Kg, const uint8_t *Vg, const Range &r) {
  int issued = 0;
  for (int b = 0; b < r.nblk; ++b) {
    const int s = b % kStages;
    if (b >= kStages && !gtc::mbar_wait(S.empty + s, (unsigned)((b / kStages) - 1) & 1u)) break;
    const unsigned bytes = (unsigned)(min((int64_t)kBlock, r.k1 - r.k0 - (int64_t)b * kBlock) * kRowBytes);
    gtc::mbar_arrive_tx(S.full + s, K_ONLY ? bytes : 2 * bytes);
    for (unsigned o = 0; o < bytes; o += kPiece) {  // pieces of 16 rows: more copies in flight at once
      const unsigned n = min(kPiece, bytes - o);
      df::bulk_copy(S.ring[s][0] + o, Kg + (int64_t)b * kBlockBytes + o, n, S.full + s);
      if (!K_ONLY) df::bulk_copy(S.ring[s][1] + o, Vg + (int64_t)b * kBlockBytes + o, n, S.full + s);
    }
    ++issued;
  }
  for (int b = max(0, issued - kStages); b < issued; ++b)  // nothing may still be landing at exit
    gtc::mbar_drain(S.full + b % kStages, (unsigned)(b / kStages) & 1u);
}

// Reference rounding, first pass: the maximum score of every 128-key block of each q head (scale applied after the
// dot product, as the reference kernel's scores), K streamed alone.
template <int GRP>
__global__ void __launch_bounds__(kThreads, 1) attn_block_max_kernel(AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem<GRP> &S = *(Smem<GRP> *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = blockIdx.x;
  Range r;
  if (!range_setup(p, r)) return;
  const uint8_t *Kg = (const uint8_t *)p.k_cache + ((int64_t)g * p.cap + r.k0) * kRowBytes;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      gtc::mbar_init(S.full + s, 1);
      gtc::mbar_init(S.empty + s, kWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < GRP * kD; i += kThreads) {
    const int j = i / kD, d = i - j * kD;
    S.q[j][d] = bf16_bits_to_f32(((const uint16_t *)p.q)[(int64_t)(g * GRP + j) * kD + d]);
  }
  __syncthreads();
  if (warp == kWarps) {
    if (lane == 0) copy_loop<GRP, true>(S, Kg, nullptr, r);
    return;
  }
  constexpr int NV = 16 * GRP, NS = NV > 32 ? NV / 32 : 1, HL = 32 / GRP;
  float(*wm)[kWarps][GRP] = reinterpret_cast<float(*)[kWarps][GRP]>(&S.w_acc[0][0][0]);  // [2][kWarps][GRP]
  const int slice = 16 * warp;
  float qr[GRP][4];
#pragma unroll
  for (int j = 0; j < GRP; ++j) {
    const float4 t = *(const float4 *)&S.q[j][4 * lane];
    qr[j][0] = t.x, qr[j][1] = t.y, qr[j][2] = t.z, qr[j][3] = t.w;
  }
  // every compute warp takes every barrier, whatever its waits returned
  bool ok = true;
  for (int b = 0; b < r.nblk; ++b) {
    const int s = b % kStages;
    ok = ok && __all_sync(0xffffffffu, gtc::mbar_wait(S.full + s, (unsigned)(b / kStages) & 1u));
    const int nvalid = (int)min((int64_t)16, r.k1 - r.k0 - (int64_t)b * kBlock - slice);
    float bm = -INFINITY;
    if (ok && nvalid > 0) {
      float v[NV];
      slice_scores<GRP>(S.ring[s][0] + (size_t)slice * kRowBytes, qr, v);
#pragma unroll
      for (int t = 0; t < NS; ++t)
        if (slice_key<GRP>(lane, t) < nvalid) bm = fmaxf(bm, v[t] * p.scale);
#pragma unroll
      for (int o = HL / 2; o >= 1; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
    }
    __syncwarp();
    if (ok && lane == 0) gtc::mbar_arrive(S.empty + s);
#pragma unroll
    for (int j = 0; j < GRP; ++j) {
      const float bj = __shfl_sync(0xffffffffu, bm, j * HL);
      if (lane == 0) wm[b & 1][warp][j] = bj;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory");
    if (warp == 0 && lane < GRP) {
      float m = wm[b & 1][0][lane];
      for (int w = 1; w < kWarps; ++w) m = fmaxf(m, wm[b & 1][w][lane]);
      block_max_base(p, g * GRP + lane)[r.k0 / kBlock + b] = m;
    }
  }
}

template <int GRP, bool REF>
__global__ void __launch_bounds__(kThreads, 1) attn_stream_kernel(AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem<GRP> &S = *(Smem<GRP> *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, split = blockIdx.y;
  Range r;
  if (!range_setup(p, r)) return;
  const int64_t k0 = r.k0, k1 = r.k1;
  const int nsplit = r.nsplit, nblk = r.nblk;
  const uint8_t *Kg = (const uint8_t *)p.k_cache + ((int64_t)g * p.cap + k0) * kRowBytes;
  const uint8_t *Vg = (const uint8_t *)p.v_cache + ((int64_t)g * p.cap + k0) * kRowBytes;
  // scores in base-2 exponent units (q pre-scaled by scale log2(e), ex2) or, with the reference rounding, natural
  // units with the scale applied after the dot product (expf), as the first pass computed the block maxima
  const float qs = REF ? 1.f : p.scale * 1.4426950408889634f;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      gtc::mbar_init(S.full + s, 1);
      gtc::mbar_init(S.empty + s, kWarps);  // every compute warp releases every block
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < GRP * kD; i += kThreads) {
    const int j = i / kD, d = i - j * kD;
    S.q[j][d] = bf16_bits_to_f32(((const uint16_t *)p.q)[(int64_t)(g * GRP + j) * kD + d]) * qs;
  }
  __syncthreads();

  if (warp == kWarps) {
    // ---------------------------------------------------------------- copy warp
    if (lane == 0) copy_loop<GRP, false>(S, Kg, Vg, r);
  } else {
    // ---------------------------------------------------------------- compute warps
    // every block: warp w takes keys 16 w .. 16 w + 15 (slice_scores); lane l accumulates P.V for dims
    // 4l .. 4l + 3 of every head
    constexpr int NV = 16 * GRP, NS = NV > 32 ? NV / 32 : 1;  // totals held per lane after the reduce-scatter
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
    const float *bmx = nullptr;  // reference rounding: this head's block maxima
    if (REF) {
      // the running maximum before the range: the maxima of the blocks before it (the head's lanes share them)
      bmx = block_max_base(p, g * GRP + head);
      const int kb0 = (int)(k0 / kBlock);
      float mb = -INFINITY;
      for (int b = lane % HL; b < kb0; b += HL) mb = fmaxf(mb, __ldcg(bmx + b));
#pragma unroll
      for (int o = HL / 2; o >= 1; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      m_run = mb;
      bmx += kb0;
    }
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
        slice_scores<GRP>(Ks, qr, v);
        float x[NS];
        float bm = -INFINITY;
#pragma unroll
        for (int t = 0; t < NS; ++t) {
          x[t] = slice_key<GRP>(lane, t) < nvalid ? (REF ? v[t] * p.scale : v[t]) : -INFINITY;
          bm = fmaxf(bm, x[t]);
        }
        if (REF) {
          bm = __ldcg(bmx + b);  // the block's maximum over all its keys: the reference kernel's running maximum
        } else {
#pragma unroll
          for (int o = HL / 2; o >= 1; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        }
        const float m_new = fmaxf(m_run, bm);  // finite: the slice has a valid key
        const float alpha = m_run == -INFINITY ? 0.f : (REF ? expf(m_run - m_new) : ex2(m_run - m_new));
        m_run = m_new;
        float pr[NS];
        float psum = 0.f;
#pragma unroll
        for (int t = 0; t < NS; ++t) {
          const float pv = x[t] == -INFINITY ? 0.f : (REF ? expf(x[t] - m_new) : ex2(x[t] - m_new));
          psum += pv;
          pr[t] = round_bf16(pv);  // P.V takes the bf16 probability
        }
        if (GRP == 1 && (lane & 1)) psum = 0.f;  // the odd lane of a pair holds a second copy
        l_lane = l_lane * alpha + psum;
        // head j's alpha and probabilities come from the lanes that hold them
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
      }  // a warp without keys in the range's last block keeps its state relative to its own last maximum
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
      const float f = REF ? expf(S.w_m[w][j] - M) : ex2(S.w_m[w][j] - M);
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
      const float f = REF ? expf(__ldcg(base + s * (kD + 2)) - M) : ex2(__ldcg(base + s * (kD + 2)) - M);
      lsum += ls * f;
      a += __ldcg(base + s * (kD + 2) + 2 + d) * f;
    }
    ((uint16_t *)p.out)[(int64_t)h * kD + d] = f32_to_bf16_bits(a / lsum);
  }
}

template <int GRP, bool REF>
cudaError_t launch_grp(const AttnParams &p, cudaStream_t st, bool pdl) {
  static int configured[64] = {0};  // the shared-memory opt-in, per device
  const size_t smem = sizeof(Smem<GRP>) + 128;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_stream_kernel<GRP, REF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e == cudaSuccess && REF)
      e = cudaFuncSetAttribute(attn_block_max_kernel<GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const dim3 grid(p.nkv, p.split_cap);
  if (REF) {  // block maxima first; the attention pass follows in stream order
    const cudaError_t e = launch_kernel((const void *)attn_block_max_kernel<GRP>, grid, dim3(kThreads), smem, st, pdl, p);
    if (e != cudaSuccess) return e;
    return launch_kernel((const void *)attn_stream_kernel<GRP, REF>, grid, dim3(kThreads), smem, st, false, p);
  }
  return launch_kernel((const void *)attn_stream_kernel<GRP, REF>, grid, dim3(kThreads), smem, st, pdl, p);
}

}  // namespace ast

// Ranges per kv head for the streamed kernels: about one CTA per SM over the grid, at most max_split; with the
// reference rounding the workspace slots past the ranges must also hold the block maxima of the longest context
// (0: the streamed kernels do not take the call).
static int attn_stream_ranges(const AttnParams &p, bool ref) {
  int cap = std::max(1, std::min(p.max_split, std::max(1, num_sms() / p.nkv)));
  if (!ref) return (cap > 1 && (!p.ws_f || !p.ws_cnt)) ? 1 : cap;
  if (!p.ws_f || !p.ws_cnt) return 0;
  const int64_t blocks = (p.cap + ast::kBlock - 1) / ast::kBlock;
  const int64_t slots = (blocks + ast::kD + 2 - 1) / (ast::kD + 2);  // partial slots the maxima take per head
  cap = (int)std::min<int64_t>(cap, (int64_t)p.max_split - slots);
  return cap >= 1 ? cap : 0;
}

// Whether egpt_attn_decode takes the streamed kernels for this call.
bool attn_stream_applies(const AttnParams &p, int64_t m, int d, int dtype, unsigned flags) {
  if (m != 1 || d != ast::kD || dtype != EGPT_BF16 || (flags & (EGPT_FLAG_APPEND | EGPT_FLAG_RAGGED)) ||
      !(p.group == 1 || p.group == 2 || p.group == 4))
    return false;
  return attn_stream_ranges(p, (flags & EGPT_FLAG_REF_SOFTMAX) != 0) > 0;
}

cudaError_t attn_stream_launch(AttnParams p, cudaStream_t st, bool pdl) {
  const bool ref = (p.flags & EGPT_FLAG_REF_SOFTMAX) != 0;
  p.split_cap = attn_stream_ranges(p, ref);
  switch (p.group) {
    case 1: return ref ? ast::launch_grp<1, true>(p, st, pdl) : ast::launch_grp<1, false>(p, st, pdl);
    case 2: return ref ? ast::launch_grp<2, true>(p, st, pdl) : ast::launch_grp<2, false>(p, st, pdl);
    default: return ref ? ast::launch_grp<4, true>(p, st, pdl) : ast::launch_grp<4, false>(p, st, pdl);
  }
}

}  // namespace egpt
