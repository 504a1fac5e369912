// Library plumbing (error reporting, device queries) and the whole-token decode step of the Qwen3 family.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace egpt {

static thread_local std::string t_error;

int set_error(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

void clear_error() { t_error.clear(); }

int check_launch(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return EGPT_OK;
  return set_error(EGPT_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

size_t smem_limit() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 227 * 1024;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0) v = 227 * 1024;
    cache[dev] = v;
  }
  return (size_t)cache[dev];
}

}  // namespace egpt

using namespace egpt;

extern "C" const char *egpt_version(void) { return "efficientgpt-b200 0.1.0 (sm_100a)"; }

extern "C" const char *egpt_last_error(void) { return t_error.c_str(); }

extern "C" int egpt_num_sms(void) { return num_sms(); }

extern "C" int egpt_device_error(int clear) {
  clear_error();
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "device_error: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "device_error: %s", cudaGetErrorString(e));
  if (clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "device_error: %s", cudaGetErrorString(e));
  }
  if (v) set_error(v, "a kernel reported device error %d", v);
  return v;
}

extern "C" int egpt_decode_step(const egpt_qwen3_plan *P, void *stream) {
  clear_error();
  if (!P || !P->layers || !P->embed || !P->final_norm || !P->w_lm || !P->s_lm || !P->rope_cos || !P->rope_sin ||
      !P->token || !P->position || !P->h || !P->qkv || !P->attn || !P->act || !P->lm_ws)
    return set_error(EGPT_ERR_ARG, "decode_step: null pointer in plan");
  if (P->n_layers < 1 || P->hidden < 1 || P->n_q_heads < 1 || P->n_kv_heads < 1 || P->head_dim < 1 ||
      P->intermediate < 1 || P->vocab < 1 || P->cap < 1)
    return set_error(EGPT_ERR_SHAPE, "decode_step: bad model sizes");
  if (P->tp_world > 1)
    return set_error(EGPT_ERR_ARG, "decode_step: tensor parallelism runs on egpt_decode_step_persistent only");
  const unsigned pdl = P->flags & EGPT_FLAG_PDL;
  const int sdt = P->scale_dtype;
  // GEMVs on the exact int8 tensor-core kernel (the persistent step's arithmetic) where the shapes allow it
  const int64_t reg_max = 12 * 512;
  bool exact_ok = P->hidden % 16 == 0 && P->intermediate % 16 == 0 && (P->n_q_heads * P->head_dim) % 16 == 0 &&
                  P->hidden <= reg_max && (int64_t)P->n_q_heads * P->head_dim <= 2 * reg_max &&
                  P->intermediate <= 2 * reg_max && (uintptr_t)P->embed % 16 == 0 && (uintptr_t)P->h % 16 == 0 &&
                  (uintptr_t)P->attn % 16 == 0 && (uintptr_t)P->act % 16 == 0;
  for (int l = 0; exact_ok && l < P->n_layers; ++l) {
    const egpt_qwen3_layer &L = P->layers[l];
    exact_ok = (uintptr_t)L.w_qkv % 16 == 0 && (uintptr_t)L.w_o % 16 == 0 && (uintptr_t)L.w_gu % 16 == 0 &&
               (uintptr_t)L.w_down % 16 == 0;
  }
  const unsigned gx = exact_ok ? EGPT_FLAG_EXACT : 0u;
  const int64_t H = P->hidden, D = P->head_dim, NQ = P->n_q_heads, NKV = P->n_kv_heads, I = P->intermediate;
  const int64_t nqkv = (NQ + 2 * NKV) * D;
  for (int l = 0; l < P->n_layers; ++l) {
    const egpt_qwen3_layer &L = P->layers[l];
    const void *x = l == 0 ? P->embed : P->h;
    const unsigned f0 = EGPT_FLAG_RMSNORM | pdl | gx | (l == 0 ? EGPT_FLAG_EMBED : 0u);
    const int64_t ldx = l == 0 ? P->vocab : H;  // embedding mode: ldx = table rows
    int rc = egpt_gemv_i8(P->qkv, x, EGPT_BF16, 1, ldx, nqkv, L.w_qkv, L.s_qkv, sdt, nqkv, H, nullptr, P->h,
                          EGPT_EPI_NONE, L.ln_in, P->eps, P->token, f0, stream);
    if (rc) return rc;
    rc = egpt_attn_decode(P->attn, NQ * D, P->qkv, nqkv, L.k_cache, L.v_cache, P->cap, P->position, 1, (int)NQ,
                          (int)NKV, (int)D, L.q_norm, L.k_norm, P->eps, P->rope_cos, P->rope_sin, P->attn_scale,
                          P->attn_max_split, P->attn_ws, P->attn_ws_bytes, EGPT_BF16,
                          EGPT_FLAG_APPEND | EGPT_FLAG_REF_SOFTMAX | pdl, stream);
    if (rc) return rc;
    rc = egpt_gemv_i8(P->h, P->attn, EGPT_BF16, 1, NQ * D, H, L.w_o, L.s_o, sdt, H, NQ * D, nullptr, P->h,
                      EGPT_EPI_RESIDUAL, nullptr, 0.f, nullptr, pdl | gx, stream);
    if (rc) return rc;
    rc = egpt_gemv_i8(P->act, P->h, EGPT_BF16, 1, H, I, L.w_gu, L.s_gu, sdt, 2 * I, H, nullptr, nullptr,
                      EGPT_EPI_SILU_MUL, L.ln_post, P->eps, nullptr, EGPT_FLAG_RMSNORM | pdl | gx, stream);
    if (rc) return rc;
    rc = egpt_gemv_i8(P->h, P->act, EGPT_BF16, 1, I, H, L.w_down, L.s_down, sdt, H, I, nullptr, P->h,
                      EGPT_EPI_RESIDUAL, nullptr, 0.f, nullptr, pdl | gx, stream);
    if (rc) return rc;
  }
  const unsigned gl = (gx && P->vocab % 16 == 0 && (uintptr_t)P->w_lm % 16 == 0) ? EGPT_FLAG_EXACT : 0u;
  return egpt_lm_head_argmax(P->token, P->position, P->logits, P->h, P->w_lm, P->s_lm, sdt, P->vocab, H,
                             P->final_norm, P->eps, P->lm_ws, P->lm_ws_bytes,
                             EGPT_FLAG_RMSNORM | EGPT_FLAG_ADVANCE | pdl | gl, stream);
}

// ---------------------------------------------------------------------------------------- tensor parallelism
// Exchange region: 16-byte LL slots, lm_head keys [8] at 0, fp64 partial sums [2][8][hidden] at 4096.
extern "C" size_t egpt_tp_xchg_bytes(int64_t hidden) {
  return hidden > 0 ? (size_t)4096 + (size_t)2 * 8 * (size_t)hidden * 16 : 0;
}

extern "C" int egpt_tp_xchg_alloc(void **ptr, size_t bytes) {
  clear_error();
  if (!ptr || bytes == 0) return set_error(EGPT_ERR_ARG, "tp_xchg_alloc: null pointer or zero size");
  *ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "tp_xchg_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(EGPT_ERR_LAUNCH, "tp_xchg_alloc: cudaMemset: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return EGPT_OK;
}

extern "C" int egpt_tp_xchg_free(void *ptr) {
  clear_error();
  if (!ptr) return EGPT_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? EGPT_OK : set_error(EGPT_ERR_LAUNCH, "tp_xchg_free: %s", cudaGetErrorString(e));
}

extern "C" int egpt_ipc_handle(const void *ptr, void *handle64) {
  clear_error();
  if (!ptr || !handle64) return set_error(EGPT_ERR_ARG, "ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
  if (e != cudaSuccess) return set_error(EGPT_ERR_LAUNCH, "ipc_handle: %s", cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  return EGPT_OK;
}

extern "C" int egpt_ipc_open(const void *handle64, void **ptr) {
  clear_error();
  if (!ptr || !handle64) return set_error(EGPT_ERR_ARG, "ipc_open: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? EGPT_OK : set_error(EGPT_ERR_LAUNCH, "ipc_open: %s", cudaGetErrorString(e));
}

extern "C" int egpt_ipc_close(void *ptr) {
  clear_error();
  if (!ptr) return EGPT_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? EGPT_OK : set_error(EGPT_ERR_LAUNCH, "ipc_close: %s", cudaGetErrorString(e));
}
