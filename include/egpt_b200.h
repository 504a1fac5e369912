/*
 * efficientgpt-b200: C-ABI of the batch-1 int8 decode engine for NVIDIA B200 (sm_100a).
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t passed as `void *` (NULL = the
 * legacy default stream), launches stream-ordered work and returns an int status (EGPT_OK = 0). Nothing
 * here allocates device memory except egpt_tp_xchg_alloc (CUDA IPC exports whole allocations, so the
 * tensor-parallel exchange region is one of its own): callers own weights, activations, KV cache and
 * workspaces, so every call can be captured in a CUDA graph. On a non-zero status egpt_last_error() returns a message for the
 * calling thread.
 *
 * The "replaces" line above each function names the reference symbol (BagelsFun/efficientgpt, paths
 * relative to that project) whose behaviour the entry point provides.
 */
#ifndef EGPT_B200_H
#define EGPT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EGPT_API __attribute__((visibility("default")))
#else
#define EGPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------------------- */
#define EGPT_OK 0
#define EGPT_ERR_SHAPE 1     /* a size is out of range or inconsistent                                    */
#define EGPT_ERR_DTYPE 2     /* unsupported dtype combination                                             */
#define EGPT_ERR_ALIGN 3     /* a pointer or leading dimension breaks the 16-byte rule of the fast path   */
#define EGPT_ERR_LAUNCH 4    /* the CUDA launch failed (message from the runtime in egpt_last_error)      */
#define EGPT_ERR_TIMEOUT 5   /* a device-side wait gave up (reported by egpt_device_error)                */
#define EGPT_ERR_ARG 6       /* null pointer or bad flag                                                  */
#define EGPT_ERR_WORKSPACE 7 /* workspace too small                                                       */

/* ---- dtypes ---------------------------------------------------------------------------------------- */
#define EGPT_F32 0
#define EGPT_BF16 1

/* ---- GEMV epilogues -------------------------------------------------------------------------------- */
#define EGPT_EPI_NONE 0     /* y = round(acc * s[n]) (+ bias[n])                                          */
#define EGPT_EPI_RESIDUAL 1 /* y = round(residual[n] + round(acc * s[n]))   (in place when out==residual) */
#define EGPT_EPI_SILU_MUL 2 /* w = cat(gate, up) [2I, K]: y[i] = round(round(silu(g_i)) * u_i), I outputs  */
#define EGPT_EPI_GELU 3     /* fp32 only: y = gelu_erf(acc * s[n] + bias[n])                              */

/* ---- flags ----------------------------------------------------------------------------------------- */
#define EGPT_FLAG_DOUBLE_ROUND 1u /* round acc to bf16 before the scale (the reference's >16-row branch)  */
#define EGPT_FLAG_RMSNORM 2u      /* prologue: x <- RMSNorm(x) * norm_w (bf16 rounding as HF Qwen3)        */
#define EGPT_FLAG_PDL 4u          /* launch with programmatic dependent launch                            */
#define EGPT_FLAG_EMBED 8u        /* prologue: x <- embed[*token] and residual <- the same row            */
#define EGPT_FLAG_ADVANCE 16u     /* lm_head argmax: also *position += 1                                  */
#define EGPT_FLAG_APPEND 32u      /* attention: q/k-RMSNorm + RoPE + KV append of this step's row in-kernel */
#define EGPT_FLAG_NO_TMA 64u      /* GEMV: force the plain-load kernel (any K)                            */
#define EGPT_FLAG_REF_SOFTMAX 128u /* attention: bf16 probabilities rounded as the reference GPU kernel does */
#define EGPT_FLAG_X_F32 256u      /* lm_head argmax: x and logits are fp32 (nanoGPT), no bf16 rounding      */
#define EGPT_FLAG_EXACT 512u      /* GEMV, one bf16 row: exact int8 tensor-core sums, one rounding per row    */
#define EGPT_FLAG_RAGGED 1024u    /* attention: the m rows are m sequences, row i at position[i] with its own
                                     cache (kv heads [i nkv, (i + 1) nkv) of caches laid out [m nkv][cap][d]) */
#define EGPT_FLAG_ADD_OUT 2048u   /* GEMM: y holds the residual on entry and becomes bf16(y + result)         */

/* ---- library ---------------------------------------------------------------------------------------- */
EGPT_API const char *egpt_version(void);
EGPT_API const char *egpt_last_error(void);
/* Reads (and with clear != 0 resets) the device error word that kernels set when a bounded wait gives up.
 * Synchronises the device. Returns the code (EGPT_OK when no kernel reported a problem). */
EGPT_API int egpt_device_error(int clear);
/* Number of SMs of the current device (used to size grids and workspaces). */
EGPT_API int egpt_num_sms(void);

/* ---- quantiser --------------------------------------------------------------------------------------
 * replaces: research/realmodel/int8_linear.py:106-117 quantize_weight
 * s[n] = max(max_k |w[n,k]| / 127, 1e-12) (fp32, stored as scale_dtype); q = clamp(rint(w / s), -127, 127).
 * w is fp32 or bf16 [n, k] row-major with leading dimension k. Bit-identical to the reference formula. */
EGPT_API int egpt_quantize_rows(int8_t *q, void *scale, int scale_dtype, const void *w, int w_dtype, int64_t n, int64_t k,
                       void *stream);

/* ---- int8 weight-only GEMV / small GEMM ------------------------------------------------------------
 * replaces: research/realmodel/int8_linear.py:26-85 (_dot16, _part, _reduce, int8_matmul) and the
 *           op efficientgpt::int8_linear (int8_linear.py:88-98) for M <= 16 rows
 * out[m, n] = epilogue(s[n] * sum_k x[m, k] * q[n, k]) with fp32 accumulation; x/out/residual/bias have
 * dtype x_dtype (bf16 for the Qwen path, fp32 for the nanoGPT path), s has scale_dtype.
 * Leading dimensions: x ldx, out/residual ldo (elements). EGPT_EPI_SILU_MUL writes n/2 outputs per row.
 * token (int64, device) is read with EGPT_FLAG_EMBED, in which case x points at the embedding table
 * [vocab, K], ldx is vocab (the token is bounds-checked against it) and residual receives the selected row.
 * EGPT_FLAG_EXACT (m = 1, bf16 x, epilogue none / residual / SiLU*up, optional RMSNorm and embedding
 * prologues, n and k multiples of 16, k up to 12288 or 6144 with a prologue): the int8 tensor-core kernel of
 * the persistent decode step; the row sums are exact (fixed-point input, int64 sums) and rounded once,
 * out = bf16(fp32(sum) * s). */
EGPT_API int egpt_gemv_i8(void *out, const void *x, int x_dtype, int64_t m, int64_t ldx, int64_t ldo, const int8_t *w,
                 const void *scale, int scale_dtype, int64_t n, int64_t k, const void *bias, void *residual,
                 int epilogue, const void *norm_w, float eps, const int64_t *token, unsigned flags, void *stream);

/* ---- lm_head + greedy argmax ------------------------------------------------------------------------
 * replaces: transformers Qwen3ForCausalLM lm_head (modeling_qwen3.py:503-505) on the int8 op, followed by
 *           research/realmodel/fast_decode.py:48 (argmax(-1), first index on ties) and :49 (position += 1)
 * token[0] = argmax_n bf16(s[n] * sum_k xn[k] q[n, k]) where xn = RMSNorm(x)*norm_w if EGPT_FLAG_RMSNORM.
 * logits ([n], nullable; bf16, or fp32 with EGPT_FLAG_X_F32) receives the logits. ws must hold egpt_lm_head_ws_bytes(n) bytes,
 * zero-filled once before first use (the kernel leaves its counter at zero). EGPT_FLAG_EXACT (bf16 x, n and k
 * multiples of 16): the logits come from the exact int8 tensor-core kernel, bf16(fp32(exact sum) * s). */
EGPT_API size_t egpt_lm_head_ws_bytes(int64_t n);
EGPT_API int egpt_lm_head_argmax(int64_t *token, int64_t *position, void *logits, const void *x, const int8_t *w,
                        const void *scale, int scale_dtype, int64_t n, int64_t k, const void *norm_w, float eps,
                        void *ws, size_t ws_bytes, unsigned flags, void *stream);

/* ---- norms and embedding ----------------------------------------------------------------------------
 * replaces: transformers Qwen3RMSNorm.forward (modeling_qwen3.py:59-64): y = w * bf16(x * rsqrt(mean(x^2)+eps))
 * x, w, y bf16; rows of length dim. */
EGPT_API int egpt_rmsnorm(void *out, const void *x, const void *w, int64_t rows, int64_t dim, float eps, void *stream);
/* nanoGPT LayerNorm (model.py:18-27), fp32: y = (x - mean) / sqrt(var + eps) * w + b (b nullable). */
EGPT_API int egpt_layernorm_f32(float *out, const float *x, const float *w, const float *b, int64_t rows, int64_t dim,
                       float eps, void *stream);
/* Embedding rows: out[i] = table[ids[i]] (+ pos_table[p0 + i] when pos_table is non-null, fp32 only, with
 * p0 = pos0 + *position when position (device int64) is non-null, else pos0).
 * replaces: tr.wte(ids) + tr.wpe(pos) (model.py:176-180; research/phase4/decoder.py:20,130).
 * dtype bf16 or fp32; ids int64 on the device. */
EGPT_API int egpt_embed(void *out, const int64_t *ids, int64_t rows, const void *table, const void *pos_table,
               int64_t pos0, const int64_t *position, int64_t vocab, int64_t dim, int dtype, void *stream);

/* ---- attention --------------------------------------------------------------------------------------
 * replaces: transformers Qwen3Attention.forward core (modeling_qwen3.py:258-291: q/k RMSNorm, RoPE,
 *           StaticLayer.update index_copy, SDPA with GQA and the causal mask over the static cache) and the
 *           split-K decode attention design of research/phase5/decode_attention.py:22-71
 *
 * egpt_qk_norm_rope_kv_append: for rows i < m at position pos0 + i (pos0 = *position):
 *   q_out[i] = RoPE(RMSNorm(q_i) * q_norm_w), K[pos0+i] = RoPE(RMSNorm(k_i) * k_norm_w), V[pos0+i] = v_i.
 *   qkv rows are [nq*d | nkv*d | nkv*d] bf16 with leading dimension ldqkv. Caches are [nkv][cap][d] bf16.
 *   rope_cos / rope_sin are bf16 [cap][d/2] (the HF table, cos[i] == cos[i + d/2]).
 *   q_norm_w / k_norm_w may be NULL (no q/k norm: nanoGPT-style attention), rope_cos NULL = no RoPE.
 * egpt_attn_decode: out[i, h] = softmax(scale * q_i,h . K[0..L_i)) V[0..L_i), L_i = pos0 + i + 1, GQA head
 *   h uses kv head h / (nq / nkv). With EGPT_FLAG_APPEND (m must be 1, or any m with EGPT_FLAG_RAGGED) the
 *   norm/RoPE/append above is done in-kernel from the raw qkv row, else q comes from q (ldq) already rotated.
 *   With EGPT_FLAG_RAGGED (ragged batches, research/phase5/ragged.py) row i is its own sequence at
 *   position[i] (position is an int64 array of m) with its own cache heads [i nkv, (i + 1) nkv).
 *   Work is split over up to max_split ranges of whole 128-key blocks per kv head; ws must hold
 *   egpt_attn_ws_bytes(m, nq, nkv, d, max_split) bytes, zero-filled once before first use.
 *   bf16: probabilities enter P.V rounded to bf16. With EGPT_FLAG_REF_SOFTMAX they are rounded relative to
 *   the running maximum of the 128-key block walk of the reference's GPU SDPA kernel (a range then rescores
 *   the keys before it); without it each range starts its own walk (same accuracy, less work). One bf16 row
 *   (m = 1) with d = 128 and neither APPEND nor RAGGED streams the cache through shared memory with bulk copies
 *   (one CTA per SM over the grid; the same workspace; with REF_SOFTMAX a first pass over K writes the 128-key
 *   block maxima into the workspace's unused partial slots, and calls whose workspace lacks the room for the
 *   maxima of cap keys run the split kernel).
 *   dtype: bf16 (Qwen) or fp32 (nanoGPT, no norm/RoPE). */
EGPT_API int egpt_qk_norm_rope_kv_append(void *q_out, const void *qkv, int64_t ldqkv, void *k_cache, void *v_cache,
                                int64_t cap, const int64_t *position, int64_t m, int nq, int nkv, int d,
                                const void *q_norm_w, const void *k_norm_w, float eps, const void *rope_cos,
                                const void *rope_sin, int dtype, void *stream);
EGPT_API size_t egpt_attn_ws_bytes(int64_t m, int nq, int nkv, int d, int max_split);
EGPT_API int egpt_attn_decode(void *out, int64_t ldo, const void *q, int64_t ldq, void *k_cache, void *v_cache, int64_t cap,
                     const int64_t *position, int64_t m, int nq, int nkv, int d, const void *q_norm_w,
                     const void *k_norm_w, float eps, const void *rope_cos, const void *rope_sin, float scale,
                     int max_split, void *ws, size_t ws_bytes, int dtype, unsigned flags, void *stream);

/* egpt_attn_decode_noalloc: egpt_attn_decode without a caller workspace. No counterpart in the reference.
 * For callers that must not allocate device memory themselves: code running inside another framework's
 * operator whose device memory belongs to that framework's allocator, or a serving path that plans all of its
 * memory up front and forbids allocations afterwards. The split partials and counters use one built-in device
 * array of EGPT_ATTN_NOALLOC_SCRATCH_BYTES (512 KiB, held by every GPU that loads the library until exit);
 * calls whose egpt_attn_ws_bytes(m, nq, nkv, d, max_split) exceeds it return EGPT_ERR_WORKSPACE and launch
 * nothing. No cudaMalloc, cudaFree or other allocating call is made. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current); make that first call before any
 * stream capture. Every call clears the array's arrival counters on `stream` (cudaMemsetAsync) before its
 * kernel; the partials are overwritten by each call. All calls on a device share the array, so calls whose
 * kernels can overlap on the GPU (different streams without ordering between them) race: order them. */
#define EGPT_ATTN_NOALLOC_SCRATCH_BYTES 524288
EGPT_API int egpt_attn_decode_noalloc(void *out, int64_t ldo, const void *q, int64_t ldq, void *k_cache,
                                      void *v_cache, int64_t cap, const int64_t *position, int64_t m, int nq,
                                      int nkv, int d, const void *q_norm_w, const void *k_norm_w, float eps,
                                      const void *rope_cos, const void *rope_sin, float scale, int max_split,
                                      int dtype, unsigned flags, void *stream);

/* ---- causal attention over a prompt (prefill) on the tcgen05 tensor cores ----------------------------
 * replaces: the SDPA call of the HF Qwen3 attention over the prompt (modeling_qwen3.py:258-291 with
 *           is_causal), as GraphGreedyDecoder's prefill runs it (research/realmodel/fast_decode.py:77-85).
 * out[i, h] = softmax(scale * q[i, h] . K[0 .. pos0 + i]) V[0 .. pos0 + i] for rows i < m; q bf16 [m][ldq]
 * (head h at columns h*d, already normed and rotated), caches bf16 [nkv][cap][d] holding keys 0 .. pos0 + m - 1,
 * out bf16 [m][ldo]; GQA head h reads kv head h / (nq / nkv). d = 128. fp32 scores and sums, probabilities
 * rounded to bf16 relative to the running row maximum before P.V, one bf16 rounding of the output. pos0 > 0
 * continues a prompt whose first pos0 keys are already cached (chunked prefill; m = 1 is one decode row).
 * Pointers 16-byte aligned, ldq and ldo multiples of 8. No workspace. */
EGPT_API int egpt_attn_prefill(void *out, int64_t ldo, const void *q, int64_t ldq, const void *k_cache,
                               const void *v_cache, int64_t cap, int64_t pos0, int64_t m, int nq, int nkv, int d,
                               float scale, void *stream);

/* ---- argmax over rows of bf16/fp32 logits -----------------------------------------------------------
 * replaces: logits[:, -1].argmax(-1) (research/realmodel/fast_decode.py:48,84): first index on ties. */
EGPT_API int egpt_argmax_rows(int64_t *out, const void *logits, int64_t rows, int64_t n, int64_t ld, int dtype, void *stream);

/* ---- int8-weight GEMM for prefill on the tcgen05 tensor cores --------------------------------------------
 * replaces: research/realmodel/int8_linear.py:96-97, the op's > 16-row branch bf16(bf16(x @ bf16(q).T) * s)
 * (with EGPT_FLAG_DOUBLE_ROUND; without it bf16(fp32 sum * s)). x bf16 [M, K] (leading dimension ldx),
 * q int8 [N, K] row-major, s [N] bf16 or fp32, y bf16 [M, N] (leading dimension ldy). fp32 accumulation on
 * tcgen05.mma (128 x 256 tiles, int8 widened to bf16 in shared memory). K a multiple of 64; x, y, q 16-byte
 * aligned, ldx and ldy multiples of 8. When the tiles alone leave SMs idle (few rows) K is split over several
 * CTAs per tile if ws holds egpt_gemm_i8_tc_ws_bytes(M, N, K) bytes (16-byte aligned; fp32 partials, no
 * zero-fill needed), followed by a reduce launch; with a smaller (or NULL) ws one CTA takes each tile. */
EGPT_API size_t egpt_gemm_i8_tc_ws_bytes(int64_t M, int64_t N, int64_t K);
/* With EGPT_FLAG_ADD_OUT y is also the residual: y = bf16(y + bf16(result)), the HF residual add of o_proj and
 * down_proj fused into the epilogue. */
EGPT_API int egpt_gemm_i8_tc(void *y, int64_t ldy, const void *x, int64_t ldx, int64_t M, const int8_t *q,
                             const void *s, int s_dtype, int64_t N, int64_t K, unsigned flags, void *ws,
                             size_t ws_bytes, void *stream);

/* ---- SwiGLU activation over prefill rows ----------------------------------------------------------------
 * replaces: act_fn(gate_proj(x)) * up_proj(x) of the HF Qwen3 MLP (modeling_qwen3.py:81-82) on the prompt rows:
 * out[r, i] = bf16(bf16(silu(g)) * u), g = gu[r, i], u = gu[r, inter + i] for the gate|up GEMM output gu [rows][ldg]
 * (gate columns, then up columns), out [rows][ldo], bf16, inter even. */
EGPT_API int egpt_silu_mul(void *out, int64_t ldo, const void *gu, int64_t ldg, int64_t rows, int64_t inter,
                           void *stream);

/* ---- stochastic sampling: temperature -> top-k -> top-p -> inverse CDF -------------------------------
 * replaces: filtered_probs + sample_from (research/phase5/sampling.py:39-71; the Triton families
 * temperature_softmax / topk_softmax / inverse_cdf_sample of research/kernelagent/templates.py:131-343).
 * One token per row of `rows` x V logits (V <= 2^24; bf16 or fp32, leading dimension ld): x = logit / temperature; top_k > 0
 * keeps x >= the k-th largest x (ties kept; 0 = off); top_p < 1 keeps the smallest prefix of the stable descending
 * order of softmax(x) whose exclusive prefix mass stays below top_p, then renormalises (1 = off); the token is the
 * first index whose cumulative probability exceeds u * total, never a zero-probability token. u for row r is
 * u[r * u_ld + (u_index ? *u_index : 0)]; with u_index the call adds 1 to *u_index after drawing (one uniform per
 * generated token, as the reference's pre-drawn uniforms). Result in out[r * out_ld] (int64).
 * Workspace: egpt_sample_ws_bytes(rows) bytes, 16-byte aligned, zero-filled once by the caller; every call leaves
 * it zeroed. Deterministic (integer histograms and fixed-order sums). Errors: temperature <= 0, top_k < 0 or top_p
 * outside (0, 1] -> EGPT_ERR_ARG with the reference's messages. */
EGPT_API size_t egpt_sample_ws_bytes(int64_t rows);
EGPT_API int egpt_sample(const void *logits, int dtype, int64_t rows, int64_t V, int64_t ld, float temperature,
                         int64_t top_k, float top_p, const float *u, int64_t u_ld, int64_t *u_index, int64_t *out,
                         int64_t out_ld, void *ws, size_t ws_bytes, void *stream);

/* ---- whole decode step (Qwen3 family) ---------------------------------------------------------------
 * replaces: research/realmodel/fast_decode.py:45-49 GraphGreedyDecoder._step (HF Qwen3 forward with
 *           StaticCache + argmax + position += 1), captured into one CUDA graph by the caller.
 * Launches 5 kernels per layer + the lm_head/argmax kernel (the GEMVs on the exact tensor-core kernel,
 * EGPT_FLAG_EXACT, when the shapes and pointers allow it). Reads *token and *position on the device,
 * writes the next token to *token and increments *position. */
typedef struct egpt_qwen3_layer {
  const int8_t *w_qkv;  /* [(nq + 2 nkv) d, hidden]: q_proj, k_proj, v_proj rows concatenated          */
  const void *s_qkv;    /* scales for w_qkv                                                             */
  const int8_t *w_o;    /* [hidden, nq d]                                                               */
  const void *s_o;
  const int8_t *w_gu;   /* [2 inter, hidden]: gate_proj rows then up_proj rows                          */
  const void *s_gu;
  const int8_t *w_down; /* [hidden, inter]                                                              */
  const void *s_down;
  const void *ln_in;    /* input_layernorm.weight, bf16 [hidden]                                        */
  const void *ln_post;  /* post_attention_layernorm.weight, bf16 [hidden]                               */
  const void *q_norm;   /* self_attn.q_norm.weight, bf16 [d]                                            */
  const void *k_norm;   /* self_attn.k_norm.weight, bf16 [d]                                            */
  void *k_cache;        /* bf16 [nkv][cap][d]                                                           */
  void *v_cache;        /* bf16 [nkv][cap][d]                                                           */
} egpt_qwen3_layer;

typedef struct egpt_qwen3_plan {
  int32_t n_layers, hidden, n_q_heads, n_kv_heads, head_dim, intermediate;
  int64_t vocab, cap;
  float eps, attn_scale;
  int32_t scale_dtype;          /* EGPT_F32 or EGPT_BF16                                                  */
  uint32_t flags;               /* EGPT_FLAG_PDL to chain the step's kernels with PDL                    */
  int32_t attn_max_split;
  const egpt_qwen3_layer *layers; /* host array of n_layers entries                                      */
  const void *embed;            /* bf16 [vocab, hidden]                                                   */
  const void *final_norm;       /* bf16 [hidden]                                                          */
  const int8_t *w_lm;           /* [vocab, hidden]                                                        */
  const void *s_lm;
  const void *rope_cos, *rope_sin; /* bf16 [cap][d/2]                                                     */
  int64_t *token, *position;    /* device int64 [1] each                                                  */
  void *h, *qkv, *attn, *act;   /* bf16 activations: [hidden], [(nq+2nkv) d], [nq d], [inter]             */
  void *logits;                 /* nullable bf16 [vocab]                                                  */
  void *attn_ws;
  size_t attn_ws_bytes;
  void *lm_ws;
  size_t lm_ws_bytes;
  /* used by egpt_decode_step_persistent only */
  const egpt_qwen3_layer *layers_dev; /* device copy of `layers`                                          */
  void *sync_ws;                /* egpt_step_sync_ws_bytes() bytes, zero-filled once (grid barrier state) */
  uint64_t *trace;              /* nullable: 5 + 15 * n_layers %globaltimer stamps (ns) written by CTA 0:
                                   [0] start, [1+2b] / [2+2b] arrival at / release from grid barrier b,
                                   [1+2B] lm_head stage done, [2+2B] token written, [3+2B] unused,
                                   [4+2B+k] stage k's input ready (k < B: the stage before barrier k+1;
                                   k = B: lm_head) (B = 5 * n_layers barriers)                            */
  /* tensor parallelism (egpt_decode_step_persistent only; tp_world 0 or 1 = one GPU). With tp_world > 1 the
     sizes n_q_heads, n_kv_heads, intermediate and vocab, the layer weights, lm_head and KV caches are this
     rank's shard (egpt_tp_* below); hidden, the embedding and the norms are whole.                        */
  int32_t tp_rank, tp_world;    /* world 2, 4 or 8; every rank runs the same step at the same epoch        */
  void *tp_xchg[8];             /* exchange region of every rank (egpt_tp_xchg_bytes(hidden) bytes, zero-
                                   filled before the first step), mapped in this process; [tp_rank] is own */
  void *h2;                     /* tp: second bf16 [hidden] residual buffer (the layer's two residual sums
                                   alternate between h and h2)                                            */
  /* used by egpt_decode_step_dataflow only */
  void *df_ws;                  /* egpt_dataflow_ws_bytes(plan) bytes, 256-byte aligned, zero-filled once, then
                                   egpt_dataflow_prepare(plan) before the first step                      */
  size_t df_ws_bytes;
} egpt_qwen3_plan;

EGPT_API int egpt_decode_step(const egpt_qwen3_plan *plan, void *stream);

/* Persistent variant of egpt_decode_step: the whole token in ONE cooperative kernel with one CTA per SM.
 * Every warp streams its share of every weight matrix of the step (16-row tiles in 256-column items)
 * through its own shared-memory ring (cp.async, 2 items in flight) across stage boundaries, while the CTAs
 * run the stages separated by bounded grid barriers. The GEMVs are exact: the stage input is staged as
 * fixed point (x = X 2^E, |X| < 2^30, four int8 digit planes), int8 tensor-core MMAs give exact int64 row
 * sums, and each row is rounded once (then scaled and rounded at the reference's bf16 points), so results
 * can differ from egpt_decode_step's fp32 sums in the last bits. Needs plan->layers_dev and plan->sync_ws;
 * after a device error (egpt_device_error) sync_ws and the workspaces must be zero-filled again. Built for
 * head_dim 128 with 2 or 4 q heads per kv head and head_dim 32 with 2; hidden and nq*d up to 6144, the
 * intermediate size up to 6144 (12288 with head_dim 128, 4 q heads per kv head and one GPU: the 8B shape), all
 * multiples of 16, vocab a multiple of 16; other shapes return EGPT_ERR_SHAPE.
 * egpt_decode_step_persistent_check runs the same host-side checks without launching anything. */
EGPT_API size_t egpt_step_sync_ws_bytes(void);
EGPT_API int egpt_decode_step_persistent(const egpt_qwen3_plan *plan, void *stream);
EGPT_API int egpt_decode_step_persistent_check(const egpt_qwen3_plan *plan);

/* Dataflow variant of egpt_decode_step_persistent (one GPU): the same arithmetic in ONE cooperative kernel with
 * one CTA per SM and no grid barrier. The last n_kv_heads CTAs run the attention of one kv head each (holding its
 * cached K/V rows in shared memory when they fit); every warp of the other CTAs streams its share of every weight
 * matrix of the step (16-row x 256-column items, each as two TMA tensor loads, no multicast, this GPU's memory)
 * through its own ring of shared-memory slots guarded by mbarriers, running ahead across stage boundaries. Every
 * stage output (q|k|v, attention, residual stream, act) is published as LL words in plan->df_ws (two bf16 values
 * and a 32-bit tag of step, layer and site in one 8-byte word); consumers poll the words of their input until
 * every tag matches, so data and readiness arrive together. Every wait is bounded (EGPT_ERR_TIMEOUT via
 * egpt_device_error). RMSNorm sums its bf16 squares in fp64 (exact in practice, independent of the thread
 * layout). egpt_dataflow_ws_bytes: size of plan->df_ws for this plan (step epoch and LL words; zero-filled once).
 * egpt_dataflow_prepare checks the plan and encodes the weights' tensor maps into a host-side cache keyed by
 * plan->df_ws and the weight pointers (call once after the weight pointers are set, before any stream capture;
 * the step re-encodes by itself when the pointers change). Built for head_dim 128 with 2 or 4 q heads per kv head
 * and head_dim 32 with 2; hidden, intermediate and nq*d multiples of 64 up to 7680, vocab a multiple of 16, at
 * most 56 layers; tp_world <= 1. egpt_decode_step_dataflow_check runs the host-side checks. */
EGPT_API size_t egpt_dataflow_ws_bytes(const egpt_qwen3_plan *plan);
EGPT_API int egpt_dataflow_prepare(const egpt_qwen3_plan *plan);
EGPT_API int egpt_decode_step_dataflow(const egpt_qwen3_plan *plan, void *stream);
EGPT_API int egpt_decode_step_dataflow_check(const egpt_qwen3_plan *plan);

/* ---- tensor-parallel decode step (2, 4 or 8 GPUs of one NVLink/NVSwitch box, one process per GPU) ------
 * No counterpart in the reference (its decode runs on one GPU): the Megatron-style split of the step.
 * Rank r of g holds q heads [r nq/g, (r+1) nq/g) with their kv heads (q|k|v rows, KV cache), the matching
 * columns of o_proj, gate/up rows and down_proj columns [r I/g, (r+1) I/g), and lm_head rows
 * [r V/g, (r+1) V/g). egpt_decode_step_persistent with plan->tp_world = g runs the whole token in one kernel
 * per GPU: after o_proj and down_proj every CTA stores its rows' exact partial sums (fp64, unscaled) into
 * every rank's exchange region over NVLink (plain peer stores, no multicast) as 16-byte LL slots (two
 * 8-byte words, each a 32-bit sequence number above 32 payload bits), and the next stage on every rank
 * waits for the slots it reads, adds the g partials in rank order, scales, rounds and adds the residual as
 * the one-GPU step does (no grid barrier after those two stages). The lm_head stage exchanges one
 * (logit, index) key per rank the same way; every rank writes the same token. All waits are bounded
 * (EGPT_ERR_TIMEOUT via egpt_device_error). The exchange region holds key slots [8] and partial-sum slots
 * [2][8][hidden]; trace stamps (plan->trace) then cover the 3 * n_layers grid barriers that remain.
 * egpt_tp_xchg_alloc: cudaMalloc + zero fill of one region on the current device (free with
 * egpt_tp_xchg_free). egpt_ipc_handle writes the 64-byte CUDA IPC handle of such a region; egpt_ipc_open
 * maps a peer's handle into this process (peer access enabled), egpt_ipc_close unmaps it. */
EGPT_API size_t egpt_tp_xchg_bytes(int64_t hidden);
EGPT_API int egpt_tp_xchg_alloc(void **ptr, size_t bytes);
EGPT_API int egpt_tp_xchg_free(void *ptr);
EGPT_API int egpt_ipc_handle(const void *ptr, void *handle64);
EGPT_API int egpt_ipc_open(const void *handle64, void **ptr);
EGPT_API int egpt_ipc_close(void *ptr);

#ifdef __cplusplus
}
#endif

#endif /* EGPT_B200_H */
