"""Native batch-1 decode engine for transformers Qwen3 models quantised with `quantize_model`.

Everything per token runs in libegpt_b200.so: `step()` is one C-ABI call that reads the current token and
position from device memory and writes the next ones; the caller captures it in one CUDA graph. Three steps
with the same arithmetic: egpt_decode_step_dataflow (default: one cooperative kernel, a TMA-fed weight ring per
SM, stage outputs exchanged as tagged LL words, no grid barrier), egpt_decode_step_persistent (one cooperative
kernel with grid barriers; also the tensor-parallel step) and egpt_decode_step (5 kernels per layer plus the
fused final-RMSNorm/lm_head/argmax kernel).

HBM layout (all owned here, allocated once):
  w_qkv [(nq+2nkv)d, H] int8  q_proj|k_proj|v_proj rows;   w_gu [2I, H] int8  gate_proj|up_proj rows
  (the model's Int8Linear buffers are re-pointed to views of these, so weights are not duplicated)
  kv    [L, 2, nkv, cap, d] bf16  per layer and head one contiguous key stream (and value stream)
  rope  cos/sin [cap, d/2] bf16  HF's own table (model.model.rotary_emb), computed once on the device
  state token, position int64 [1]; activations h [H], qkv, attn [nq d], act [I] bf16; small workspaces

Prefill (`prefill`) reproduces the reference's eager HF forward over the prompt with the same kernels run on
row blocks: the op's >16-row branch rounding for prompts longer than 16 tokens, causal attention per row, and
the lm_head on the last row only (int8_linear.py:88-98, modeling_qwen3.py:503-505).
"""
import ctypes
import math

import torch

from . import _lib as L
from . import ops
from .int8_linear import Int8Linear


PREFILL_GEMM_MIN = 16  # prompts longer than this take the GEMM prefill (the op's own branch point, > 16 rows)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _fused(parts):
    """The row-concatenation of `parts` (same dtype, device and trailing shape). When they already sit back to back
    in one storage (views made by an earlier engine) the result is a view of it, else a new contiguous tensor."""
    first = parts[0]
    rows = sum(p.shape[0] for p in parts)
    shape = (rows,) + tuple(first.shape[1:])
    adjacent = all(p.is_contiguous() for p in parts) and all(
        p.untyped_storage().data_ptr() == first.untyped_storage().data_ptr() for p in parts)
    if adjacent:
        off = first.storage_offset()
        for p in parts:
            if p.storage_offset() != off:
                adjacent = False
                break
            off += p.numel()
    if adjacent:
        return torch.empty(0, dtype=first.dtype, device=first.device).set_(
            first.untyped_storage(), first.storage_offset(), shape, torch.empty(shape, device='meta').stride())
    return torch.cat(parts).contiguous()


class Qwen3Engine:
    def __init__(self, model, max_cache_len, pdl=True, attn_max_split=None, keep_logits=False, persistent=None,
                 step=None):
        """step: 'dataflow' (egpt_decode_step_dataflow: one cooperative kernel per token, TMA weight ring, LL
        activation exchange, no grid barrier), 'persistent' (egpt_decode_step_persistent: one cooperative kernel
        with grid barriers), 'sequence' (egpt_decode_step: per-stage launches), or None: the first of these the
        model's shapes allow. persistent=False is step='sequence'; persistent=True asks for a one-kernel step
        (dataflow when it fits, else persistent)."""
        if not torch.cuda.is_available():
            raise RuntimeError('Qwen3Engine needs a CUDA device (there is no CPU path)')
        self.model = model
        c = model.config
        self.device = next(model.parameters()).device
        if self.device.type != 'cuda':
            raise ValueError('the model must be on a CUDA device')
        self.n_layers = c.num_hidden_layers
        self.hidden = c.hidden_size
        self.nq = c.num_attention_heads
        self.nkv = c.num_key_value_heads
        self.d = getattr(c, 'head_dim', None) or c.hidden_size // c.num_attention_heads
        self.inter = c.intermediate_size
        self.vocab = c.vocab_size
        self.eps = float(c.rms_norm_eps)
        self.cap = int(max_cache_len)
        self.scale = self.d ** -0.5
        inner = model.model
        lins = []
        for blk in inner.layers:
            a, m = blk.self_attn, blk.mlp
            group = [a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj, m.down_proj]
            if not all(isinstance(x, Int8Linear) for x in group):
                raise ValueError('Qwen3Engine needs a model quantised with efficientgpt_b200.quantize_model')
            if any(x.bias is not None for x in group):
                raise ValueError('biased projections are not supported by the Qwen3 decode step')
            lins.append(group)
        if not isinstance(model.lm_head, Int8Linear):
            raise ValueError('lm_head must be quantised (quantize_model(include_lm_head=True))')
        sdt = lins[0][0].scale.dtype
        if any(x.scale.dtype != sdt for g in lins for x in g) or model.lm_head.scale.dtype != sdt:
            raise ValueError('all scales must share one dtype')
        self.scale_dtype = L.EGPT_BF16 if sdt == torch.bfloat16 else L.EGPT_F32

        # ---- weights: fuse q|k|v and gate|up, re-point the modules' buffers to views (no duplicate copy; a second
        #      engine on the same model finds the buffers already fused and shares them)
        self.layers = []
        for blk, (q, k, v, o, g, u, dn) in zip(inner.layers, lins):
            w_qkv = _fused([q.qweight, k.qweight, v.qweight])
            s_qkv = _fused([q.scale, k.scale, v.scale])
            w_gu = _fused([g.qweight, u.qweight])
            s_gu = _fused([g.scale, u.scale])
            r0 = 0
            for lin in (q, k, v):
                n = lin.qweight.shape[0]
                lin.qweight, lin.scale = w_qkv[r0:r0 + n], s_qkv[r0:r0 + n]
                r0 += n
            g.qweight, g.scale = w_gu[:self.inter], s_gu[:self.inter]
            u.qweight, u.scale = w_gu[self.inter:], s_gu[self.inter:]
            self.layers.append({'w_qkv': w_qkv, 's_qkv': s_qkv, 'w_o': o.qweight, 's_o': o.scale, 'w_gu': w_gu,
                                's_gu': s_gu, 'w_down': dn.qweight, 's_down': dn.scale,
                                'ln_in': blk.input_layernorm.weight, 'ln_post': blk.post_attention_layernorm.weight,
                                'q_norm': blk.self_attn.q_norm.weight, 'k_norm': blk.self_attn.k_norm.weight})
        for lay in self.layers:
            for key in ('ln_in', 'ln_post', 'q_norm', 'k_norm'):
                if lay[key].dtype != torch.bfloat16:
                    raise ValueError('norm weights must be bf16')
        self.embed = inner.embed_tokens.weight
        self.final_norm = inner.norm.weight
        self.w_lm, self.s_lm = model.lm_head.qweight, model.lm_head.scale
        if self.embed.dtype != torch.bfloat16:
            raise ValueError('the model must be bf16 (model.to(torch.bfloat16))')

        dev = self.device
        with torch.no_grad():
            pos = torch.arange(self.cap, device=dev)[None]
            cos, sin = inner.rotary_emb(self.embed[:1], pos)  # HF's own table, on the device, model dtype
        half = self.d // 2
        self.rope_cos = cos[0, :, :half].to(torch.bfloat16).contiguous()
        self.rope_sin = sin[0, :, :half].to(torch.bfloat16).contiguous()

        self.kv = torch.zeros((self.n_layers, 2, self.nkv, self.cap, self.d), dtype=torch.bfloat16, device=dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.position = torch.zeros(1, dtype=torch.int64, device=dev)
        nqkv = (self.nq + 2 * self.nkv) * self.d
        self.h = torch.zeros(self.hidden, dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros(nqkv, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros(self.nq * self.d, dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros(self.inter, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(self.vocab, dtype=torch.bfloat16, device=dev) if keep_logits else None
        nsm = L.load().egpt_num_sms()
        self.attn_max_split = attn_max_split or max(1, min(64, nsm // self.nkv))
        self.attn_ws = ops.attn_ws(1, self.nq, self.nkv, self.d, self.attn_max_split, dev)
        self.lm_ws = ops.lm_head_ws(self.vocab, dev)
        self.sync_ws = torch.zeros(int(L.load().egpt_step_sync_ws_bytes()), dtype=torch.uint8, device=dev)
        self.pdl = pdl
        self.df_ws = None
        self._build_plan()
        lib = L.load()
        fits_v1 = self.vocab // 2 >= nsm and lib.egpt_decode_step_persistent_check(ctypes.byref(self.plan)) == 0
        msg_v1 = L.last_error()
        fits_df = lib.egpt_decode_step_dataflow_check(ctypes.byref(self.plan)) == 0
        msg_df = L.last_error()
        if step is None and persistent is False:
            step = 'sequence'
        if step is None:
            step = 'dataflow' if fits_df else 'persistent' if fits_v1 else 'sequence'
            if persistent and step == 'sequence':
                raise ValueError('no one-kernel decode step is built for this model shape: ' + msg_v1)
        if step not in ('dataflow', 'persistent', 'sequence'):
            raise ValueError(f'unknown step {step!r}')
        if step == 'dataflow' and not fits_df:
            raise ValueError('the dataflow decode step is not built for this model shape: ' + msg_df)
        if step == 'persistent' and not fits_v1:
            raise ValueError('the persistent decode step is not built for this model shape: ' + msg_v1)
        self.step_kind = step
        self.persistent = step != 'sequence'
        if step == 'dataflow':
            L.check(lib.egpt_dataflow_prepare(ctypes.byref(self.plan)), 'dataflow_prepare')

    def _build_plan(self):
        arr = (L.Qwen3Layer * self.n_layers)()
        for i, lay in enumerate(self.layers):
            e = arr[i]
            for f in ('w_qkv', 's_qkv', 'w_o', 's_o', 'w_gu', 's_gu', 'w_down', 's_down', 'ln_in', 'ln_post', 'q_norm',
                      'k_norm'):
                setattr(e, f, lay[f].data_ptr())
            e.k_cache = self.kv[i, 0].data_ptr()
            e.v_cache = self.kv[i, 1].data_ptr()
        p = L.Qwen3Plan()
        p.n_layers, p.hidden, p.n_q_heads, p.n_kv_heads = self.n_layers, self.hidden, self.nq, self.nkv
        p.head_dim, p.intermediate, p.vocab, p.cap = self.d, self.inter, self.vocab, self.cap
        p.eps, p.attn_scale, p.scale_dtype = self.eps, self.scale, self.scale_dtype
        p.flags = L.FLAG_PDL if self.pdl else 0
        p.attn_max_split = self.attn_max_split
        p.layers = arr
        p.embed, p.final_norm = self.embed.data_ptr(), self.final_norm.data_ptr()
        p.w_lm, p.s_lm = self.w_lm.data_ptr(), self.s_lm.data_ptr()
        p.rope_cos, p.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
        p.token, p.position = self.token.data_ptr(), self.position.data_ptr()
        p.h, p.qkv, p.attn, p.act = self.h.data_ptr(), self.qkv.data_ptr(), self.attn.data_ptr(), self.act.data_ptr()
        p.logits = self.logits.data_ptr() if self.logits is not None else None
        p.attn_ws, p.attn_ws_bytes = self.attn_ws.data_ptr(), self.attn_ws.numel()
        p.lm_ws, p.lm_ws_bytes = self.lm_ws.data_ptr(), self.lm_ws.numel()
        raw = bytes(memoryview(arr).cast('B'))
        self.layers_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
        p.layers_dev = self.layers_dev.data_ptr()
        p.sync_ws = self.sync_ws.data_ptr()
        nbytes = int(L.load().egpt_dataflow_ws_bytes(ctypes.byref(p)))
        self.df_ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        p.df_ws, p.df_ws_bytes = self.df_ws.data_ptr(), nbytes
        self._layer_arr = arr  # keep alive
        self.plan = p

    # ------------------------------------------------------------------------------------------ decode
    def step(self):
        """One decode token on the current stream: token <- argmax(model(token, position)); position += 1."""
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if self.step_kind == 'dataflow':
            L.check(L.load().egpt_decode_step_dataflow(ctypes.byref(self.plan), stream), 'decode_step_dataflow')
        elif self.step_kind == 'persistent':
            L.check(L.load().egpt_decode_step_persistent(ctypes.byref(self.plan), stream), 'decode_step_persistent')
        else:
            L.check(L.load().egpt_decode_step(ctypes.byref(self.plan), stream), 'decode_step')

    # ------------------------------------------------------------------------------------------ prefill
    def _linear(self, x, w, s, **kw):
        return ops.gemv_i8_rows(x, w, s, double_round=x.shape[0] > ops.MAX_KERNEL_ROWS, **kw)

    @torch.no_grad()
    def prefill(self, input_ids):
        """Run the prompt (int64 [p] or [1, p] on the device) from position 0; leaves token = first generated id
        and position = p. Returns the token tensor (device). Prompts longer than PREFILL_GEMM_MIN tokens (the
        reference op's >16-row branch) run the GEMM prefill (efficientgpt_b200.prefill: tcgen05 projections with
        the >16-row rounding, the tcgen05 causal attention kernel over the prompt) up to the last row's hidden state, then the final norm and the
        lm_head argmax on that row; shorter ones run the per-stage kernels on one block of rows."""
        ids = input_ids.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        p = ids.numel()
        if p < 1 or p > self.cap:
            raise ValueError('prompt length must be in [1, max_cache_len]')
        if p > PREFILL_GEMM_MIN:
            from .prefill import fill_kv
            h_last = fill_kv(ids, self.layers, self.embed, self.kv, self.rope_cos, self.rope_sin, self.nq, self.nkv,
                             self.d, self.eps, last_hidden=True)
            ops.lm_head_argmax(h_last[0], self.w_lm, self.s_lm, self.lm_ws, norm_w=self.final_norm, eps=self.eps,
                               logits=self.logits, token=self.token, exact=True)
            self.position.fill_(p)
            return self.token
        self.position.zero_()
        h = ops.embed(ids, self.embed)
        ws = ops.attn_ws(p, self.nq, self.nkv, self.d, self.attn_max_split, self.device)
        for i, lay in enumerate(self.layers):
            x = ops.rmsnorm(h, lay['ln_in'], self.eps)
            qkv = self._linear(x, lay['w_qkv'], lay['s_qkv'])
            q = ops.qk_norm_rope_kv_append(qkv, self.kv[i, 0], self.kv[i, 1], self.position, self.nq, self.nkv, self.d,
                                           q_norm_w=lay['q_norm'], k_norm_w=lay['k_norm'], eps=self.eps,
                                           rope_cos=self.rope_cos, rope_sin=self.rope_sin)
            a = ops.attn_decode(q, self.kv[i, 0], self.kv[i, 1], self.position, self.nq, self.nkv, self.d,
                                scale=self.scale, max_split=self.attn_max_split, ws=ws, ref_softmax=True)
            h = self._linear(a, lay['w_o'], lay['s_o'], epilogue=L.EPI_RESIDUAL, residual=h)
            x = ops.rmsnorm(h, lay['ln_post'], self.eps)
            act = self._linear(x, lay['w_gu'], lay['s_gu'], epilogue=L.EPI_SILU_MUL)
            h = self._linear(act, lay['w_down'], lay['s_down'], epilogue=L.EPI_RESIDUAL, residual=h)
        ops.lm_head_argmax(h[p - 1], self.w_lm, self.s_lm, self.lm_ws, norm_w=self.final_norm, eps=self.eps,
                           logits=self.logits, token=self.token, exact=True)
        self.position.fill_(p)
        return self.token

    def reset(self):
        """Forget the sequence (the next prefill starts at position 0; stale cache slots are never read)."""
        self.position.zero_()
        self.token.zero_()

    # ------------------------------------------------------------------------------------------ accounting
    def weight_bytes(self):
        """Bytes of weights one decode step streams (int8 matrices, scales, norms, one embedding row)."""
        b = 0
        for lay in self.layers:
            for k in ('w_qkv', 's_qkv', 'w_o', 's_o', 'w_gu', 's_gu', 'w_down', 's_down', 'ln_in', 'ln_post', 'q_norm',
                      'k_norm'):
                b += lay[k].numel() * lay[k].element_size()
        b += self.w_lm.numel() + self.s_lm.numel() * self.s_lm.element_size()
        b += self.final_norm.numel() * 2 + self.hidden * 2
        return b

    def kv_bytes_per_token(self, ctx):
        """KV-cache bytes one decode step reads at context length ctx (all layers, K and V)."""
        return self.n_layers * 2 * self.nkv * ctx * self.d * 2
