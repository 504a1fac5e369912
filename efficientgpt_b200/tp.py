"""Tensor-parallel batch-1 decode of Qwen3-family models on 2, 4 or 8 GPUs of one box (one process per GPU).

No counterpart in the reference (its decode runs on one GPU); the split is the Megatron one of the linear layers:
rank r of g holds q heads [r nq/g, (r+1) nq/g) with their kv heads (q|k|v rows of `w_qkv`, its KV cache), the
matching columns of o_proj, gate/up rows and down_proj columns [r I/g, (r+1) I/g), and lm_head rows
[r V/g, (r+1) V/g); the embedding and the norms are whole. The quantisation is the one-GPU model's (per output
row over the whole row), so a shard's int8 values and scales are slices of the one-GPU tensors.

Each token is ONE launch per GPU of the persistent step (egpt_decode_step_persistent with tp_world = g): the
o_proj / down_proj partial sums cross NVLink inside the kernel (peer stores of sequence-tagged slots into every
rank's exchange region; the consuming stage waits, bounded, on the slots themselves), with no collective call on
the path. Prompts longer than 64 tokens fill the KV cache with the GEMM prefill (efficientgpt_b200.prefill). The exchange regions are allocated by the library
(cudaMalloc: CUDA IPC exports whole allocations) and mapped into every rank with CUDA IPC handles passed
over the process group. torch.distributed is only the plumbing that moves those handles and the barriers
around set-up and tear-down.

HBM layout per rank: the shard's fused weights (`w_qkv` [(nq/g + 2 nkv/g) d, H], `w_o` [H, nq d / g],
`w_gu` [2 I/g, H], `w_down` [H, I/g], `w_lm` [V/g, H]), KV cache [L, 2, nkv/g, cap, d] bf16, two bf16 [H]
residual buffers, the exchange region (4 KB of lm_head key slots + fp64 partial-sum slots [2][8][H], 16 bytes each).
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from . import ops
from .int8_linear import Int8Linear

LAYER_KEYS = ('w_qkv', 's_qkv', 'w_o', 's_o', 'w_gu', 's_gu', 'w_down', 's_down', 'ln_in', 'ln_post', 'q_norm',
              'k_norm')


@dataclass
class Qwen3Shape:
    n_layers: int
    hidden: int
    nq: int
    nkv: int
    d: int
    inter: int
    vocab: int
    eps: float
    rope_theta: float

    @classmethod
    def from_config(cls, c):
        return cls(c.num_hidden_layers, c.hidden_size, c.num_attention_heads, c.num_key_value_heads,
                   getattr(c, 'head_dim', None) or c.hidden_size // c.num_attention_heads, c.intermediate_size,
                   c.vocab_size, float(c.rms_norm_eps), float(getattr(c, 'rope_theta', None) or
                                                               c.rope_parameters['rope_theta']))


def full_weights(model):
    """The fused one-GPU weights of a model quantised with quantize_model: per layer q|k|v rows and gate|up rows
    concatenated (the layout of Qwen3Engine), plus embedding, final norm and lm_head."""
    inner = model.model
    layers = []
    for blk in inner.layers:
        a, m = blk.self_attn, blk.mlp
        lins = (a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj, m.down_proj)
        if not all(isinstance(x, Int8Linear) for x in lins):
            raise ValueError('tensor parallelism needs a model quantised with efficientgpt_b200.quantize_model')
        if any(x.bias is not None for x in lins):
            raise ValueError('biased projections are not supported by the Qwen3 decode step')
        q, k, v, o, g, u, dn = lins
        layers.append({'w_qkv': torch.cat([q.qweight, k.qweight, v.qweight]), 's_qkv': torch.cat([q.scale, k.scale, v.scale]),
                       'w_o': o.qweight, 's_o': o.scale, 'w_gu': torch.cat([g.qweight, u.qweight]),
                       's_gu': torch.cat([g.scale, u.scale]), 'w_down': dn.qweight, 's_down': dn.scale,
                       'ln_in': blk.input_layernorm.weight, 'ln_post': blk.post_attention_layernorm.weight,
                       'q_norm': a.q_norm.weight, 'k_norm': a.k_norm.weight})
    if not isinstance(model.lm_head, Int8Linear):
        raise ValueError('lm_head must be quantised (quantize_model(include_lm_head=True))')
    return {'layers': layers, 'embed': inner.embed_tokens.weight, 'final_norm': inner.norm.weight,
            'w_lm': model.lm_head.qweight, 's_lm': model.lm_head.scale, 'rotary': inner.rotary_emb}


def check_shardable(shape, world):
    """Raise ValueError unless `shape` splits evenly over `world` ranks (whole kv-head groups, 16-row tiles)."""
    if world not in (1, 2, 4, 8):
        raise ValueError('tensor parallelism runs on 1, 2, 4 or 8 GPUs')
    if shape.nkv % world or shape.nq % world:
        raise ValueError(f'{shape.nkv} kv heads / {shape.nq} q heads do not split over {world} ranks')
    if shape.inter % (16 * world) or shape.vocab % (16 * world):
        raise ValueError(f'intermediate {shape.inter} and vocab {shape.vocab} must split into 16-row tiles per rank')


def shard(full, shape, rank, world):
    """Rank `rank`'s shard of the fused one-GPU weights (new contiguous tensors; inputs are not modified)."""
    check_shardable(shape, world)
    if not 0 <= rank < world:
        raise ValueError('rank out of range')
    d, nq, nkv, inter, V = shape.d, shape.nq, shape.nkv, shape.inter, shape.vocab
    nq_l, nkv_l, i_l, v_l = nq // world, nkv // world, inter // world, V // world
    q0, k0, v0 = rank * nq_l * d, nq * d + rank * nkv_l * d, (nq + nkv) * d + rank * nkv_l * d
    rows_qkv = (slice(q0, q0 + nq_l * d), slice(k0, k0 + nkv_l * d), slice(v0, v0 + nkv_l * d))
    rows_gu = (slice(rank * i_l, (rank + 1) * i_l), slice(inter + rank * i_l, inter + (rank + 1) * i_l))
    cols_o = slice(rank * nq_l * d, (rank + 1) * nq_l * d)
    cols_down = slice(rank * i_l, (rank + 1) * i_l)
    layers = []
    for lay in full['layers']:
        layers.append({
            'w_qkv': torch.cat([lay['w_qkv'][r] for r in rows_qkv]).contiguous(),
            's_qkv': torch.cat([lay['s_qkv'][r] for r in rows_qkv]).contiguous(),
            'w_o': lay['w_o'][:, cols_o].contiguous(), 's_o': lay['s_o'].clone(),
            'w_gu': torch.cat([lay['w_gu'][r] for r in rows_gu]).contiguous(),
            's_gu': torch.cat([lay['s_gu'][r] for r in rows_gu]).contiguous(),
            'w_down': lay['w_down'][:, cols_down].contiguous(), 's_down': lay['s_down'].clone(),
            'ln_in': lay['ln_in'].clone(), 'ln_post': lay['ln_post'].clone(),
            'q_norm': lay['q_norm'].clone(), 'k_norm': lay['k_norm'].clone()})
    lm = slice(rank * v_l, (rank + 1) * v_l)
    out = {'layers': layers, 'embed': full['embed'].clone(), 'final_norm': full['final_norm'].clone(),
           'w_lm': full['w_lm'][lm].contiguous(), 's_lm': full['s_lm'][lm].contiguous()}
    if 'rotary' in full:
        out['rotary'] = full['rotary']
    return out


def rope_tables(shape, cap, device, rotary=None):
    """HF's RoPE table (transformers Qwen3RotaryEmbedding, computed on the device, bf16), first half of d. rotary:
    the model's own module (its inv_freq buffer is bf16 after model.to(torch.bfloat16)); None = a new module cast
    the same way."""
    rot = rotary
    if rot is None:
        from transformers import Qwen3Config
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
        cfg = Qwen3Config(hidden_size=shape.hidden, num_attention_heads=shape.nq, num_key_value_heads=shape.nkv,
                          head_dim=shape.d, rope_theta=shape.rope_theta, max_position_embeddings=max(cap, 1))
        with torch.device(device):
            rot = Qwen3RotaryEmbedding(config=cfg).to(torch.bfloat16)
    x = torch.zeros(1, dtype=torch.bfloat16, device=device)
    cos, sin = rot(x, torch.arange(cap, device=device)[None])
    half = shape.d // 2
    return cos[0, :, :half].to(torch.bfloat16).contiguous(), sin[0, :, :half].to(torch.bfloat16).contiguous()


class TPQwen3Engine:
    """One rank of the tensor-parallel decode step. Every rank of `group` constructs it with its own shard
    (`shard(full_weights(model), shape, rank, world)`) on its own GPU, then all ranks call step() / feed() in
    lockstep. With world 1 it is the one-GPU persistent step (or the launch sequence for shapes the persistent
    kernel is not built for)."""

    def __init__(self, shape, weights, rank, world, max_cache_len, group=None, keep_logits=False, attn_max_split=None,
                 exchange=None):
        """exchange: None = allocate this rank's exchange region and map the peers' over `group` (CUDA IPC);
        else a list of `world` device addresses of regions the caller has mapped (egpt_tp_xchg_bytes(hidden)
        bytes each, zero-filled), used as they are and never freed here."""
        if not torch.cuda.is_available():
            raise RuntimeError('TPQwen3Engine needs a CUDA device (there is no CPU path)')
        check_shardable(shape, world)
        self.shape, self.rank, self.world, self.group = shape, rank, world, group
        self.device = weights['w_lm'].device
        if self.device.type != 'cuda':
            raise ValueError('the shard must be on a CUDA device')
        self.lib = L.load()
        s = shape
        self.nq, self.nkv, self.inter, self.vocab = s.nq // world, s.nkv // world, s.inter // world, s.vocab // world
        self.cap = int(max_cache_len)
        self.w = weights
        sdt = weights['s_lm'].dtype
        self.scale_dtype = L.EGPT_BF16 if sdt == torch.bfloat16 else L.EGPT_F32
        dev = self.device
        with torch.no_grad():
            self.rope_cos, self.rope_sin = rope_tables(s, self.cap, dev, weights.get('rotary'))
        self.kv = torch.zeros((s.n_layers, 2, self.nkv, self.cap, s.d), dtype=torch.bfloat16, device=dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.position = torch.zeros(1, dtype=torch.int64, device=dev)
        self.h = torch.zeros(s.hidden, dtype=torch.bfloat16, device=dev)
        self.h2 = torch.zeros(s.hidden, dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros((self.nq + 2 * self.nkv) * s.d, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros(self.nq * s.d, dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros(self.inter, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(self.vocab, dtype=torch.bfloat16, device=dev) if keep_logits else None
        nsm = self.lib.egpt_num_sms()
        self.attn_max_split = attn_max_split or max(1, min(64, nsm // self.nkv))
        self.attn_ws = ops.attn_ws(1, self.nq, self.nkv, s.d, self.attn_max_split, dev)
        self.lm_ws = ops.lm_head_ws(self.vocab, dev)
        self.sync_ws = torch.zeros(int(self.lib.egpt_step_sync_ws_bytes()), dtype=torch.uint8, device=dev)
        self._own_xchg = None
        self._peers = []
        self._started = exchange is not None
        self._build_plan()
        if world > 1 and exchange is not None:
            if len(exchange) != world:
                raise ValueError('exchange needs one region per rank')
            for r, a in enumerate(exchange):
                self.plan.tp_xchg[r] = int(a)
        elif world > 1:
            self._map_exchange()
        self.persistent = self.lib.egpt_decode_step_persistent_check(ctypes.byref(self.plan)) == 0
        self.step_kind = 'persistent' if self.persistent else 'sequence'
        if world > 1 and not self.persistent:
            raise ValueError('the tensor-parallel step needs the persistent kernel: ' + L.last_error())

    def _build_plan(self):
        s = self.shape
        arr = (L.Qwen3Layer * s.n_layers)()
        for i, lay in enumerate(self.w['layers']):
            for f in LAYER_KEYS:
                setattr(arr[i], f, lay[f].data_ptr())
            arr[i].k_cache = self.kv[i, 0].data_ptr()
            arr[i].v_cache = self.kv[i, 1].data_ptr()
        p = L.Qwen3Plan()
        p.n_layers, p.hidden, p.n_q_heads, p.n_kv_heads = s.n_layers, s.hidden, self.nq, self.nkv
        p.head_dim, p.intermediate, p.vocab, p.cap = s.d, self.inter, self.vocab, self.cap
        p.eps, p.attn_scale, p.scale_dtype = s.eps, s.d ** -0.5, self.scale_dtype
        p.flags = L.FLAG_PDL
        p.attn_max_split = self.attn_max_split
        p.layers = arr
        p.embed, p.final_norm = self.w['embed'].data_ptr(), self.w['final_norm'].data_ptr()
        p.w_lm, p.s_lm = self.w['w_lm'].data_ptr(), self.w['s_lm'].data_ptr()
        p.rope_cos, p.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
        p.token, p.position = self.token.data_ptr(), self.position.data_ptr()
        p.h, p.qkv, p.attn, p.act = self.h.data_ptr(), self.qkv.data_ptr(), self.attn.data_ptr(), self.act.data_ptr()
        p.h2 = self.h2.data_ptr()
        p.logits = self.logits.data_ptr() if self.logits is not None else None
        p.attn_ws, p.attn_ws_bytes = self.attn_ws.data_ptr(), self.attn_ws.numel()
        p.lm_ws, p.lm_ws_bytes = self.lm_ws.data_ptr(), self.lm_ws.numel()
        raw = bytes(memoryview(arr).cast('B'))
        self.layers_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
        p.layers_dev = self.layers_dev.data_ptr()
        p.sync_ws = self.sync_ws.data_ptr()
        p.tp_rank, p.tp_world = (self.rank, self.world) if self.world > 1 else (0, 0)
        self._layer_arr = arr
        self.plan = p

    def _map_exchange(self):
        """Allocate this rank's exchange region, swap IPC handles over the group, map every peer's region."""
        import torch.distributed as dist
        lib = self.lib
        torch.cuda.synchronize(self.device)
        ptr = ctypes.c_void_p()
        L.check(lib.egpt_tp_xchg_alloc(ctypes.byref(ptr), lib.egpt_tp_xchg_bytes(self.shape.hidden)), 'tp_xchg_alloc')
        self._own_xchg = ptr.value
        handle = (ctypes.c_char * 64)()
        L.check(lib.egpt_ipc_handle(ctypes.c_void_p(self._own_xchg), handle), 'ipc_handle')
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        for r in range(self.world):
            if r == self.rank:
                self.plan.tp_xchg[r] = self._own_xchg
                continue
            peer = ctypes.c_void_p()
            L.check(lib.egpt_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(peer)), 'ipc_open')
            self._peers.append(peer.value)
            self.plan.tp_xchg[r] = peer.value
        dist.barrier(group=self.group)  # every region is zero-filled and mapped before any rank's first step

    # ------------------------------------------------------------------------------------------ decode
    def step(self):
        """One decode token on the current stream, on every rank in lockstep: token <- argmax(model(token,
        position)) (the same token on every rank); position += 1."""
        if self.world > 1 and not self._started:
            # the ranks' first kernels must start within the slot waits' bound of one another: line up first
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self._started = True
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        if self.persistent:
            L.check(self.lib.egpt_decode_step_persistent(ctypes.byref(self.plan), stream), 'decode_step_persistent')
        else:
            L.check(self.lib.egpt_decode_step(ctypes.byref(self.plan), stream), 'decode_step')

    @torch.no_grad()
    def feed(self, ids, gemm_min=64):
        """Run the prompt from position 0; leaves token = the first generated id and position = len(ids). Prompts
        longer than gemm_min tokens fill the KV cache of all but the last token with the GEMM prefill
        (efficientgpt_b200.prefill; o_proj / down_proj partial products summed over the group) and run the last
        token through the decode step; shorter ones go token by token through the decode step."""
        ids = ids.reshape(-1).to(device=self.device, dtype=torch.int64)
        p = ids.numel()
        if p < 1 or p > self.cap:
            raise ValueError('prompt length must be in [1, max_cache_len]')
        self.position.zero_()
        if p > gemm_min:
            from .prefill import fill_kv
            allreduce = None
            if self.world > 1:
                import torch.distributed as dist
                allreduce = lambda y: dist.all_reduce(y, group=self.group)
            fill_kv(ids[:-1].contiguous(), self.w['layers'], self.w['embed'], self.kv, self.rope_cos, self.rope_sin,
                    self.nq, self.nkv, self.shape.d, self.shape.eps, allreduce)
            self.position.fill_(p - 1)
            self.token.copy_(ids[-1:])
            self.step()
            return self.token
        for i in range(p):
            self.token.copy_(ids[i:i + 1])
            self.step()
        return self.token

    @torch.no_grad()
    def generate(self, ids, max_new_tokens):
        """Greedy tokens after the prompt (device-side loop; one host read at the end)."""
        if max_new_tokens < 1:
            raise ValueError('max_new_tokens must be >= 1')
        if ids.numel() + max_new_tokens > self.cap:
            raise ValueError('prompt + new tokens exceed max_cache_len')
        out = torch.empty(max_new_tokens, dtype=torch.int64, device=self.device)
        self.feed(ids)
        out[0:1].copy_(self.token)
        for i in range(1, max_new_tokens):
            self.step()
            out[i:i + 1].copy_(self.token)
        return out.tolist()

    def close(self):
        """Unmap the peers' regions and free this rank's (after a group barrier: no rank still uses them)."""
        if self.world > 1 and (self._peers or self._own_xchg):
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for p in self._peers:
                self.lib.egpt_ipc_close(ctypes.c_void_p(p))
            self._peers = []
            dist.barrier(group=self.group)
            if self._own_xchg:
                self.lib.egpt_tp_xchg_free(ctypes.c_void_p(self._own_xchg))
                self._own_xchg = None

    # ------------------------------------------------------------------------------------------ accounting
    def weight_bytes(self):
        """Bytes of weights this rank's step streams (its int8 shard, scales, norms, one embedding row)."""
        b = 0
        for lay in self.w['layers']:
            for k in LAYER_KEYS:
                b += lay[k].numel() * lay[k].element_size()
        b += self.w['w_lm'].numel() + self.w['s_lm'].numel() * self.w['s_lm'].element_size()
        return b + self.w['final_norm'].numel() * 2 + self.shape.hidden * 2

    def kv_bytes_per_token(self, ctx):
        """KV-cache bytes this rank's step reads at context length ctx."""
        return self.shape.n_layers * 2 * self.nkv * ctx * self.shape.d * 2
