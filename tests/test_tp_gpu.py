"""GPU: the tensor-parallel persistent step (one process per GPU, partial sums exchanged over NVLink inside the
kernel) against the one-GPU persistent step, and its bounded flag waits. The multi-GPU cases run when the box
has 2 or more GPUs; the rest need one."""
import os
import socket

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import parity
from oracle.bf16 import from_torch

pytestmark = pytest.mark.gpu


def _config(world):
    """tiny_config (head_dim 32, 2 kv heads) for 2 ranks; a head_dim-128 model with 8 kv heads for 4 and 8."""
    c = gi.tiny_config()
    if world > 2:
        from transformers import Qwen3Config
        c = Qwen3Config(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                        num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=256,
                        tie_word_embeddings=True, initializer_range=0.05)
    return c


def _model(world, device):
    from efficientgpt_b200.int8_linear import quantize_model
    model = gi.build_model(_config(world)).to(device)
    quantize_model(model, scale_dtype=torch.bfloat16)
    return model


def _run(eng, prompt, n_new):
    """Prompt token by token, then n_new greedy steps; tokens and this rank's bf16 logits per generated token."""
    toks, logs = [], []
    eng.feed(prompt)
    for i in range(n_new):
        toks.append(int(eng.token.item()))
        logs.append(from_torch(eng.logits.float()).copy())
        if i < n_new - 1:
            eng.step()
    return toks, logs


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_new, out):
    import torch.distributed as dist
    from efficientgpt_b200 import tp
    from efficientgpt_b200._lib import device_error
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)  # IPC handles and barriers only
    eng = None
    try:
        dev = torch.device('cuda', rank)
        model = _model(world, dev)
        shape = tp.Qwen3Shape.from_config(model.config)
        full = tp.full_weights(model)
        eng = tp.TPQwen3Engine(shape, tp.shard(full, shape, rank, world), rank, world, 96, keep_logits=True)
        prompt = gi.tiny_prompts()[37].to(dev) % shape.vocab
        toks, logs = _run(eng, prompt, n_new)
        err = device_error()
        res = {'tokens': toks, 'logits': logs, 'err': err}
        if rank == 0:  # the one-GPU persistent step on the whole model, same token-by-token feed
            one = tp.TPQwen3Engine(shape, full, 0, 1, 96, keep_logits=True)
            assert one.persistent
            res['one_tokens'], res['one_logits'] = _run(one, prompt, n_new)
        out[rank] = res
    finally:
        if eng is not None:
            eng.close()
        dist.destroy_process_group()


def _world():
    n = torch.cuda.device_count()
    return max(w for w in (1, 2, 4, 8) if w <= n)


@pytest.mark.parametrize('world', [2, 4, 8])
def test_tp_step_matches_one_gpu_step(cuda, world):
    if _world() < world:
        pytest.skip(f'needs {world} GPUs, the box has {torch.cuda.device_count()}')
    import torch.multiprocessing as mp
    n_new = 48
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), n_new, out), nprocs=world, join=True,
                           start_method='spawn')
        res = dict(out)
    assert all(res[r]['err'] == 0 for r in range(world)), [res[r]['err'] for r in range(world)]
    for r in range(1, world):
        assert res[r]['tokens'] == res[0]['tokens'], f'rank {r} wrote another token'
    want_t, want_l = res[0]['one_tokens'], res[0]['one_logits']
    got_t = res[0]['tokens']
    margins = [float(np.sort(l)[-1] - np.sort(l)[-2]) for l in want_l]
    tops = [float(l.max()) for l in want_l]
    ok, first, detail = parity.near_tie_match(want_t, margins, tops, got_t)
    assert ok, detail
    exact = 0
    for i in range(n_new if first is None else first):
        got_l = np.concatenate([res[r]['logits'][i] for r in range(world)])
        close, det = parity.logits_close(got_l, want_l[i])
        assert close, (i, det)
        exact += int(np.array_equal(got_l, want_l[i]))
    # the partial sums are exact (fp64) and added in rank order: almost every logit row is the one-GPU row
    assert exact >= 0.9 * (n_new if first is None else first), exact


def test_tp_world_one_is_the_one_gpu_step(cuda):
    """TPQwen3Engine(world 1) = Qwen3Engine's persistent step on the same weights (same kernel, same tokens)."""
    from efficientgpt_b200 import tp
    from efficientgpt_b200.engine import Qwen3Engine
    model = _model(2, cuda)
    shape = tp.Qwen3Shape.from_config(model.config)
    one = tp.TPQwen3Engine(shape, tp.full_weights(model), 0, 1, 96, keep_logits=True)
    ref = Qwen3Engine(model, 96, keep_logits=True)
    assert one.persistent and ref.persistent
    prompt = gi.tiny_prompts()[5].to(cuda)
    a = _run(one, prompt, 24)
    ref.position.zero_()
    for t in prompt.reshape(-1):
        ref.token.fill_(int(t))
        ref.step()
    b_t = []
    for i in range(24):
        b_t.append(int(ref.token.item()))
        if i < 23:
            ref.step()
    assert a[0] == b_t


def test_tp_flag_wait_times_out_and_reports(cuda):
    """A rank-0 step of a 2-way split whose peer region is never serviced: every flag wait gives up after its
    bound, the kernel returns, egpt_device_error reports EGPT_ERR_TIMEOUT and the context stays usable."""
    import ctypes
    from efficientgpt_b200 import _lib as L
    from efficientgpt_b200 import tp
    lib = L.load()
    model = _model(2, cuda)
    shape = tp.Qwen3Shape.from_config(model.config)
    full = tp.full_weights(model)
    nbytes = lib.egpt_tp_xchg_bytes(shape.hidden)
    regions = []
    for _ in range(2):
        p = ctypes.c_void_p()
        L.check(lib.egpt_tp_xchg_alloc(ctypes.byref(p), nbytes), 'tp_xchg_alloc')
        regions.append(p.value)
    try:
        eng = tp.TPQwen3Engine(shape, tp.shard(full, shape, 0, 2), 0, 2, 96, exchange=regions)
        assert L.device_error() == 0
        eng.token.fill_(3)
        eng.step()
        assert L.device_error(clear=True) == L.EGPT_ERR_TIMEOUT
        # the context still works: a fresh one-GPU engine decodes normally
        one = tp.TPQwen3Engine(shape, full, 0, 1, 96)
        one.token.fill_(3)
        one.step()
        assert L.device_error() == 0 and 0 <= int(one.token.item()) < shape.vocab
    finally:
        for p in regions:
            lib.egpt_tp_xchg_free(ctypes.c_void_p(p))
