"""Host side of the tensor-parallel decode (CPU): the product's shard() against the oracle's slicing, the argmax
key order, and the TP restatement of the decode step run as two gloo ranks against the one-rank oracle."""
import os
import socket

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import parity
from oracle.bf16 import round_bf16
from oracle.qwen3_ref import Qwen3Ref
from oracle.tp_ref import TPQwen3Ref, argmax_key, first_argmax, key_index


def _full_from_oracle(ref):
    """The product's fused one-GPU weight dict (tp.full_weights layout) from the oracle's quantised layers."""
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)) if dt is None else torch.from_numpy(
        np.ascontiguousarray(a)).to(dt)
    layers = []
    for L in ref.layers:
        layers.append({'w_qkv': t(np.concatenate([L['q'][0], L['k'][0], L['v'][0]])),
                       's_qkv': t(np.concatenate([L['q'][1], L['k'][1], L['v'][1]])),
                       'w_o': t(L['o'][0]), 's_o': t(L['o'][1]),
                       'w_gu': t(np.concatenate([L['gate'][0], L['up'][0]])),
                       's_gu': t(np.concatenate([L['gate'][1], L['up'][1]])),
                       'w_down': t(L['down'][0]), 's_down': t(L['down'][1]),
                       'ln_in': t(L['ln_in']), 'ln_post': t(L['ln_post']), 'q_norm': t(L['q_norm']),
                       'k_norm': t(L['k_norm'])})
    return {'layers': layers, 'embed': t(ref.embed), 'final_norm': t(ref.final_norm), 'w_lm': t(ref.lm_q),
            's_lm': t(ref.lm_s)}


def _shape(cfg):
    from efficientgpt_b200.tp import Qwen3Shape
    return Qwen3Shape.from_config(cfg)


def test_shard_matches_oracle_slices():
    from efficientgpt_b200.tp import shard
    cfg = gi.tiny_config()
    ref = Qwen3Ref.from_hf(gi.build_model(cfg), 64, 'fp32', semantics='cpu')
    full = _full_from_oracle(ref)
    shape = _shape(cfg)
    world = 2
    parts = [shard(full, shape, r, world) for r in range(world)]
    for r, p in enumerate(parts):
        o = TPQwen3Ref(ref, r, world, lambda a: [a])
        for L, S in zip(ref.layers, p['layers']):
            want = np.concatenate([L['q'][0][o.q_rows], L['k'][0][o.kv_rows], L['v'][0][o.kv_rows]])
            np.testing.assert_array_equal(S['w_qkv'].numpy(), want)
            np.testing.assert_array_equal(S['w_o'].numpy(), L['o'][0][:, o.q_rows])
            np.testing.assert_array_equal(S['s_o'].numpy(), L['o'][1])
            np.testing.assert_array_equal(S['w_gu'].numpy(),
                                          np.concatenate([L['gate'][0][o.i_rows], L['up'][0][o.i_rows]]))
            np.testing.assert_array_equal(S['s_gu'].numpy(),
                                          np.concatenate([L['gate'][1][o.i_rows], L['up'][1][o.i_rows]]))
            np.testing.assert_array_equal(S['w_down'].numpy(), L['down'][0][:, o.i_rows])
            assert S['w_o'].is_contiguous() and S['w_down'].is_contiguous()
        np.testing.assert_array_equal(p['w_lm'].numpy(), ref.lm_q[o.v_rows])
    # the shards' columns put back together are the one-GPU matrices
    for li, L in enumerate(ref.layers):
        np.testing.assert_array_equal(torch.cat([p['layers'][li]['w_o'] for p in parts], 1).numpy(), L['o'][0])
        np.testing.assert_array_equal(torch.cat([p['layers'][li]['w_down'] for p in parts], 1).numpy(), L['down'][0])
    np.testing.assert_array_equal(torch.cat([p['w_lm'] for p in parts]).numpy(), ref.lm_q)


def test_check_shardable_guards():
    from efficientgpt_b200.tp import Qwen3Shape, check_shardable, shard
    s = Qwen3Shape(2, 128, 4, 2, 32, 256, 512, 1e-6, 1e6)
    check_shardable(s, 2)
    for world in (3, 16):
        with pytest.raises(ValueError):
            check_shardable(s, world)
    with pytest.raises(ValueError, match='kv heads'):
        check_shardable(s, 4)
    with pytest.raises(ValueError, match='16-row tiles'):
        check_shardable(Qwen3Shape(2, 128, 4, 2, 32, 264, 512, 1e-6, 1e6), 2)
    with pytest.raises(ValueError, match='rank'):
        shard({'layers': []}, s, 2, 2)


def test_argmax_key_order():
    """Larger logit wins, then the lower global index; NaN above everything; -0 == +0 (argmax_better's order)."""
    vals = [(-3.5, 7), (-0.0, 9), (0.0, 4), (0.0, 11), (1.25, 100), (1.25, 3), (float('inf'), 50), (float('nan'), 60),
            (float('nan'), 2), (-float('inf'), 0)]
    keys = [argmax_key(v, i) for v, i in vals]
    best = max(keys)
    assert key_index(best) == 2
    finite = [argmax_key(v, i) for v, i in vals if not np.isnan(v)]
    assert key_index(max(finite)) == 50
    assert key_index(max(argmax_key(v, i) for v, i in vals[:4])) == 4  # zero of either sign: lowest index
    assert key_index(max(argmax_key(v, i) for v, i in vals[4:6])) == 3
    rng = np.random.default_rng(0)
    for _ in range(200):  # the per-rank key maximum equals the first-index argmax of the concatenated logits
        lg = round_bf16(rng.standard_normal(64).astype(np.float32) * 2)
        lg[rng.integers(0, 64, 3)] = lg.max()  # ties across ranks
        per = [lg[r * 16:(r + 1) * 16] for r in range(4)]
        ks = [argmax_key(p[first_argmax(p)], first_argmax(p) + r * 16) for r, p in enumerate(per)]
        assert key_index(max(ks)) == first_argmax(lg)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port, prompt, n_new, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        ref = Qwen3Ref.from_hf(gi.build_model(gi.tiny_config()), 64, 'bf16', semantics='cpu')

        def allgather(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            got = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(got, t)
            return [g.numpy() for g in got]

        toks, logs = TPQwen3Ref(ref, rank, world, allgather).feed_and_generate(prompt, n_new)
        out[rank] = (toks, [np.asarray(lg) for lg in logs])
    finally:
        dist.destroy_process_group()


def test_tp_oracle_two_gloo_ranks_match_one_rank():
    """The TP restatement (fp64 partials exchanged over gloo, rank-order sums) gives the one-rank oracle's greedy
    tokens under the near-tie rule and its logits within 1e-2."""
    import torch.multiprocessing as mp
    prompt, n_new, world = gi.tiny_prompts()[5][0].tolist(), 12, 2
    ref = Qwen3Ref.from_hf(gi.build_model(gi.tiny_config()), 64, 'bf16', semantics='cpu')
    want_t, want_l = [], []
    for pos, t in enumerate(prompt):  # token by token, as the TP ranks feed it
        lg = ref.forward([t], pos)
    pos = len(prompt)
    for i in range(n_new):
        want_t.append(int(np.argmax(lg)))
        want_l.append(lg)
        if i < n_new - 1:
            lg = ref.forward([want_t[-1]], pos)
            pos += 1
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_tp_rank, args=(world, _free_port(), prompt, n_new, out), nprocs=world, join=True,
                           start_method='spawn')
        res = dict(out)
    assert res[0][0] == res[1][0], 'ranks disagree on the token'
    got_t = res[0][0]
    margins = [float(np.sort(l)[-1] - np.sort(l)[-2]) for l in want_l]
    tops = [float(l.max()) for l in want_l]
    ok, first, detail = parity.near_tie_match(want_t, margins, tops, got_t)
    assert ok, detail
    upto = n_new if first is None else first
    for i in range(upto):
        got_l = np.concatenate([res[r][1][i] for r in range(world)])
        assert parity.logits_close(got_l, want_l[i])[0], i


def test_rope_table_without_a_model_equals_the_bf16_models():
    """A fresh rotary module cast to bf16 gives the table of a bf16 HF model (whose inv_freq buffer is cast too)."""
    from efficientgpt_b200.tp import rope_tables
    cfg = gi.tiny_config()
    model = gi.build_model(cfg)
    shape = _shape(cfg)
    a = rope_tables(shape, 96, 'cpu')
    b = rope_tables(shape, 96, 'cpu', model.model.rotary_emb)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
