"""The serving decode layer (efficientgpt_b200/backend.py), after assistant/backends.py:160-167,221-280:
capacity buckets on the CPU, the LRU pool of graph decoders on the GPU."""
import gc
import weakref

import pytest
import torch

import golden_inputs as gi
from oracle import parity


def test_pick_bucket_matches_the_reference_rule():
    from efficientgpt_b200.backend import GRAPH_BUCKETS, pick_bucket
    assert pick_bucket(1, GRAPH_BUCKETS, 4096) == 256
    assert pick_bucket(256, GRAPH_BUCKETS, 4096) == 256
    assert pick_bucket(257, GRAPH_BUCKETS, 4096) == 384
    assert pick_bucket(2049, GRAPH_BUCKETS, 4096) == 4096
    assert pick_bucket(4097, GRAPH_BUCKETS, 4096) is None
    assert pick_bucket(600, GRAPH_BUCKETS, 1000) == 1000  # buckets above the limit are skipped, the limit is last
    assert pick_bucket(300, (384, 256), 300) == 300
    assert pick_bucket(10, (), 64) == 64


@pytest.mark.gpu
def test_bucketed_decoders_reuse_evict_and_match_the_golden(cuda, golden):
    """Requests of three lengths through a pool of at most two decoders (buckets 64 / 96 / 128): tokens equal the
    single GraphGreedyDecoder's and follow the reference's golden under the near-tie rule, a bucket is reused, the
    least recently used decoder is dropped when a third bucket is needed, and its KV cache is released."""
    from efficientgpt_b200.backend import BucketedGraphDecoder
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    from test_decoder_gpu import _quantize
    model = gi.build_model(gi.tiny_config()).cuda()
    _quantize(model, torch.float32, 'cpu')
    runs = golden['tiny_qwen3']['runs']['fp32']
    prompts = gi.tiny_prompts()
    pool = BucketedGraphDecoder(model, buckets=(64, 96, 128), max_decoders=2, limit=128)
    ref = GraphGreedyDecoder(model, max_cache_len=128)

    def run(p, n):
        x = prompts[p].cuda()
        got, st = pool.generate(x, n)
        want, _ = ref.generate(x, n)
        assert got == want, (p, n)
        g = runs[str(p)]
        m = min(n, len(g['tokens']))  # the golden holds 40 tokens per prompt
        ok, _, detail = parity.near_tie_match(g['tokens'][:m], g['margins'][:m], g['tops'][:m], got[:m])
        assert ok, (p, detail)
        return st

    assert run(1, 40)['bucket'] == 64          # 41 positions
    assert run(37, 40)['bucket'] == 96         # 77 positions
    assert pool.cached_buckets == [64, 96]
    assert run(5, 40)['bucket'] == 64          # reused (no new decoder), now most recently used
    assert pool.cached_buckets == [96, 64]
    kv96 = weakref.ref(pool._pool[96].engine.kv)
    before = torch.cuda.memory_allocated()
    st = run(37, 80)                           # 117 positions: bucket 128, the pool is full, 96 is dropped
    assert st['bucket'] == 128 and pool.cached_buckets == [64, 128]
    gc.collect()
    assert kv96() is None, 'the evicted decoder still holds its KV cache'
    with pytest.raises(ValueError):
        pool.generate(prompts[37].cuda(), 100)  # 137 positions > limit
    pool.close()
    gc.collect()
    assert torch.cuda.memory_allocated() < before
