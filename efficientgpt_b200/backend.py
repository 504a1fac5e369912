"""Request-sized CUDA-graph decoders for serving: the decode layer of the reference's HFBackend.

Drop-in for BagelsFun/efficientgpt assistant/backends.py:160-167 `pick_bucket`, :221-222 `GRAPH_BUCKETS` /
`MAX_GRAPH_DECODERS` and the decoder cache of :232-280 `HFBackend._chat_graph`. The static-cache attention of a decode
step reads the whole cache it was captured with, so each request runs on the smallest capacity bucket that holds its
prompt plus new tokens. Here a step reads only the positions up to the current one, but a bucket still sizes the KV
cache and the captured graph, so requests of different lengths keep memory proportional to what they need.

`BucketedGraphDecoder(model)` keeps at most `max_decoders` GraphGreedyDecoders (one KV cache and one captured graph
each), keyed by bucket and ordered by last use: a request reuses its bucket's decoder (generate() starts it from
position 0; stale cache slots are never read) and, when a new bucket is needed and the pool is full, the least
recently used decoder is dropped and its device memory released. All decoders share the model's int8 weights.
Tokenisation, chat templates and the streamer's text assembly stay with the caller (the assistant application).
"""
import time
from collections import OrderedDict

import torch

from .fast_decode import GraphGreedyDecoder

GRAPH_BUCKETS = (256, 384, 512, 1024, 2048, 4096)
MAX_GRAPH_DECODERS = 3


def pick_bucket(need, buckets, limit):
    """The smallest capacity >= need among `buckets` no larger than `limit`, then `limit` itself; None when even
    `limit` is too small."""
    for cap in sorted(b for b in buckets if b <= limit) + [limit]:
        if cap >= need:
            return cap
    return None


class BucketedGraphDecoder:
    """Greedy decoding through a pool of request-sized GraphGreedyDecoders (least recently used dropped first)."""

    def __init__(self, model, buckets=GRAPH_BUCKETS, max_decoders=MAX_GRAPH_DECODERS, limit=4096, lookahead=8,
                 **decoder_kw):
        if max_decoders < 1:
            raise ValueError('max_decoders must be >= 1')
        self.model, self.buckets, self.max_decoders, self.limit = model, tuple(buckets), max_decoders, limit
        self.lookahead, self.decoder_kw = lookahead, decoder_kw
        self._pool = OrderedDict()  # bucket -> GraphGreedyDecoder, least recently used first

    @property
    def cached_buckets(self):
        """Buckets with a live decoder, least recently used first."""
        return list(self._pool)

    def decoder_for(self, need):
        """(decoder, seconds spent building it) for a request of `need` positions (prompt + new tokens)."""
        cap = pick_bucket(need, self.buckets, self.limit)
        if cap is None:
            raise ValueError(f'prompt + max_new_tokens = {need} exceeds the largest capacity {self.limit}')
        built = 0.0
        if cap in self._pool:
            self._pool.move_to_end(cap)
        else:
            while len(self._pool) >= self.max_decoders:
                self._release(next(iter(self._pool)))
            t = time.perf_counter()
            self._pool[cap] = GraphGreedyDecoder(self.model, max_cache_len=cap, lookahead=self.lookahead,
                                                 **self.decoder_kw)
            built = time.perf_counter() - t
        return self._pool[cap], built

    def _release(self, cap):
        dec = self._pool.pop(cap)
        dec.graph = None  # the captured graph and its memory pool go with the last reference
        del dec
        torch.cuda.empty_cache()

    def generate(self, input_ids, max_new_tokens, eos_ids=(), on_token=None):
        """GraphGreedyDecoder.generate on the request's bucket; stats add 'bucket' and fold the decoder's build time
        into 'capture_s' (outside the time to first token, as the reference reports it)."""
        dec, built = self.decoder_for(input_ids.shape[1] + max_new_tokens)
        out, st = dec.generate(input_ids, max_new_tokens, eos_ids=eos_ids, on_token=on_token)
        st['capture_s'] = st.get('capture_s', 0.0) + built
        st['bucket'] = dec.max_cache_len
        n = len(out)
        st['decode_tok_s'] = (n - 1) / (st['total_s'] - st['ttft_s']) if n > 1 and st['total_s'] > st['ttft_s'] \
            else float('nan')
        return out, st

    def close(self):
        for cap in list(self._pool):
            self._release(cap)
