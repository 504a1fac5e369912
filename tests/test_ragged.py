"""Ragged small-batch greedy decoding (efficientgpt_b200.ragged) on the tiny Qwen3: the contract of
research/phase5/ragged.py. CPU: the request checks. GPU: every row against the reference's own greedy tokens of
that prompt (tests/golden/golden.json, made by the reference) under the near-tie rule, the graph decoder equal to
the eager engine, equal prompts giving equal rows, and pad values never read."""
import pytest
import torch

import golden_inputs as gi
from oracle import parity


def test_check_ragged():
    from efficientgpt_b200.ragged import check_ragged
    p = torch.zeros(3, 8, dtype=torch.long)
    ok = torch.tensor([1, 8, 3])
    check_ragged(p, ok, 4, 12)
    for prompts, lengths, count, cap in [(p, torch.tensor([0, 8, 3]), 4, 12), (p, torch.tensor([1, 9, 3]), 4, 12),
                                         (p, ok.int(), 4, 12), (p, ok, 0, 12), (p, ok, 5, 12),
                                         (torch.zeros(17, 8, dtype=torch.long), torch.ones(17, dtype=torch.long), 1, 12)]:
        with pytest.raises(ValueError):
            check_ragged(prompts, lengths, count, cap)


def _model(scale_dtype=torch.bfloat16):
    from efficientgpt_b200.int8_linear import quantize_model
    model = gi.build_model(gi.tiny_config()).cuda()
    quantize_model(model, scale_dtype=scale_dtype)
    return model


def _batch(pad_seed=0):
    prompts = gi.tiny_prompts()
    lens = sorted(prompts)
    pmax = max(lens)
    g = torch.Generator().manual_seed(pad_seed)
    x = torch.randint(0, 512, (len(lens), pmax), generator=g)  # pads: arbitrary ids, never read
    for r, p in enumerate(lens):
        x[r, :p] = prompts[p][0]
    return x, torch.tensor(lens, dtype=torch.long), lens


@pytest.mark.gpu
def test_ragged_rows_match_reference_golden(cuda, golden):
    from efficientgpt_b200.ragged import RaggedGraphDecoder
    model = _model()
    x, lengths, lens = _batch()
    count = 24
    dec = RaggedGraphDecoder(model, len(lens), max(lens) + count)
    out = dec.generate(x.cuda(), lengths.cuda(), count).cpu().tolist()
    for r, p in enumerate(lens):
        run = golden['tiny_qwen3']['runs']['bf16'][str(p)]
        ok, first, detail = parity.near_tie_match(run['tokens'][:count], run['margins'][:count], run['tops'][:count],
                                                  out[r])
        assert ok, (p, detail)


@pytest.mark.gpu
def test_ragged_graph_equals_eager_and_pads_unread(cuda):
    from efficientgpt_b200.ragged import RaggedEngine, RaggedGraphDecoder
    model = _model()
    x, lengths, lens = _batch(pad_seed=1)
    count = 20
    cap = max(lens) + count
    eager = RaggedEngine(model, len(lens), cap).generate_eager(x.cuda(), lengths.cuda(), count)
    graph = RaggedGraphDecoder(model, len(lens), cap)
    a = graph.generate(x.cuda(), lengths.cuda(), count)
    assert torch.equal(eager, a)
    x2, _, _ = _batch(pad_seed=2)  # other pad values
    b = graph.generate(x2.cuda(), lengths.cuda(), count)  # the decoder reused with new pads
    assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize('rows', [2, 8])
def test_ragged_equal_rows(cuda, golden, rows):
    """Equal prompts give equal rows, on the GEMV (2 rows) and on the tcgen05 GEMM (8 rows) projections, and the
    row matches the reference's greedy tokens under the near-tie rule."""
    from efficientgpt_b200.ragged import RaggedGraphDecoder
    model = _model()
    p = gi.tiny_prompts()[5]
    x = p.repeat(rows, 1)
    dec = RaggedGraphDecoder(model, rows, 5 + 16)
    assert dec.engine.use_gemm == (rows >= 4)
    out = dec.generate(x.cuda(), torch.full((rows,), 5, dtype=torch.long).cuda(), 16)
    assert all(torch.equal(out[0], out[r]) for r in range(1, rows))
    run = golden['tiny_qwen3']['runs']['bf16']['5']
    ok, _, detail = parity.near_tie_match(run['tokens'][:16], run['margins'][:16], run['tops'][:16], out[0].tolist())
    assert ok, detail
