"""Generate the golden fixtures of tests/golden/ by running the REFERENCE implementation on CPU.

    python tests/golden/make_golden.py --reference /path/to/efficientgpt [--skip-big]

Needs the BagelsFun/efficientgpt checkout (imported from --reference) and transformers; it is run once in the
development container and its outputs (*.npz, golden.json) are committed. Nothing on the test or GPU side
imports the reference. Inputs are rebuilt from seeds (golden_inputs.py); the fixtures hold the reference's
outputs and the SHA-256 of every input. What each fixture pins:

* quantize.npz: research/realmodel/int8_linear.py:106-117 quantize_weight on seeded bf16 weights (8200 rows, so
  the 8192-row chunking is crossed) and on hand-made edge rows (zeros, exact .5 ties, huge/tiny/subnormal values).
* prefill_linear.npz: the op efficientgpt::int8_linear (int8_linear.py:88-98) on its >16-row branch (the branch
  that runs on CPU): bf16(bf16(x @ bf16(q).T) * s).
* tiny_qwen3.npz / golden.json["tiny_qwen3"]: the reference's own test model (research/realmodel/
  test_fast_decode.py:9-15, initializer_range 0.2), quantised by the reference's quantize_model, greedy-decoded by
  HF generate(cache_implementation='static') for prompts of length 1, 5 and 37 (40 new tokens), with fp32 and
  bf16 scales; first-step logits for prompt 5. The Triton decode kernel cannot run on CPU, so the <=16-row branch
  of int8_matmul is replaced by its arithmetic, bf16((x.float() @ q.float().T) * s) (fp32 accumulation).
* golden.json["qwen3_1p7b"]: BASELINE config 2 (Qwen3-1.7B shape, N(0, 0.02) init, torch.manual_seed(0) on CPU),
  bf16 scales, same path, 32 prompt ids (seed 0) and 16 greedy tokens, with the top-2 logit margin of every step
  (for the near-tie rule of research/phase5/benchmark_review.py:54-67).
"""
import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402


def bf16_bits(t):
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def patch_reference_decode_branch(il):
    def cpu_int8_matmul(x2, w, s):  # arithmetic of the Triton _dot16 kernel: fp32 accumulation, scale, bf16
        if x2.shape[0] > il.MAX_DECODE_ROWS:
            raise ValueError('more than 16 rows')
        return ((x2.float() @ w.float().t()) * s).to(torch.bfloat16)
    il.int8_matmul = cpu_int8_matmul


def greedy_loop(model, ids, n_new, max_cache_len):
    """Static-cache greedy loop (the GraphGreedyDecoder step without graphs); returns tokens, top-2 margins,
    top-1 logit values."""
    from transformers import StaticCache
    cache = StaticCache(config=model.config, max_cache_len=max_cache_len)
    toks, margins, tops = [], [], []
    with torch.inference_mode():
        logits = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1).logits[0, -1]
        p = ids.shape[1]
        for i in range(n_new):
            top = logits.float().topk(2).values
            margins.append(float(top[0] - top[1]))
            tops.append(float(top[0]))
            tok = int(logits.argmax(-1))
            toks.append(tok)
            if i == n_new - 1:
                break
            logits = model(input_ids=torch.tensor([[tok]]), position_ids=torch.tensor([[p + i]]), past_key_values=cache,
                           use_cache=True, logits_to_keep=1).logits[0, -1]
    return toks, margins, tops


def hf_greedy(model, x, n):
    out = model.generate(input_ids=x, attention_mask=torch.ones_like(x), max_new_tokens=n, min_new_tokens=n,
                         do_sample=False, cache_implementation='static', pad_token_id=0)
    return out[0, x.shape[1]:].tolist()


def to_bf16_scales(il, model):
    for mod in model.modules():
        if isinstance(mod, il.Int8Linear):
            mod.scale = mod.scale.to(torch.bfloat16)


def make_quantize(il, meta):
    w = gi.quantize_input()
    q, s = il.quantize_weight(w)
    edge = gi.quantize_edge_rows()
    qe, se = il.quantize_weight(edge)
    np.savez_compressed(HERE / 'quantize.npz', q=q.numpy(), s=s.numpy(), edge_q=qe.numpy(), edge_s=se.numpy())
    meta['quantize'] = {'reference': 'research/realmodel/int8_linear.py:106-117 quantize_weight',
                        'w_sha256': gi.sha(w), 'edge_sha256': gi.sha(edge)}


def make_prefill_linear(il, meta):
    arrays, shas = {}, []
    for i in range(len(gi.PREFILL_SHAPES)):
        x, q, s = gi.prefill_case(i)
        arrays[f'y{i}'] = bf16_bits(il.int8_linear(x, q, s))
        shas.append([gi.sha(x), gi.sha(q), gi.sha(s)])
    np.savez_compressed(HERE / 'prefill_linear.npz', **arrays)
    meta['prefill_linear'] = {'reference': 'research/realmodel/int8_linear.py:88-98 (>16-row branch)',
                              'shapes_mkn': gi.PREFILL_SHAPES, 'input_sha256': shas}


def make_tiny(il, meta):
    out = {'reference': 'research/realmodel/test_fast_decode.py:9-15 model + int8_linear.quantize_model + HF generate',
           'runs': {}}
    arrays = {}
    for scale_dtype in ('fp32', 'bf16'):
        model = gi.build_model(gi.tiny_config())
        out['state_sha256'] = gi.state_hash(model)
        il.quantize_model(model)
        if scale_dtype == 'bf16':
            to_bf16_scales(il, model)
        runs = {}
        for p, x in gi.tiny_prompts().items():
            toks = hf_greedy(model, x, 40)
            loop, margins, tops = greedy_loop(model, x, 40, 128)
            assert loop == toks, (scale_dtype, p)
            runs[str(p)] = {'prompt': x[0].tolist(), 'tokens': toks, 'margins': margins, 'tops': tops}
            if p == 5:
                with torch.inference_mode():
                    lg = model(input_ids=x, logits_to_keep=1).logits[0, -1]
                arrays[f'logits_p5_{scale_dtype}'] = bf16_bits(lg)
        out['runs'][scale_dtype] = runs
    np.savez_compressed(HERE / 'tiny_qwen3.npz', **arrays)
    meta['tiny_qwen3'] = out


def make_big(il, meta):
    t = time.time()
    model = gi.build_model(gi.qwen3_1p7b_config())
    h = gi.state_hash(model)
    il.quantize_model(model)
    to_bf16_scales(il, model)
    x = gi.big_prompt()
    toks, margins, tops = greedy_loop(model, x, 16, 64)
    meta['qwen3_1p7b'] = {'reference': 'BASELINE config 2 shape through int8_linear.quantize_model (bf16 scales)',
                          'state_sha256': h, 'prompt': x[0].tolist(), 'tokens': toks, 'margins': margins, 'tops': tops,
                          'seconds': round(time.time() - t, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    ap.add_argument('--skip-big', action='store_true')
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import research.realmodel.int8_linear as il
    patch_reference_decode_branch(il)
    import transformers
    meta = {'torch': torch.__version__, 'transformers': transformers.__version__}
    old = HERE / 'golden.json'
    if a.skip_big and old.exists():
        prev = json.loads(old.read_text())
        if 'qwen3_1p7b' in prev:
            meta['qwen3_1p7b'] = prev['qwen3_1p7b']
    make_quantize(il, meta)
    make_prefill_linear(il, meta)
    make_tiny(il, meta)
    if not a.skip_big:
        make_big(il, meta)
    (HERE / 'golden.json').write_text(json.dumps(meta, indent=1))
    print('wrote', sorted(p.name for p in HERE.iterdir()))


if __name__ == '__main__':
    main()
