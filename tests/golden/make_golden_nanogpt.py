"""Generate the nanoGPT golden fixture (tests/golden/nanogpt_tiny.npz, nanogpt.json) by running the REFERENCE on CPU.

    python tests/golden/make_golden_nanogpt.py --reference /path/to/efficientgpt

The model is the reference's own decoder test model (research/phase4/test_decoder.py:10-15: GPT block 32, vocab
128, 2 layers, 32 dims, bias, torch.manual_seed(10)) with ONE head instead of two (head_dim 32: the native attention
kernels are built for head dims 32, 64 and 128), quantised by research/realmodel/int8_linear.py
quantize_model (int8 per row, fp32 scales; the tied lm_head becomes an int8 copy). The int8 op refuses fp32
activations (int8_linear.py:92-93), so, as BASELINE config 1 states, every Int8Linear runs the torch dequant matmul
x @ (q.float() * s[:, None]).T + b. Greedy tokens come from research/phase4/decoder.py generate_reference (dynamic
K/V concatenation) and are checked against StaticKVDecoder.generate_eager. The fixture holds the model's fp32
parameters (the GPU side has no reference model code), the prompts, the reference's tokens with top-2 margins and
the first-step fp32 logits.
"""
import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
PROMPTS = ((3, 8, 1), (7, 6, 3), (13, 4, 5), (29, 3, 7))  # (length, new tokens, seed): test_decoder.py:17-33 cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from model import GPT, GPTConfig
    import research.realmodel.int8_linear as il
    from research.phase4.decoder import StaticKVDecoder, generate_reference, reference_step

    def dequant_forward(self, x):
        y = x @ (self.qweight.float() * self.scale.float()[:, None]).t()
        return y if self.bias is None else y + self.bias
    il.Int8Linear.forward = dequant_forward

    torch.manual_seed(10)
    model = GPT(GPTConfig(block_size=32, vocab_size=128, n_layer=2, n_head=1, n_embd=32, dropout=0.0, bias=True)).eval()
    params = {k: v.detach().float().numpy().copy() for k, v in model.state_dict().items()}
    il.quantize_model(model)
    arrays = {'param.' + k: v for k, v in params.items()}
    meta = {'reference': 'research/phase4/test_decoder.py model; int8_linear.quantize_model; decoder.generate_reference',
            'config': {'block_size': 32, 'vocab_size': 128, 'n_layer': 2, 'n_head': 1, 'n_embd': 32, 'bias': True},
            'params_sha256': hashlib.sha256(b''.join(params[k].tobytes() for k in sorted(params))).hexdigest(),
            'runs': []}
    for length, count, seed in PROMPTS:
        torch.manual_seed(seed)
        ids = torch.randint(0, 128, (1, length))
        toks = generate_reference(model, ids, count)[0, length:].tolist()
        eager = StaticKVDecoder(model, 1).generate_eager(ids, count)[0, length:].tolist()
        assert toks == eager, (length, toks, eager)
        margins = []
        with torch.inference_mode():
            logits, cache = reference_step(model, ids)
            arrays[f'logits_first_{length}'] = logits[0, -1].numpy().copy()
            for i in range(count):
                top = logits[0, -1].topk(2).values
                margins.append(float(top[0] - top[1]))
                tok = logits.argmax(-1)
                if i != count - 1:
                    logits, cache = reference_step(model, tok, cache)
        meta['runs'].append({'prompt': ids[0].tolist(), 'tokens': toks, 'margins': margins})
    np.savez_compressed(HERE / 'nanogpt_tiny.npz', **arrays)
    (HERE / 'nanogpt.json').write_text(json.dumps(meta, indent=1))
    print('wrote nanogpt_tiny.npz, nanogpt.json', [len(r['tokens']) for r in meta['runs']])


if __name__ == '__main__':
    main()
