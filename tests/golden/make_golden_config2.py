"""Generate tests/golden/qwen3_1p7b_256.json: BASELINE config 2 greedy decode, all 256 steps, by the REFERENCE.

    python tests/golden/make_golden_config2.py --reference /path/to/efficientgpt [--no-diagnostic]

Runs once in the development container (CPU) and its output is committed; nothing on the test or GPU side imports
the reference. The model is BASELINE config 2 (Qwen3-1.7B shape, N(0, 0.02) init under torch.manual_seed(0) on the
CPU, golden_inputs.build_model), quantised by the reference's own quantize_model (research/realmodel/
int8_linear.py:137-157) with bf16 scales, prompt golden_inputs.big_prompt() (32 ids), then 256 greedy tokens
through HF's Qwen3 forward with a static cache (the GraphGreedyDecoder step of research/realmodel/fast_decode.py:
45-49 without graphs). The Triton decode kernel cannot run on the CPU, so the <= 16-row branch of int8_matmul is
replaced by its arithmetic bf16((x.float() @ q.float().T) * s) (fp32 accumulation, as make_golden.py does).

Recorded per step: the token, the top-2 logit margin, the top-1 logit and the runner-up index.
--diagnostic-only keeps the recorded greedy run and redoes the diagnostic below.

Diagnostic (skipped with --no-diagnostic): the same reference forward, teacher-forced along the golden tokens,
with only the decode GEMV's summation changed to the exact sum rounded once to fp32 (fp64 accumulation of the
bf16 x int8 products, which it holds exactly). The steps whose argmax then differs from the golden show how many
greedy choices of this model turn on the fp32 summation order of the int8 GEMV alone, with no other change; the
logits of the golden's top-1 and runner-up tokens in that run show how far the summation order alone moves the
decisive logits.
"""
import argparse
import json
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402

N_NEW = 256
CAP = 32 + N_NEW


def set_decode_branch(il, exact):
    def cpu_int8_matmul(x2, w, s):
        if x2.shape[0] > il.MAX_DECODE_ROWS:
            raise ValueError('more than 16 rows')
        if exact:
            acc = (x2.double() @ w.double().t()).float()
        else:
            acc = x2.float() @ w.float().t()
        return (acc * s).to(torch.bfloat16)
    il.int8_matmul = cpu_int8_matmul


def run(model, prompt, forced=None, probe=None):
    """Greedy static-cache loop; with `forced` (token list) the input of step i + 1 is forced[i] instead of the
    step's own argmax. Returns tokens (argmax per step), margins, top-1 logits, runner-up ids and, with `probe` (per
    step a list of vocabulary ids), the logits at those ids."""
    from transformers import StaticCache
    cache = StaticCache(config=model.config, max_cache_len=CAP)
    toks, margins, tops, second, probed = [], [], [], [], []
    p = prompt.shape[1]
    with torch.inference_mode():
        logits = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1).logits[0, -1]
        for i in range(N_NEW):
            top = logits.float().topk(2)
            margins.append(float(top.values[0] - top.values[1]))
            tops.append(float(top.values[0]))
            tok = int(logits.argmax(-1))
            second.append(int(top.indices[1]) if int(top.indices[0]) == tok else int(top.indices[0]))
            toks.append(tok)
            if probe is not None:
                probed.append([float(logits[j]) for j in probe[i]])
            if i == N_NEW - 1:
                break
            nxt = forced[i] if forced is not None else tok
            logits = model(input_ids=torch.tensor([[nxt]]), position_ids=torch.tensor([[p + i]]), past_key_values=cache,
                           use_cache=True, logits_to_keep=1).logits[0, -1]
            if i % 32 == 31:
                print(f'  step {i + 1}', flush=True)
    return toks, margins, tops, second, probed


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    ap.add_argument('--no-diagnostic', action='store_true')
    ap.add_argument('--diagnostic-only', action='store_true', help='keep the golden run, redo the diagnostic')
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import research.realmodel.int8_linear as il
    import transformers
    torch.set_num_threads(torch.get_num_threads())
    t = time.time()
    model = gi.build_model(gi.qwen3_1p7b_config())
    h = gi.state_hash(model)
    il.quantize_model(model)
    for mod in model.modules():
        if isinstance(mod, il.Int8Linear):
            mod.scale = mod.scale.to(torch.bfloat16)
    prompt = gi.big_prompt()
    if a.diagnostic_only:
        out = json.loads((HERE / 'qwen3_1p7b_256.json').read_text())
        assert out['state_sha256'] == h
        toks, margins, tops, second = out['tokens'], out['margins'], out['tops'], out['runner_up']
    else:
        set_decode_branch(il, exact=False)
        toks, margins, tops, second, _ = run(model, prompt)
    out = {'reference': 'BASELINE config 2 through research/realmodel/int8_linear.quantize_model (bf16 scales), HF '
                        'Qwen3 forward with a static cache, greedy; int8 decode branch as fp32-accumulated arithmetic',
           'torch': torch.__version__, 'transformers': transformers.__version__, 'state_sha256': h,
           'prompt': prompt[0].tolist(), 'tokens': toks, 'margins': margins, 'tops': tops, 'runner_up': second,
           'seconds': round(time.time() - t, 1)}
    if not a.no_diagnostic:
        t = time.time()
        set_decode_branch(il, exact=True)
        pairs = [[toks[i], second[i]] for i in range(N_NEW)]
        ex, ex_m, _, _, probed = run(model, prompt, forced=toks, probe=pairs)
        diff = [i for i in range(N_NEW) if ex[i] != toks[i]]
        want = [[tops[i], tops[i] - margins[i]] for i in range(N_NEW)]
        err = [abs(p - w) for pw, ww in zip(probed, want) for p, w in zip(pw, ww)]
        within = sum(1 for e, ww in zip(err, [w for ww in want for w in ww]) if e <= 1e-2 + 1e-2 * abs(ww)) / len(err)
        out['exact_sum_diagnostic'] = {
            'what': 'same forward teacher-forced along `tokens`, int8 decode GEMV as the exact sum rounded once',
            'steps_differing': diff, 'identical': N_NEW - len(diff),
            'golden_margins_at_differing_steps': [margins[i] for i in diff],
            'decisive_logits': probed,
            'decisive_logits_max_abs_diff': max(err), 'decisive_logits_within_1e-2_abs_rel': within,
            'seconds': round(time.time() - t, 1)}
    (HERE / 'qwen3_1p7b_256.json').write_text(json.dumps(out, indent=1))
    print('wrote qwen3_1p7b_256.json', out.get('exact_sum_diagnostic', {}).get('identical'))


if __name__ == '__main__':
    main()
