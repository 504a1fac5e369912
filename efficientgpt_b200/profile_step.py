"""Small, self-contained decode workload for profilers (ncu captures must stay small).

    python -m efficientgpt_b200.profile_step [--layers 4] [--steps 3] [--launch-sequence]

Builds the Qwen3-1.7B shape with `--layers` decoder layers (random init, seed 0, int8 weights with bf16 scales), runs
a 32-token prefill and `--steps` decode steps of the persistent kernel (or the per-stage launch sequence), checks the
device error word and prints the last token and position. The full 28-layer model is `bench.py`'s workload.
"""
import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--layers', type=int, default=4)
    ap.add_argument('--steps', type=int, default=3)
    ap.add_argument('--launch-sequence', action='store_true')
    a = ap.parse_args()
    from . import _lib
    from .configs import qwen3_1p7b_config, random_model
    from .engine import Qwen3Engine
    from .int8_linear import quantize_model
    cfg = qwen3_1p7b_config()
    cfg.num_hidden_layers = a.layers
    model = random_model(cfg, 'cuda', 0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    eng = Qwen3Engine(model, 288, persistent=False if a.launch_sequence else None)
    eng.prefill(torch.randint(0, cfg.vocab_size, (1, 32), generator=torch.Generator().manual_seed(0)).cuda())
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    if _lib.device_error() != 0:
        raise RuntimeError('device error ' + str(_lib.device_error()))
    print('ok', int(eng.token), int(eng.position), 'persistent' if eng.persistent else 'launch sequence')


if __name__ == '__main__':
    main()
