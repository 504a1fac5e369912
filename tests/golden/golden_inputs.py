"""Seeded inputs of the golden fixtures (shared by make_golden.py and the tests).

The fixtures store the reference's outputs plus a SHA-256 of every input; the inputs themselves are rebuilt
from these seeds with torch's CPU generator (deterministic for a given torch build), and the tests check the
hash before comparing, so a changed generator fails loudly instead of comparing against the wrong data.
"""
import hashlib

import torch

PREFILL_SHAPES = [(17, 100, 70), (32, 128, 64), (24, 256, 48), (20, 2048, 32)]


def sha(t):
    return hashlib.sha256(t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def quantize_input():
    g = torch.Generator().manual_seed(0)
    return (torch.randn(8200, 16, generator=g) * 0.05).to(torch.bfloat16)


def quantize_edge_rows():
    edge = torch.zeros(8, 16)
    edge[1] = torch.arange(16) - 7.5
    edge[2] = torch.tensor([127.0, 63.5, -63.5, 0.5, -0.5, 1.5, 2.5, -2.5] * 2)
    edge[3] = torch.full((16,), 3.0e38) * torch.tensor([1, -1] * 8)
    edge[4] = torch.full((16,), 1e-30) * torch.arange(16)
    edge[5] = torch.full((16,), -2.0)
    edge[6] = torch.tensor([1e-40] * 16)
    edge[7] = torch.linspace(-1, 1, 16)
    return edge


def prefill_case(i):
    m, k, n = PREFILL_SHAPES[i]
    g = torch.Generator().manual_seed(100 + i)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    s = torch.rand(n, generator=g) * 0.01 + 1e-4
    return x, q, s


def tiny_config():
    """research/realmodel/test_fast_decode.py:9-15 (initializer_range 0.2 so greedy output is not degenerate)."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=32, max_position_embeddings=256, tie_word_embeddings=True,
                       initializer_range=0.2)


def qwen3_1p7b_config():
    """Qwen3-1.7B architecture, N(0, 0.02) init, tied embeddings."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                       rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True, initializer_range=0.02)


def build_model(cfg, seed=0):
    """HF Qwen3ForCausalLM, random init under torch.manual_seed(seed) on the CPU, cast to bf16, eval mode."""
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(seed)
    return Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()


def state_hash(model):
    h = hashlib.sha256()
    for name, t in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def tiny_prompts():
    """Prompts of the reference test (lengths 1, 5, 37 from Generator(1))."""
    g = torch.Generator().manual_seed(1)
    return {p: torch.randint(0, 512, (1, p), generator=g) for p in (1, 5, 37)}


def big_prompt():
    return torch.randint(0, 151936, (1, 32), generator=torch.Generator().manual_seed(0))


def sampling_logits(v, seed, scale, dtype=torch.bfloat16):
    """One row of seeded logits for the sampling cases: N(0, scale^2) on the CPU generator, rounded to `dtype`."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(v, generator=g) * scale).to(dtype)


def sampling_uniforms(n, seed):
    g = torch.Generator().manual_seed(10_000 + seed)
    return torch.rand(n, generator=g)
