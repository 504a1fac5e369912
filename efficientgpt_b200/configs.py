"""Model configurations of the benchmarked workloads (transformers configs, random init; no checkpoints)."""


def qwen3_1p7b_config():
    """Qwen3-1.7B architecture: 28 layers, hidden 2048, 16 q / 8 kv heads of 128, SwiGLU 6144, vocab 151936,
    RoPE theta 1e6, tied embeddings, N(0, 0.02) init."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                       rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True, initializer_range=0.02)


def qwen3_8b_config():
    """Qwen3-8B architecture: 36 layers, hidden 4096, 32 q / 8 kv heads of 128, SwiGLU 12288, untied lm_head."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                       rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=False, initializer_range=0.02)


def random_model(cfg, device, seed=0):
    """transformers Qwen3ForCausalLM with its own random init under torch.manual_seed(seed), built directly on
    `device`, cast to bf16, eval mode."""
    import torch
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()
