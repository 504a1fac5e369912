"""CPU oracle for the batch-1 int8 decode path — TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this package, and
only as the checker or the timed CPU baseline. The product (efficientgpt_b200) never imports it and has no CPU
fallback.

Contents (each function cites the reference file:line it restates):
  bf16.py       bf16 round-to-nearest-even on float32 arrays (PyTorch's cast semantics)
  int8_ref.py   quantize_weight, the op's <=16-row and >16-row arithmetic, fp64 truth
                (BagelsFun/efficientgpt research/realmodel/int8_linear.py)
  qwen3_ref.py  Qwen3 decoder forward and greedy static-cache loop in numpy, eager bf16 rounding points
                (transformers modeling_qwen3.py as called by research/realmodel/fast_decode.py)
  attn_ref.py   fp64 attention truth (masked SDPA semantics) and the split/LSE-combine restatement
                (research/phase5/decode_attention.py)
  torch_ref.py  the reference's CPU path: HF transformers model + the int8 op restated in torch
                (x.float() @ q.float().T * s), used for the timed CPU baseline

Pinning: tests/test_oracle.py checks these restatements against the golden vectors of tests/golden/, which
were produced by running the reference itself (tests/golden/make_golden.py).
"""
