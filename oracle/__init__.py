"""CPU oracle of the reference's hot path — TEST INFRASTRUCTURE ONLY.

Restatements of imoshka2009-lab/hackathon `solution/` kernels on the CPU, used as the checker
by tests/, by `__graft_entry__.smoke()` and by bench.py's `cpu_baseline` / `--impl reference`
legs. Nothing in the product (`hackathon_b200/`) imports this package.

  nf4_ref.py   numpy: NF4 + double-quant dequant bit for bit (fp16/fp32/bf16 with
               round-to-nearest-even), the quantiser, the Philox-4x32-10 dropout stream
  ops_ref.py   torch fp32 on CPU: RMSNorm, RoPE, SwiGLU, scaled add, cross-entropy with the
               TRL/Soup metrics, and a Qwen2 decoder layer with NF4 + LoRA linears
  nf4_ref.c    plain C: NF4 dequant (the CPU baseline of the standalone dequant sweep)

Pinning: tests/golden/ holds fixtures produced by running the reference's own Triton kernels in
Triton's CPU interpreter (tests/golden/make_golden.py); tests/test_oracle.py checks every
restatement here against them. The interpreter rounds fp32->bf16 by truncation, so bf16
fixtures are compared after re-rounding the fixture's fp32 result; fp16/fp32 fixtures are
compared bit for bit.
"""
