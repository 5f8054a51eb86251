"""The reference's eager PyTorch path of the QLoRA step, timed on the host CPU — TEST
INFRASTRUCTURE ONLY (bench.py's `cpu_baseline` and `--impl reference` legs).

The reference is Python + Triton; its only CPU-runnable form of the step is the eager code its
tests compare against: the Qwen2 decoder layer (solution/test_rmsnorm.py:9-14 RMSNorm,
test_rope.py:9-17 RoPE, test_kernels.py:24-25 SwiGLU), bitsandbytes-style linears that rebuild
the bf16 weight from NF4 in forward and again in backward (solution/nf4.py:95-112, the dequant
here is the C restatement oracle/nf4_ref.c), peft LoRA with dropout, and ForCausalLMLoss over
the lm_head (test_cross_entropy.py:9-30).

A full 7B step on a CPU takes hours, so this times a bounded SAMPLE: one decoder layer of the
configured shape on `tokens` tokens (forward, checkpoint recompute, backward) and the head + CE
on the same rows, and scales to the model: step_time = layers * layer_time + head_time, so
tokens/s = tokens / step_time. Attention is timed at the sample's sequence length (shorter than
the configured one), which flatters the CPU; the JSON line says so.
"""

import os
import time

import numpy as np
import torch
import torch.nn.functional as F

from . import c_ref, nf4_ref, ops_ref


class _DequantLinear(torch.autograd.Function):
    """F.linear with the weight rebuilt from NF4 in forward and again in backward."""

    @staticmethod
    def forward(ctx, x, mod):
        w = mod.dequant()
        ctx.mod = mod
        return F.linear(x, w, mod.bias)

    @staticmethod
    def backward(ctx, g):
        return g @ ctx.mod.dequant(), None


class CpuNF4LoRALinear(torch.nn.Module):
    def __init__(self, in_f, out_f, bias, r, alpha, p, rng, threads):
        super().__init__()
        n = in_f * out_f
        self.shape = (out_f, in_f)
        self.packed = rng.integers(0, 256, n // 2, dtype=np.uint8)
        self.absmax_q = rng.integers(0, 256, n // 64, dtype=np.uint8)
        from hackathon_b200.nf4 import signed_dynamic_code
        self.code2 = signed_dynamic_code().numpy()
        self.absmax2 = (rng.random((n // 64 + 255) // 256) * 0.05 + 0.01).astype(np.float32)
        self.offset = 0.03
        self.threads = threads
        self.bias = (torch.randn(out_f) * 0.02).to(torch.bfloat16) if bias else None
        self.A = torch.nn.Parameter(torch.empty(r, in_f).uniform_(-in_f ** -0.5, in_f ** -0.5))
        self.B = torch.nn.Parameter(torch.randn(out_f, r) * 0.01)
        self.scaling = alpha / r
        self.p = p

    def dequant(self):
        bits = c_ref.dequant_nf4_bf16(self.packed, self.shape[0] * self.shape[1], self.absmax_q,
                                      self.code2, self.absmax2, self.offset, 64, 256,
                                      threads=self.threads)
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(self.shape)

    def forward(self, x):
        base = _DequantLinear.apply(x, self)
        xd = F.dropout(x, self.p, training=True) if self.p > 0 else x
        lo = F.linear(F.linear(xd, self.A.to(x.dtype)), self.B.to(x.dtype))
        return base + lo * self.scaling


class CpuDecoderLayer(torch.nn.Module):
    def __init__(self, shape, rng, threads):
        super().__init__()
        s = shape
        H, I, D = s.hidden, s.intermediate, s.head_dim
        mk = lambda i, o, b: CpuNF4LoRALinear(i, o, b, s.lora_r, s.lora_alpha, s.lora_dropout,
                                             rng, threads)
        self.s = s
        self.q, self.k, self.v = mk(H, s.heads * D, True), mk(H, s.kv_heads * D, True), \
            mk(H, s.kv_heads * D, True)
        self.o = mk(s.heads * D, H, False)
        self.gate, self.up, self.down = mk(H, I, False), mk(H, I, False), mk(I, H, False)
        self.ln1 = torch.ones(H, dtype=torch.bfloat16)
        self.ln2 = torch.ones(H, dtype=torch.bfloat16)

    def forward(self, h, cos, sin):
        s = self.s
        B, S, _ = h.shape
        x = ops_ref.rmsnorm_ref(h, self.ln1, s.eps)
        q = self.q(x).view(B, S, s.heads, s.head_dim).transpose(1, 2)
        k = self.k(x).view(B, S, s.kv_heads, s.head_dim).transpose(1, 2)
        v = self.v(x).view(B, S, s.kv_heads, s.head_dim).transpose(1, 2)
        q, k = ops_ref.rope_ref(q, k, cos, sin)
        rep = s.heads // s.kv_heads
        a = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1),
                                           v.repeat_interleave(rep, 1), is_causal=True)
        h = h + self.o(a.transpose(1, 2).reshape(B, S, -1))
        x = ops_ref.rmsnorm_ref(h, self.ln2, s.eps)
        m = ops_ref.swiglu_ref(self.gate(x), self.up(x)).to(x.dtype)
        return h + self.down(m)


def usable_cores():
    """Host cores this process may run on: the affinity mask, capped by a cgroup v2 CPU quota
    (a container's os.cpu_count() reports the whole machine; oversubscribing a quota makes
    the thread pools stall)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            quota, period = f.read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n or 1)


class CpuSample:
    """The bounded sample of the eager CPU step, built once: one decoder layer of `shape` on
    `tokens` tokens and the lm_head + CE on the same rows. run() times one sample and returns
    (layer seconds, head seconds)."""

    def __init__(self, shape, tokens=128, threads=None, seed=0):
        self.shape, self.tokens = shape, tokens
        self.threads = threads or usable_cores()
        torch.set_num_threads(self.threads)
        rng = np.random.default_rng(seed)
        torch.manual_seed(seed)
        self.layer = CpuDecoderLayer(shape, rng, self.threads)
        self.cos, self.sin = ops_ref.qwen_cos_sin(1, tokens, shape.head_dim, shape.theta,
                                                  torch.bfloat16)
        self.h0 = (torch.randn(1, tokens, shape.hidden) * 0.5).to(torch.bfloat16)
        self.head = (torch.randn(shape.vocab, shape.hidden) * 0.02).to(torch.bfloat16)
        self.labels = torch.randint(0, shape.vocab, (1, tokens))

    def run(self):
        t0 = time.perf_counter()
        with torch.no_grad():            # the checkpoint's first forward
            self.layer(self.h0, self.cos, self.sin)
        h = self.h0.clone().requires_grad_()
        out = self.layer(h, self.cos, self.sin)   # recompute in backward
        out.float().sum().backward()
        t1 = time.perf_counter()
        hn = self.h0.clone().float().requires_grad_()
        loss = ops_ref.ce_ref(hn, self.head, self.labels, matmul_dtype=torch.bfloat16)[0]
        loss.backward()
        return t1 - t0, time.perf_counter() - t1

    def scaled_tokens_per_s(self, t_layer, t_head):
        """tokens/s of the whole model's step, from one sample's layer and head times."""
        return self.tokens / (self.shape.layers * t_layer + t_head)

    def describe(self):
        s = self.shape
        return (f"1 decoder layer ({s.name} shapes) fwd + checkpoint recompute + bwd on "
                f"{self.tokens} tokens (seq {self.tokens}), NF4 rebuilt by the C oracle per "
                f"forward and backward, + lm_head/CE fwd+bwd on the same rows; the model figure "
                f"is {s.layers} x layer + head; attention at seq {self.tokens}")


def time_sample(shape, tokens=128, threads=None, repeats=1, seed=0):
    """(tokens/s scaled to the whole model, threads, description dict) of the eager CPU path:
    one warm-up sample, then `repeats` timed ones."""
    smp = CpuSample(shape, tokens, threads, seed)
    smp.run()  # warm-up (allocations, thread pools)
    tl = th = 0.0
    for _ in range(repeats):
        a, b = smp.run()
        tl += a
        th += b
    t_layer, t_head = tl / repeats, th / repeats
    desc = {"sample": smp.describe(), "tokens": tokens, "layer_s": round(t_layer, 4),
            "head_s": round(t_head, 4)}
    return smp.scaled_tokens_per_s(t_layer, t_head), smp.threads, desc
