"""torch-on-CPU restatements of the reference's floating-point ops — TEST INFRASTRUCTURE ONLY.

Each function follows the eager reference the reference's own tests compare against:
  rmsnorm_ref            solution/test_rmsnorm.py:9-14 (Qwen2RMSNorm.forward line for line)
  rope_ref               solution/test_rope.py:9-17 (apply_rotary_pos_emb, unsqueeze_dim=1)
  qwen_cos_sin           solution/test_rope.py:20-27
  swiglu_ref             solution/test_kernels.py:24-25
  scaled_add_ref         solution/test_lora.py:52 (peft: result.clone() + lo * scaling)
  ce_ref                 solution/test_cross_entropy.py:9-30 (ForCausalLMLoss + TRL entropy and
                         accuracy + Soup per-token CE); entropy is written as
                         logsumexp - sum(softmax * z) because trl is not installed
  NF4LoRALinearRef / decoder_layer_ref   the Cfg1 decoder layer: transformers' Qwen2 layer with
                         its linears replaced by an eager NF4-dequant + LoRA module
"""

import torch
import torch.nn.functional as F

from . import nf4_ref

IGNORE_INDEX = -100


def rmsnorm_ref(x, weight, eps):
    input_dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(input_dtype)


def rotate_half(x):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def rope_ref(q, k, cos, sin):
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def qwen_cos_sin(batch, seq, dim, theta=1e6, dtype=torch.float32, device="cpu"):
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
    pos = torch.arange(seq, dtype=torch.float)
    emb = torch.cat([torch.outer(pos, inv_freq)] * 2, dim=-1)
    return (emb.cos()[None].expand(batch, -1, -1).to(device, dtype),
            emb.sin()[None].expand(batch, -1, -1).to(device, dtype))


def swiglu_ref(gate, up):
    return F.silu(gate.float()) * up.float()


def scaled_add_ref(base, lo, scaling):
    return base.clone() + lo * scaling


def shift_labels(labels):
    return F.pad(labels, (0, 1), value=IGNORE_INDEX)[..., 1:]


def ce_ref(hidden, weight, labels, num_items_in_batch=None, matmul_dtype=torch.float32,
           logits=None):
    """(loss, token_entropy, token_loss, correct, labelled, pred) of the base run: logits in the
    matmul dtype, CE on the fp32 upcast, entropy over all positions, accuracy on labelled ones."""
    if logits is None:
        logits = (hidden.to(matmul_dtype) @ weight.to(matmul_dtype).t()).float()
    shift = shift_labels(labels)
    flat_logits, flat_shift = logits.reshape(-1, logits.shape[-1]), shift.reshape(-1)
    if num_items_in_batch is None:
        loss = F.cross_entropy(flat_logits, flat_shift, ignore_index=IGNORE_INDEX)
    else:
        loss = F.cross_entropy(flat_logits, flat_shift, ignore_index=IGNORE_INDEX,
                               reduction="sum") / num_items_in_batch
    with torch.no_grad():
        lse = torch.logsumexp(logits, -1)
        entropy = lse - (torch.softmax(logits, -1) * logits).sum(-1)
        token_loss = F.cross_entropy(flat_logits, flat_shift, ignore_index=IGNORE_INDEX,
                                     reduction="none").view(shift.shape)
        pred = logits.argmax(-1)
        mask = shift != IGNORE_INDEX
        correct = ((pred == shift) & mask).sum()
    return loss, entropy, token_loss, correct, mask.sum(), pred


# ------------------------------------------------------------------------------------------
# Cfg1 decoder layer on the CPU (eager reference path, also the CPU baseline of the step)


class NF4LoRALinearRef(torch.nn.Module):
    """y = x @ dequant(W).T + b + scaling * (dropout(x) @ A.T @ B.T), with the NF4 weight
    dequantised by nf4_ref (bf16) — the eager form of peft's bnb.Linear4bit forward."""

    def __init__(self, packed, absmax_q, code2, absmax2, offset, shape, bias, lora_a, lora_b,
                 scaling, blocksize=64, blocksize2=256, dtype=torch.bfloat16):
        super().__init__()
        n = shape[0] * shape[1]
        bits = nf4_ref.dequant_nf4(packed, n, absmax_q, True, code2, absmax2, offset, blocksize,
                                   blocksize2, out="bf16")
        w = torch.from_numpy(bits.view("int16").copy()).view(torch.bfloat16).view(shape)
        self.register_buffer("weight", w.to(dtype))
        self.register_buffer("bias", None if bias is None else bias.to(dtype))
        self.lora_a = torch.nn.Parameter(lora_a.float().clone())
        self.lora_b = torch.nn.Parameter(lora_b.float().clone())
        self.scaling = scaling

    def forward(self, x):
        base = F.linear(x, self.weight, self.bias)
        lo = F.linear(F.linear(x, self.lora_a.to(x.dtype)), self.lora_b.to(x.dtype))
        return base + lo * self.scaling
