"""Data parallelism for the QLoRA step: one process per GPU, every rank holds the whole frozen
NF4 model, the batch is split across ranks, and the only exchanges are
  * one scalar all-reduce of the labelled-token count, so every rank divides its loss by the
    GLOBAL count (ForCausalLMLoss's num_items_in_batch semantics) and
  * one fp32 all-reduce (sum) of the LoRA adapter gradients, which live in one flat buffer.
With the global denominator, the sum of the per-rank gradients is the gradient of the global
mean loss, so no division by the world size follows.
"""

import torch
import torch.distributed as dist

IGNORE_INDEX = -100


class AdapterGradSync:
    """Points every adapter parameter's .grad at a slice of one flat fp32 buffer and all-reduces
    that buffer (in `bucket_bytes` pieces) after the backward."""

    def __init__(self, params, group=None, bucket_bytes=256 << 20):
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("AdapterGradSync: no trainable parameters")
        dev = params[0].device
        total = sum(p.numel() for p in params)
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        off = 0
        for p in params:
            if p.dtype != torch.float32:
                raise TypeError("AdapterGradSync: adapters must be fp32 (master weights)")
            p.grad = self.flat[off: off + p.numel()].view_as(p)
            off += p.numel()
        self.group = group
        n = max(1, bucket_bytes // 4)
        self.buckets = [self.flat[i: i + n] for i in range(0, total, n)]

    def __call__(self):
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            for b in self.buckets:
                dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group)


def global_label_count(labels, group=None):
    """Number of scored positions over all ranks (labels shifted by one, -100 ignored), as a
    0-d tensor on the labels' device."""
    shifted = labels[..., 1:]
    n = (shifted != IGNORE_INDEX).sum().to(torch.float32).reshape(1)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(n, op=dist.ReduceOp.SUM, group=group)
    return n[0]


def shard_rows(n_rows, rank, world):
    """[start, stop) of this rank's rows when n_rows are split as evenly as possible."""
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
