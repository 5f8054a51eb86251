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
    it in buckets of about `bucket_bytes`, overlapped with the backward: each bucket is a run
    of consecutive parameters (whole parameters, in their order), and once the backward has
    accumulated the gradient of every parameter of a bucket (a post-accumulate-grad hook per
    parameter), its all-reduce is issued asynchronously - NCCL orders it after the gradient
    kernels on the current stream and runs it on its own stream while the backward goes on
    with earlier layers. Calling the object after the backward issues what is still pending
    (buckets whose parameters got no gradient) and makes the current stream wait for every
    reduction, so the optimizer reads the summed gradients.

    Each parameter must receive one gradient accumulation per backward (as the step's adapters
    do); a second one after its bucket was reduced raises. overlap=False reduces everything
    after the backward instead."""

    def __init__(self, params, group=None, bucket_bytes=32 << 20, overlap=True):
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("AdapterGradSync: no trainable parameters")
        dev = params[0].device
        total = sum(p.numel() for p in params)
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        self.group = group
        self.buckets = []           # (flat slice, number of parameters)
        bucket_of = {}
        off = start = count = 0
        limit = max(1, bucket_bytes // 4)
        for p in params:
            if p.dtype != torch.float32:
                raise TypeError("AdapterGradSync: adapters must be fp32 (master weights)")
            p.grad = self.flat[off: off + p.numel()].view_as(p)
            off += p.numel()
            bucket_of[p] = len(self.buckets)
            count += 1
            if off - start >= limit:
                self.buckets.append((self.flat[start:off], count))
                start, count = off, 0
        if count:
            self.buckets.append((self.flat[start:off], count))
        self.overlap = overlap and self._world() > 1
        self._seen = [0] * len(self.buckets)
        self._work = [None] * len(self.buckets)
        if self.overlap:
            for p in params:
                p.register_post_accumulate_grad_hook(self._hook(bucket_of[p]))

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def _launch(self, i):
        self._work[i] = dist.all_reduce(self.buckets[i][0], op=dist.ReduceOp.SUM,
                                        group=self.group, async_op=True)

    def _hook(self, i):
        def on_grad(param):
            if self._work[i] is not None:
                raise RuntimeError("AdapterGradSync: a gradient accumulated into bucket "
                                   f"{i} after its all-reduce was issued")
            self._seen[i] += 1
            if self._seen[i] == self.buckets[i][1]:
                self._launch(i)
        return on_grad

    def __call__(self):
        if self._world() <= 1:
            return
        for i in range(len(self.buckets)):
            if self._work[i] is None:
                self._launch(i)
        for i, w in enumerate(self._work):
            w.wait()
            self._work[i] = None
            self._seen[i] = 0


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
