"""The output head and the loss without the full logits: the earlier API of the reference
(solution/fused_ce.py), on the same kernels as cross_entropy.py.

  ce_rows(logits, target, write_grad)           per-row loss / entropy / correct of a logits
                                                block (the row kernel), optionally rewriting it
                                                with softmax - onehot (fused_ce.py:99-109)
  FusedLinearCE.apply(hidden, weight16, target, n_labelled, denominator)
                                                rows -> sum of their CE / denominator
                                                (fused_ce.py:112-158)
  fused_head_loss(hidden, weight, labels, attention_mask, num_items_in_batch)
                                                ForCausalLMLoss(lm_head(hidden), labels) and the
                                                metric inputs as Stats (fused_ce.py:178-219)
  patch_qwen2_causal_lm(), patch_sft_trainer()  the framework hooks (hooks.py)

Here the rows are never reordered: each row's target (IGNORE for unlabelled ones) decides
whether it scores and has a gradient, so the kernel path is the one of fused_causal_lm_loss (the
custom op qlora_b200::linear_ce). With an attention mask only the labelled and the real rows run
(one device->host read of their count); without one every row runs and nothing is read back.
A bf16 head runs on the tcgen05 kernels; any other runs in fp16, as the reference's does.
"""

import torch

from . import _lib, hooks, ops  # noqa: F401 - ops registers the custom operators
from .cross_entropy import CHUNK_ROWS, IGNORE_INDEX, shift_labels_of

IGNORE = IGNORE_INDEX
STEP_ATTR = hooks.STEP_ATTR


def ce_rows(logits, target, write_grad):
    """Per-row loss, entropy and correct flag (int32) of [n, vocab] logits; with write_grad the
    logits are overwritten by softmax - onehot (zero rows for IGNORE targets)."""
    _lib.require_cuda(logits, target, what="ce_rows")
    n, vocab = logits.shape
    dev = logits.device
    loss = torch.empty(n, dtype=torch.float32, device=dev)
    entropy = torch.empty(n, dtype=torch.float32, device=dev)
    correct = torch.empty(n, dtype=torch.int32, device=dev)
    if n:
        tgt = target.to(torch.int64).contiguous()
        _lib.call("qb_ce_rows", logits.data_ptr(), _lib.tag(logits.dtype), logits.stride(0),
                  tgt.data_ptr(), n, vocab, loss.data_ptr(), entropy.data_ptr(), None,
                  correct.data_ptr(), 1.0, int(write_grad), _lib.stream(dev))
    return loss, entropy, correct


class FusedLinearCE:
    """Rows of hidden states [n, H] -> (sum of their CE / denominator, per-row loss, entropy,
    correct). Rows whose target is IGNORE score nothing (the reference's rows past n_labelled,
    an argument this signature keeps); the gradient of the hidden states comes from the
    registered backward of qlora_b200::linear_ce."""

    @staticmethod
    def apply(hidden, weight16, target, n_labelled, denominator):
        _lib.require_cuda(hidden, weight16, what="FusedLinearCE")
        h = hidden if hidden.dtype == weight16.dtype else hidden.to(weight16.dtype)
        tgt = target.to(device=hidden.device, dtype=torch.int64)
        with_grad = torch.is_grad_enabled() and hidden.requires_grad
        loss, entropy, pred, _ = torch.ops.qlora_b200.linear_ce(h, weight16, tgt, CHUNK_ROWS,
                                                                 with_grad)
        correct = ((pred == tgt) & (tgt != IGNORE)).to(torch.int32)
        return loss.sum() / denominator, loss, entropy, correct


class Stats:
    """What the trainer's metrics read, on the device: per-token loss [B, S], the entropy summed
    over real tokens, and the correct / labelled counts."""

    __slots__ = ("token_loss", "entropy_sum", "correct", "labelled")

    def __init__(self, token_loss, entropy_sum, correct, labelled):
        self.token_loss, self.entropy_sum = token_loss, entropy_sum
        self.correct, self.labelled = correct, labelled


def fused_head_loss(hidden, weight, labels, attention_mask, num_items_in_batch):
    """ForCausalLMLoss(hidden @ weight.T, labels) - sum over labelled next-token targets divided
    by num_items_in_batch, or by their count - and Stats, without the logits."""
    B, S, H = hidden.shape
    dev = hidden.device
    target = shift_labels_of(labels.to(dev)).reshape(-1)
    labelled = target != IGNORE
    denominator = labelled.sum() if num_items_in_batch is None else (
        num_items_in_batch.to(dev) if torch.is_tensor(num_items_in_batch) else num_items_in_batch)
    h2 = hidden.reshape(B * S, H)
    mask = None if attention_mask is None else attention_mask.to(dev).reshape(-1)
    # the rows that run: every labelled row, and the real (unmasked) unlabelled ones
    rows = None if mask is None else ((mask != 0) | labelled).nonzero().squeeze(1)
    if rows is not None:
        h2, tgt = h2.index_select(0, rows), target.index_select(0, rows)
    else:
        tgt = target
    w = weight.detach()
    if w.dtype not in (torch.float16, torch.bfloat16):
        w = w.to(torch.float16)     # the reference's fp16 head; bf16 stays on the tcgen05 path
    loss, row_loss, row_entropy, row_correct = FusedLinearCE.apply(h2, w, tgt, None, denominator)
    with torch.no_grad():
        if rows is None:
            token_loss, token_entropy = row_loss, row_entropy
        else:
            token_loss = row_loss.new_zeros(B * S).index_copy_(0, rows, row_loss)
            token_entropy = row_entropy.new_zeros(B * S).index_copy_(0, rows, row_entropy)
        entropy_sum = token_entropy.sum() if mask is None else (token_entropy * mask).sum()
        stats = Stats(token_loss=token_loss.view(B, S), entropy_sum=entropy_sum,
                      correct=row_correct.sum(), labelled=labelled.sum())
    return loss, stats


def _head_loss_for_hook(hidden, head_weight, labels, attention_mask, kwargs):
    return fused_head_loss(hidden, head_weight, labels, attention_mask,
                           kwargs.get("num_items_in_batch"))


def patch_qwen2_causal_lm():
    """Qwen2ForCausalLM.forward on the fused head loss while a trainer hook has armed it
    (fused_ce.py:249-282)."""
    hooks.install_causal_lm()


def patch_sft_trainer():
    """trl.SFTTrainer.compute_loss arming fused_head_loss for its model forward; the Stats are
    left on the trainer (fused_ce.py:306-355). Needs trl (ImportError otherwise, as in the
    reference)."""
    hooks.install_trainer(_head_loss_for_hook)
