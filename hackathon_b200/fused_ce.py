"""The output head and the loss without the full logits: the earlier API of the reference
(solution/fused_ce.py), on the same row kernel as cross_entropy.py.

fused_head_loss keeps only the rows that matter — labelled positions first, then real
(attention_mask != 0) unlabelled ones for the entropy metric; padding is dropped — runs the head
in chunks of CHUNK rows into one reused buffer, and takes the gradient of the hidden states in
forward; the backward only scales it (fused_ce.py:112-219).
"""

import torch

from . import _lib

CHUNK = 512
IGNORE = -100

try:  # the attribute Soup's rewind recorder reads when a step has no logits
    from soup_cli.utils.stream_loss_chunk import STEP_ATTR
except Exception:  # noqa: BLE001
    STEP_ATTR = "_soup_chunked_step"


def ce_rows(logits, target, write_grad):
    """Per-row loss, entropy and correct flag of [n, vocab] logits; with write_grad the logits
    are overwritten by softmax - onehot (0 rows for unlabelled targets) (fused_ce.py:99-109)."""
    _lib.require_cuda(logits, target, what="ce_rows")
    n, vocab = logits.shape
    loss = torch.empty(n, dtype=torch.float32, device=logits.device)
    entropy = torch.empty(n, dtype=torch.float32, device=logits.device)
    correct = torch.empty(n, dtype=torch.int32, device=logits.device)
    if n:
        tgt = target.to(torch.int64).contiguous()
        _lib.call("qb_ce_rows", logits.data_ptr(), _lib.tag(logits.dtype), logits.stride(0),
                  tgt.data_ptr(), n, vocab, loss.data_ptr(), entropy.data_ptr(), None,
                  correct.data_ptr(), 1.0, int(write_grad), _lib.stream(logits.device))
    return loss, entropy, correct


class FusedLinearCE(torch.autograd.Function):
    """Rows of hidden states [n, hidden] -> sum of their cross-entropies / denominator.
    Rows [0, n_labelled) have a label; the rest only feed the metrics."""

    @staticmethod
    def forward(ctx, hidden, weight16, target, n_labelled, denominator):
        n, width = hidden.shape
        vocab = weight16.shape[0]
        with_grad = ctx.needs_input_grad[0]
        hidden16 = hidden.to(weight16.dtype)
        grad = torch.zeros((n, width), dtype=torch.float32, device=hidden.device) \
            if with_grad else None
        buffer = torch.empty((min(CHUNK, max(n, 1)), vocab), dtype=weight16.dtype,
                             device=hidden.device)
        losses, entropies, corrects = [], [], []
        with torch.autocast(hidden.device.type, enabled=False):
            for start in range(0, n, CHUNK):
                stop = min(n, start + CHUNK)
                logits = buffer[: stop - start]
                torch.mm(hidden16[start:stop], weight16.t(), out=logits)
                labelled = max(0, min(stop, n_labelled) - start)
                write_grad = with_grad and labelled > 0
                loss, entropy, correct = ce_rows(logits, target[start:stop], write_grad)
                losses.append(loss)
                entropies.append(entropy)
                corrects.append(correct)
                if write_grad:
                    grad[start:start + labelled] = torch.mm(logits[:labelled], weight16)
        del buffer
        row_loss = torch.cat(losses) if losses else hidden.new_zeros(0, dtype=torch.float32)
        row_entropy = torch.cat(entropies) if entropies else row_loss
        row_correct = torch.cat(corrects) if corrects else row_loss.int()
        total = row_loss.sum() / denominator
        if with_grad:
            grad /= denominator
            ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(row_loss, row_entropy, row_correct)
        return total, row_loss, row_entropy, row_correct

    @staticmethod
    def backward(ctx, grad_total, _l, _e, _c):
        (grad,) = ctx.saved_tensors
        return grad * grad_total, None, None, None, None


class Stats:
    __slots__ = ("token_loss", "entropy_sum", "correct", "labelled")

    def __init__(self, token_loss, entropy_sum, correct, labelled):
        self.token_loss, self.entropy_sum = token_loss, entropy_sum
        self.correct, self.labelled = correct, labelled


class _Step:
    """What Soup's rewind recorder reads for a step without logits."""

    __slots__ = ("token_loss",)

    def __init__(self, token_loss):
        self.token_loss = token_loss


def fused_head_loss(hidden, weight, labels, attention_mask, num_items_in_batch):
    """ForCausalLMLoss(lm_head(hidden), labels) and TRL's metric inputs without the logits
    (fused_ce.py:178-219). The head runs in fp16, as autocast makes it in the base run."""
    batch, seq, width = hidden.shape
    device = hidden.device
    labels = labels.to(device)
    target = torch.nn.functional.pad(labels, (0, 1), value=IGNORE)[:, 1:].reshape(-1)
    has_label = target != IGNORE
    if attention_mask is None:
        real = torch.ones_like(has_label)
    else:
        real = attention_mask.to(device).reshape(-1) != 0
    other = real & ~has_label
    label_rows = has_label.nonzero().squeeze(1)
    other_rows = other.nonzero().squeeze(1)
    rows = torch.cat([label_rows, other_rows])
    n_labelled = label_rows.numel()

    if num_items_in_batch is None:
        denominator = torch.tensor(float(n_labelled), device=device)
    elif torch.is_tensor(num_items_in_batch):
        denominator = num_items_in_batch.to(device)
    else:
        denominator = num_items_in_batch

    weight16 = weight if weight.dtype == torch.float16 else weight.detach().to(torch.float16)
    picked = hidden.reshape(-1, width).index_select(0, rows)
    loss, row_loss, row_entropy, row_correct = FusedLinearCE.apply(
        picked, weight16, target.index_select(0, rows), n_labelled, denominator)

    with torch.no_grad():
        token_loss = torch.zeros(batch * seq, dtype=torch.float32, device=device)
        token_loss.index_copy_(0, rows, row_loss)
        token_entropy = torch.zeros(batch * seq, dtype=torch.float32, device=device)
        token_entropy.index_copy_(0, rows, row_entropy)
        if attention_mask is None:
            entropy_sum = token_entropy.sum()
        else:
            entropy_sum = (token_entropy * attention_mask.to(device).reshape(-1)).sum()
        stats = Stats(token_loss=token_loss.view(batch, seq), entropy_sum=entropy_sum,
                      correct=row_correct[:n_labelled].sum(),
                      labelled=torch.tensor(n_labelled, device=device))
    return loss, stats


class _State:
    active = False
    stats = None


STATE = _State()
_ORIGINAL = {}


def _causal_lm(model):
    get_base_model = getattr(model, "get_base_model", None)
    return get_base_model() if callable(get_base_model) else model


def _head_fits(causal_lm):
    from transformers.models.qwen2 import modeling_qwen2

    if not isinstance(causal_lm, modeling_qwen2.Qwen2ForCausalLM):
        return False
    head = getattr(causal_lm, "lm_head", None)
    weight = getattr(head, "weight", None)
    return (type(head) is torch.nn.Linear and head.bias is None and weight is not None
            and not weight.requires_grad and weight.is_cuda
            and weight.dtype in (torch.float32, torch.float16)
            and getattr(causal_lm.config, "final_logit_softcapping", None) is None)


def patch_qwen2_causal_lm():
    """Qwen2ForCausalLM.forward -> fused_head_loss while STATE.active (fused_ce.py:249-282)."""
    from transformers.modeling_outputs import CausalLMOutputWithPast
    from transformers.models.qwen2 import modeling_qwen2

    cls = modeling_qwen2.Qwen2ForCausalLM
    if "causal_forward" in _ORIGINAL:
        return
    original = cls.forward
    _ORIGINAL["causal_forward"] = original

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, labels=None, use_cache=None,
                logits_to_keep=0, **kwargs):
        if (not STATE.active or labels is None or not self.training
                or not (isinstance(logits_to_keep, int) and logits_to_keep == 0)
                or kwargs.get("shift_labels") is not None or kwargs.get("return_dict") is False
                or not _head_fits(self)):
            return original(self, input_ids=input_ids, attention_mask=attention_mask,
                            position_ids=position_ids, past_key_values=past_key_values,
                            inputs_embeds=inputs_embeds, labels=labels, use_cache=use_cache,
                            logits_to_keep=logits_to_keep, **kwargs)
        kwargs.pop("return_dict", None)
        outputs = self.model(input_ids=input_ids, attention_mask=attention_mask,
                             position_ids=position_ids, past_key_values=past_key_values,
                             inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
        loss, STATE.stats = fused_head_loss(outputs.last_hidden_state, self.lm_head.weight,
                                            labels, attention_mask,
                                            kwargs.get("num_items_in_batch"))
        return CausalLMOutputWithPast(loss=loss, logits=None,
                                      past_key_values=outputs.past_key_values,
                                      hidden_states=outputs.hidden_states,
                                      attentions=outputs.attentions)

    cls.forward = forward


def _can_fuse(trainer, model, inputs):
    args = getattr(trainer, "args", None)
    if args is None or not isinstance(model, torch.nn.Module) or not model.training:
        return False
    if getattr(args, "use_liger_kernel", False) or getattr(args, "loss_type", "nll") != "nll":
        return False
    if getattr(trainer, "compute_loss_func", None) is not None:
        return False
    if getattr(trainer, "label_smoother", None) is not None:
        return False
    if getattr(trainer, "num_virtual_tokens", 0) or getattr(trainer, "aux_loss_enabled", False):
        return False
    if not hasattr(trainer, "_metrics") or not hasattr(trainer, "_total_train_tokens"):
        return False
    if not isinstance(inputs, dict) or "labels" not in inputs or "attention_mask" not in inputs:
        return False
    if "shift_labels" in inputs:
        return False
    return _head_fits(_causal_lm(model))


def patch_sft_trainer():
    """trl.SFTTrainer.compute_loss on the fused head loss, logging TRL's metrics by TRL's
    formulas (fused_ce.py:306-355). Needs trl (ImportError otherwise, as in the reference)."""
    import trl
    from transformers import Trainer

    cls = trl.SFTTrainer
    if "compute_loss" in _ORIGINAL:
        return
    original = cls.compute_loss
    _ORIGINAL["compute_loss"] = original

    def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
        if not _can_fuse(self, model, inputs):
            if getattr(self, STEP_ATTR, None) is not None:
                setattr(self, STEP_ATTR, None)
            return original(self, model, inputs, return_outputs=return_outputs,
                            num_items_in_batch=num_items_in_batch)
        mode = "train"
        inputs.pop("_prediction_loss_only", None)
        inputs["use_cache"] = False
        STATE.active, STATE.stats = True, None
        try:
            loss, outputs = Trainer.compute_loss(self, model, inputs, return_outputs=True,
                                                 num_items_in_batch=num_items_in_batch)
        finally:
            STATE.active = False
        stats, STATE.stats = STATE.stats, None
        if stats is None:
            raise RuntimeError("solution: the fused head loss did not run in this step")
        gather = self.accelerator.gather_for_metrics
        attention_mask = inputs["attention_mask"]
        with torch.no_grad():
            entropy = stats.entropy_sum / attention_mask.sum()
            entropy = gather(entropy).mean().item()
        self._metrics[mode]["entropy"].append(entropy)
        num_tokens_in_batch = gather(attention_mask.sum()).sum().item()
        self._total_train_tokens += num_tokens_in_batch
        self._metrics[mode]["num_tokens"] = [self._total_train_tokens]
        with torch.no_grad():
            correct_tokens = gather(stats.correct)
            total_tokens = gather(stats.labelled)
            total_sum = total_tokens.sum()
            accuracy = (correct_tokens.sum() / total_sum).item() if total_sum > 0 else 0.0
        self._metrics[mode]["mean_token_accuracy"].append(accuracy)
        setattr(self, STEP_ATTR, _Step(stats.token_loss))
        return (loss, outputs) if return_outputs else loss

    cls.compute_loss = compute_loss
