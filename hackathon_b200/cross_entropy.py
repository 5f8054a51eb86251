"""Fused linear cross-entropy + entropy + argmax over the vocabulary without the full logits
(API of solution/cross_entropy.py).

    loss = sum over labelled rows of CE(hidden @ W.T, target) / denominator
plus per-token loss, entropy and argmax (what TRL's metrics and Soup's rewind recorder read).
The head W is frozen: the gradient of the hidden states is computed in forward, chunk by chunk,
and the backward only scales it by the incoming loss gradient (cross_entropy.py:93-138).

Rows go through in chunks of `chunk_rows`: logits_chunk = h @ W.T in the matmul dtype, then the
row kernel (qb_ce_rows) streams each row once for the statistics and rewrites it in place with
(softmax - onehot) * GRAD_GAIN / denominator, then dH_chunk = dZ @ W. Only one chunk of logits
is alive at a time.
"""

import torch

from . import _common, _lib

IGNORE_INDEX = -100
CHUNK_ROWS = 4096           # rows of logits alive at a time (4096 x 152064 bf16 = 1.2 GB)
# dz is stored in the matmul dtype before the dH matmul; it is kept multiplied by GRAD_GAIN
# (a power of two, exact) so fp16 does not underflow, and divided back in fp32 (:40-44).
GRAD_GAIN = 65536.0
STEP_ATTR = "_soup_chunked_step"


# With the gradient wanted, pass 1 also stores the chunk's fp32 logits (rows x vocab x 4 bytes of
# scratch, 2.5 GB at 4096 x 152064) and dZ comes from them in one streaming pass, instead of
# recomputing the logits GEMM (2 N H V flops) in pass 2. Same z, same arithmetic, same dZ.
STORE_LOGITS = True


def linear_ce_tc(h2, w, tgt, token_loss, entropy, pred, grad_h, scale_dev, chunk_rows,
                 store_logits=None):
    """The tcgen05 path for bf16 hidden states and head: per chunk of rows, pass 1 (logits in
    TMEM -> per-tile row statistics, and the fp32 logits when `store_logits`), the reduction,
    and with grad_h the dZ pass (from the stored logits, or a second logits GEMM with dZ in its
    epilogue) followed by dH = dZ @ W into grad_h (fp32)."""
    from .gemm import gemm
    n, hdim = h2.shape
    vocab = w.shape[0]
    dev = h2.device
    s = _lib.stream(dev)
    n_vt = int(_lib.load().qb_linear_ce_vocab_tiles(vocab))
    rows_max = min(chunk_rows, n)
    partials = torch.empty((n_vt, rows_max, 4), dtype=torch.float32, device=dev)
    z_label = torch.empty(rows_max, dtype=torch.float32, device=dev)
    lse = torch.empty(rows_max, dtype=torch.float32, device=dev)
    ldz = (vocab + 7) // 8 * 8      # 16-byte rows for the dH GEMM's TMA
    dz = torch.empty((rows_max, ldz), dtype=torch.bfloat16, device=dev) \
        if grad_h is not None else None
    keep = (STORE_LOGITS if store_logits is None else store_logits) and grad_h is not None
    ldl = (vocab + 3) // 4 * 4
    logits = torch.empty((rows_max, ldl), dtype=torch.float32, device=dev) if keep else None
    for start in range(0, n, chunk_rows):
        stop = min(start + chunk_rows, n)
        rows = stop - start
        h = h2[start:stop]
        t = tgt[start:stop]
        if keep:
            _lib.call("qb_linear_ce_stats_logits", h.data_ptr(), h.stride(0), w.data_ptr(),
                      w.stride(0), t.data_ptr(), rows, vocab, hdim, partials.data_ptr(),
                      z_label.data_ptr(), logits.data_ptr(), ldl, s,
                      work=(0, 2 * rows * vocab * hdim))
        else:
            _lib.call("qb_linear_ce_stats", h.data_ptr(), h.stride(0), w.data_ptr(), w.stride(0),
                      t.data_ptr(), rows, vocab, hdim, partials.data_ptr(), z_label.data_ptr(), s,
                      work=(0, 2 * rows * vocab * hdim))
        _lib.call("qb_ce_reduce", partials.data_ptr(), n_vt, rows, vocab, t.data_ptr(),
                  z_label.data_ptr(), token_loss[start:stop].data_ptr(),
                  entropy[start:stop].data_ptr(), pred[start:stop].data_ptr(), None,
                  lse.data_ptr(), s, work=(n_vt * rows * 16 + rows * 32, 0))
        if grad_h is None:
            continue
        if keep:
            _lib.call("qb_ce_grad_from_logits", logits.data_ptr(), ldl, t.data_ptr(), rows,
                      vocab, lse.data_ptr(), scale_dev.data_ptr(), dz.data_ptr(), dz.stride(0),
                      s, work=(rows * vocab * (4 + 2), 0))
        else:
            _lib.call("qb_linear_ce_grad", h.data_ptr(), h.stride(0), w.data_ptr(), w.stride(0),
                      t.data_ptr(), rows, vocab, hdim, lse.data_ptr(), scale_dev.data_ptr(),
                      dz.data_ptr(), dz.stride(0), s, work=(0, 2 * rows * vocab * hdim))
        gemm(dz[:rows, :vocab], w.t(), out=grad_h[start:stop], out_dtype=torch.float32)


def tc_path_ok(h2, w, matmul_dtype):
    return (matmul_dtype == torch.bfloat16 and h2.is_cuda and w.is_cuda
            and h2.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and h2.shape[1] % 8 == 0 and w.stride(-1) == 1 and h2.stride(-1) == 1
            and w.stride(0) % 8 == 0 and h2.stride(0) % 8 == 0)


def ce_rows_inplace(logits, target, token_loss, entropy, pred, grad_scale, write_grad):
    """Runs the row kernel on a [rows, vocab] logits chunk (rewritten in place with the scaled
    gradient when write_grad)."""
    rows, vocab = logits.shape
    _lib.call("qb_ce_rows", logits.data_ptr(), _lib.tag(logits.dtype), logits.stride(0),
              target.data_ptr(), rows, vocab, token_loss.data_ptr(), entropy.data_ptr(),
              _lib.ptr(pred), None, float(grad_scale), int(write_grad),
              _lib.stream(logits.device),
              work=(rows * vocab * logits.element_size() * (3 if write_grad else 1), 0))


class FusedLinearCrossEntropy(torch.autograd.Function):
    """loss, per-token loss, entropy, argmax of CE(hidden @ W.T, target), W frozen."""

    @staticmethod
    def forward(ctx, hidden, weight, target, denominator, matmul_dtype, chunk_rows):
        _lib.require_cuda(hidden, weight, what="fused linear CE")
        shape = hidden.shape
        h2 = hidden.reshape(-1, shape[-1])
        tgt = target.reshape(-1).to(device=hidden.device, dtype=torch.int64).contiguous()
        n_rows = h2.shape[0]
        dev = hidden.device
        with_grad = ctx.needs_input_grad[0]

        token_loss = torch.empty(n_rows, dtype=torch.float32, device=dev)
        entropy = torch.empty(n_rows, dtype=torch.float32, device=dev)
        pred = torch.empty(n_rows, dtype=torch.int64, device=dev)
        grad_h = torch.empty((n_rows, shape[-1]), dtype=torch.float32, device=dev) \
            if with_grad else None
        w_mm = weight if weight.dtype == matmul_dtype else weight.to(matmul_dtype)
        h_mm = h2 if h2.dtype == matmul_dtype else h2.to(matmul_dtype)
        if tc_path_ok(h_mm, w_mm, matmul_dtype):
            # the gradient scale stays on the device: no host sync on the denominator
            d = torch.as_tensor(denominator, dtype=torch.float32, device=dev).reshape(1)
            scale_dev = torch.where(d != 0, GRAD_GAIN / d, torch.zeros_like(d))
            linear_ce_tc(h_mm, w_mm, tgt, token_loss, entropy, pred, grad_h, scale_dev,
                         chunk_rows)
            loss = token_loss.sum() / denominator
            ctx.save_for_backward(grad_h)
            ctx.shape, ctx.dtype = shape, hidden.dtype
            ctx.mark_non_differentiable(token_loss, entropy, pred)
            return (loss, token_loss.view(shape[:-1]), entropy.view(shape[:-1]),
                    pred.view(shape[:-1]))
        denom = float(denominator)
        grad_scale = GRAD_GAIN / denom if denom else 0.0
        with torch.autocast(device_type=dev.type, enabled=False):
            w = weight if weight.dtype == matmul_dtype else weight.to(matmul_dtype)
            for start in range(0, n_rows, chunk_rows):
                stop = min(start + chunk_rows, n_rows)
                logits = h2[start:stop].to(matmul_dtype) @ w.t()
                ce_rows_inplace(logits, tgt[start:stop], token_loss[start:stop],
                                entropy[start:stop], pred[start:stop], grad_scale, with_grad)
                if with_grad:
                    grad_h[start:stop] = logits @ w   # logits now hold dz * GRAD_GAIN / denom
                del logits
        loss = token_loss.sum() / denominator
        ctx.save_for_backward(grad_h)
        ctx.shape, ctx.dtype = shape, hidden.dtype
        ctx.mark_non_differentiable(token_loss, entropy, pred)
        return loss, token_loss.view(shape[:-1]), entropy.view(shape[:-1]), pred.view(shape[:-1])

    @staticmethod
    def backward(ctx, grad_loss, _grad_token_loss, _grad_entropy, _grad_pred):
        (grad_h,) = ctx.saved_tensors
        if grad_h is None:
            return None, None, None, None, None, None
        grad = grad_h * (grad_loss.float() / GRAD_GAIN)
        return grad.view(ctx.shape).to(ctx.dtype), None, None, None, None, None


class ChunkedStep:
    """What the fused forward leaves for the metrics: the fields of Soup's
    stream_loss_chunk.ChunkedStep (cross_entropy.py:141-150)."""

    def __init__(self, token_entropy, token_loss, pred, target):
        self.token_entropy = token_entropy
        self.token_loss = token_loss
        labelled = target != IGNORE_INDEX
        self.labelled = labelled.sum()
        self.correct = ((pred == target) & labelled).sum()


def shift_labels_of(labels):
    """Labels moved one left, as ForCausalLMLoss does (the last position scores nothing)."""
    return torch.nn.functional.pad(labels, (0, 1), value=IGNORE_INDEX)[..., 1:]


def fused_causal_lm_loss(hidden, weight, labels, num_items_in_batch=None, shift_labels=None,
                         chunk_rows=CHUNK_ROWS):
    """ForCausalLMLoss(hidden @ weight.T, labels) and a ChunkedStep, without the full logits
    (cross_entropy.py:158-172)."""
    target = shift_labels if shift_labels is not None else shift_labels_of(labels)
    target = target.to(hidden.device)
    if num_items_in_batch is None:      # mean over labelled tokens
        denominator = (target != IGNORE_INDEX).sum()
    elif torch.is_tensor(num_items_in_batch):
        denominator = num_items_in_batch.to(hidden.device)
    else:
        denominator = num_items_in_batch
    matmul_dtype = _common.autocast_dtype() or torch.promote_types(hidden.dtype, weight.dtype)
    loss, token_loss, entropy, pred = FusedLinearCrossEntropy.apply(
        hidden, weight, target, denominator, matmul_dtype, chunk_rows)
    return loss, ChunkedStep(entropy, token_loss, pred, target)


class _State:
    armed = False   # set by the patched compute_loss for exactly one model forward
    step = None


STATE = _State()


def _head_ok(lm):
    head = getattr(lm, "lm_head", None)
    return (type(head) is torch.nn.Linear and head.bias is None
            and not head.weight.requires_grad and _common.on_gpu(head.weight)
            and getattr(lm.config, "final_logit_softcapping", None) is None)


def _patch_causal_lm():
    """Qwen2ForCausalLM.forward returns the fused loss and logits=None when armed
    (cross_entropy.py:190-222)."""
    from transformers.modeling_outputs import CausalLMOutputWithPast
    from transformers.models.qwen2 import modeling_qwen2 as m

    original = m.Qwen2ForCausalLM.forward
    if getattr(original, "_solution_patch", False):
        return

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, labels=None, use_cache=None,
                logits_to_keep=0, **kwargs):
        if not (STATE.armed and labels is not None and _common.on_gpu(labels)
                and isinstance(logits_to_keep, int) and logits_to_keep == 0
                and kwargs.get("return_dict", True) is not False and _head_ok(self)):
            return original(self, input_ids=input_ids, attention_mask=attention_mask,
                            position_ids=position_ids, past_key_values=past_key_values,
                            inputs_embeds=inputs_embeds, labels=labels, use_cache=use_cache,
                            logits_to_keep=logits_to_keep, **kwargs)
        STATE.armed = False
        outputs = self.model(input_ids=input_ids, attention_mask=attention_mask,
                             position_ids=position_ids, past_key_values=past_key_values,
                             inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
        loss, STATE.step = fused_causal_lm_loss(
            outputs.last_hidden_state, self.lm_head.weight, labels,
            num_items_in_batch=kwargs.get("num_items_in_batch"),
            shift_labels=kwargs.get("shift_labels"))
        return CausalLMOutputWithPast(loss=loss, logits=None,
                                      past_key_values=outputs.past_key_values,
                                      hidden_states=outputs.hidden_states,
                                      attentions=outputs.attentions)

    forward._solution_patch = True
    m.Qwen2ForCausalLM.forward = forward


def _causal_lm_of(trainer, model):
    unwrap = getattr(getattr(trainer, "accelerator", None), "unwrap_model", None)
    inner = unwrap(model) if callable(unwrap) else model
    get_base = getattr(inner, "get_base_model", None)
    return get_base() if callable(get_base) else inner


def _can_fuse(trainer, model, inputs):
    """The trainer-state checks of cross_entropy.py:232-256."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2ForCausalLM

    args = getattr(trainer, "args", None)
    if not (isinstance(model, torch.nn.Module) and isinstance(inputs, dict) and args is not None):
        return False
    if not getattr(trainer.model, "training", False):
        return False
    if "labels" not in inputs or "shift_labels" in inputs or "attention_mask" not in inputs:
        return False
    if not _common.on_gpu(inputs["labels"], inputs["attention_mask"]):
        return False
    if getattr(args, "use_liger_kernel", False) or getattr(args, "loss_type", "nll") != "nll":
        return False
    if getattr(trainer, "num_virtual_tokens", 0) or getattr(trainer, "aux_loss_enabled", False):
        return False
    if getattr(trainer, "compute_loss_func", None) is not None or \
            getattr(trainer, "label_smoother", None) is not None:
        return False
    if getattr(trainer, "_soup_chunked_head_loss", None) is not None:
        return False
    if not all(hasattr(trainer, name) for name in ("_metrics", "_total_train_tokens")):
        return False
    lm = _causal_lm_of(trainer, model)
    return isinstance(lm, Qwen2ForCausalLM) and _head_ok(lm)


def _log_metrics(trainer, mode, inputs, step):
    """entropy, num_tokens and mean_token_accuracy by TRL's formulas (cross_entropy.py:259-276)."""
    gather = trainer.accelerator.gather_for_metrics
    attention_mask = inputs["attention_mask"]
    with torch.no_grad():
        entropy = torch.sum(step.token_entropy * attention_mask) / attention_mask.sum()
        entropy = gather(entropy).mean().item()
    trainer._metrics[mode]["entropy"].append(entropy)
    if mode == "train":
        trainer._total_train_tokens += gather(attention_mask.sum()).sum().item()
    trainer._metrics[mode]["num_tokens"] = [trainer._total_train_tokens]
    with torch.no_grad():
        correct = gather(step.correct)
        total = gather(step.labelled)
        total_sum = total.sum()
        accuracy = (correct.sum() / total_sum).item() if total_sum > 0 else 0.0
    trainer._metrics[mode]["mean_token_accuracy"].append(accuracy)


def _patch_trainer():
    """trl.SFTTrainer.compute_loss arms the fused forward and logs TRL's metrics from the kernel
    outputs (cross_entropy.py:279-316). A no-op when trl is not installed."""
    try:
        from trl import SFTTrainer
    except ImportError:
        return

    original = SFTTrainer.compute_loss
    if getattr(original, "_solution_patch", False):
        return

    def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
        if not _can_fuse(self, model, inputs):
            return original(self, model, inputs, return_outputs=return_outputs,
                            num_items_in_batch=num_items_in_batch)
        mode = "train" if self.model.training else "eval"
        inputs.pop("_prediction_loss_only", None)
        labels = inputs["labels"]
        inputs["use_cache"] = False
        STATE.armed, STATE.step = True, None
        try:
            loss, outputs = super(SFTTrainer, self).compute_loss(
                model, inputs, return_outputs=True, num_items_in_batch=num_items_in_batch)
        finally:
            STATE.armed = False
        step, STATE.step = STATE.step, None
        if step is None:
            from trl.trainer.utils import entropy_from_logits

            with torch.no_grad():
                logits = outputs.logits
                step = ChunkedStep(entropy_from_logits(logits), None, logits.argmax(dim=-1),
                                   shift_labels_of(labels))
            setattr(self, STEP_ATTR, None)
        else:
            setattr(self, STEP_ATTR, step)
        _log_metrics(self, mode, inputs, step)
        return (loss, outputs) if return_outputs else loss

    compute_loss._solution_patch = True
    SFTTrainer.compute_loss = compute_loss


def patch():
    _patch_causal_lm()
    _patch_trainer()
