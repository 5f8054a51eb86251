"""The two framework hooks the fused head loss needs, shared by cross_entropy.patch() and
fused_ce.patch_qwen2_causal_lm() / patch_sft_trainer():

  causal LM   Qwen2ForCausalLM.forward, when a trainer has armed it for the next forward,
              returns the fused loss with logits=None (the [tokens, vocab] logits never exist)
  trainer     trl.SFTTrainer.compute_loss arms it for exactly one model forward and keeps what
              the fused loss left - device tensors only: per-token loss, entropy, argmax and
              counts - on the trainer (the attribute Soup's rewind recorder reads, and
              `fused_loss_step`)

Trainer-side metric formulas (TRL's entropy / accuracy / token counts) are trainer bookkeeping,
outside this package's kernels: nothing here reads a device value back to the host. A call
the fused loss does not take goes to the unpatched upstream method unchanged.
"""

import torch

from . import _common

try:  # the attribute Soup's rewind recorder reads when a step has no logits
    from soup_cli.utils.stream_loss_chunk import STEP_ATTR
except Exception:  # noqa: BLE001 - soup is not installed here
    STEP_ATTR = "_soup_chunked_step"


class Armed:
    """The fused loss the next causal-LM forward computes (set by the trainer hook)."""
    loss_fn = None     # (hidden, head_weight, labels, attention_mask, kwargs) -> (loss, step)
    step = None        # what that forward's fused loss left


ARMED = Armed()


def head_fits(lm):
    """A bias-free, frozen, CUDA nn.Linear head without logit soft-capping: what the fused loss
    computes exactly."""
    head = getattr(lm, "lm_head", None)
    w = getattr(head, "weight", None)
    return (type(head) is torch.nn.Linear and head.bias is None and w is not None
            and not w.requires_grad and _common.on_gpu(w)
            and getattr(lm.config, "final_logit_softcapping", None) is None)


def install_causal_lm():
    """Qwen2ForCausalLM.forward: with a loss armed, labels on the GPU, every logit requested
    (logits_to_keep 0) and a head that fits, the decoder runs as usual and the armed fused loss
    replaces lm_head + ForCausalLMLoss; the output has logits=None."""
    from transformers.modeling_outputs import CausalLMOutputWithPast
    from transformers.models.qwen2 import modeling_qwen2 as m

    def build(original):
        def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                    past_key_values=None, inputs_embeds=None, labels=None, use_cache=None,
                    logits_to_keep=0, **kwargs):
            fn = ARMED.loss_fn
            if (fn is None or labels is None or not _common.on_gpu(labels)
                    or not (isinstance(logits_to_keep, int) and logits_to_keep == 0)
                    or kwargs.get("return_dict", True) is False or not head_fits(self)):
                return original(self, input_ids=input_ids, attention_mask=attention_mask,
                                position_ids=position_ids, past_key_values=past_key_values,
                                inputs_embeds=inputs_embeds, labels=labels,
                                use_cache=use_cache, logits_to_keep=logits_to_keep, **kwargs)
            ARMED.loss_fn = None     # one forward per arming
            kwargs.pop("return_dict", None)
            fwd_kwargs = {k: v for k, v in kwargs.items()
                          if k not in ("num_items_in_batch", "shift_labels")}
            out = self.model(input_ids=input_ids, attention_mask=attention_mask,
                             position_ids=position_ids, past_key_values=past_key_values,
                             inputs_embeds=inputs_embeds, use_cache=use_cache, **fwd_kwargs)
            loss, ARMED.step = fn(out.last_hidden_state, self.lm_head.weight, labels,
                                  attention_mask, kwargs)
            return CausalLMOutputWithPast(loss=loss, logits=None,
                                          past_key_values=out.past_key_values,
                                          hidden_states=out.hidden_states,
                                          attentions=out.attentions)
        return forward

    _common.install(m.Qwen2ForCausalLM, "forward", build)


def _inner_lm(trainer, model):
    unwrap = getattr(getattr(trainer, "accelerator", None), "unwrap_model", None)
    lm = unwrap(model) if callable(unwrap) else model
    base = getattr(lm, "get_base_model", None)
    return base() if callable(base) else lm


def trainer_takes_fused(trainer, model, inputs):
    """The SFTTrainer configurations whose loss is plain next-token NLL over a Qwen2 causal LM
    with a head that fits: training, labels and attention mask on the GPU, no shift_labels,
    no Liger kernels, no custom loss / label smoothing / prompt tuning / aux loss."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2ForCausalLM
    args = getattr(trainer, "args", None)
    if args is None or not isinstance(inputs, dict) or not isinstance(model, torch.nn.Module):
        return False
    if not getattr(getattr(trainer, "model", None), "training", False):
        return False
    if "shift_labels" in inputs or not _common.on_gpu(inputs.get("labels"),
                                                      inputs.get("attention_mask")):
        return False
    if getattr(args, "use_liger_kernel", False) or getattr(args, "loss_type", "nll") != "nll":
        return False
    for name in ("compute_loss_func", "label_smoother", "_soup_chunked_head_loss"):
        if getattr(trainer, name, None) is not None:
            return False
    if getattr(trainer, "num_virtual_tokens", 0) or getattr(trainer, "aux_loss_enabled", False):
        return False
    lm = _inner_lm(trainer, model)
    return isinstance(lm, Qwen2ForCausalLM) and head_fits(lm)


TRAINER_LOSS = [None]   # the fused loss the trainer hook arms (the last install_trainer's)


def install_trainer(loss_fn):
    """trl.SFTTrainer.compute_loss arms `loss_fn` for its model forward when the configuration
    fits, and leaves the device-side step it produced on the trainer. Raises ImportError when
    trl is absent (as the reference does). A later call switches the loss it arms."""
    from transformers import Trainer
    from trl import SFTTrainer

    TRAINER_LOSS[0] = loss_fn

    def build(original):
        def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
            if not trainer_takes_fused(self, model, inputs):
                setattr(self, STEP_ATTR, None)
                return original(self, model, inputs, return_outputs=return_outputs,
                                num_items_in_batch=num_items_in_batch)
            inputs.pop("_prediction_loss_only", None)
            inputs["use_cache"] = False
            ARMED.loss_fn, ARMED.step = TRAINER_LOSS[0], None
            try:
                loss, outputs = Trainer.compute_loss(self, model, inputs, return_outputs=True,
                                                     num_items_in_batch=num_items_in_batch)
            finally:
                ARMED.loss_fn = None
            step, ARMED.step = ARMED.step, None
            if step is None:
                raise RuntimeError("qlora_b200: the armed fused head loss did not run")
            self.fused_loss_step = step
            setattr(self, STEP_ATTR, step)
            return (loss, outputs) if return_outputs else loss
        return compute_loss

    _common.install(SFTTrainer, "compute_loss", build)
