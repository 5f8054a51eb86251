"""Fused linear cross-entropy + entropy + argmax over the vocabulary without the full logits
(API of solution/cross_entropy.py).

    loss = sum over labelled rows of CE(hidden @ W.T, target) / denominator
plus per-token loss, entropy and argmax (what TRL's metrics and Soup's rewind recorder read).
The head W is frozen. The custom op qlora_b200::linear_ce computes, chunk by chunk of rows, the
per-row statistics and each row's loss gradient w.r.t. its hidden state; the backward only
scales those rows by the incoming gradient (cross_entropy.py:93-138).

bf16 head and hidden states take the tcgen05 kernels: the logits tile lives in TMEM, pass 1
reduces it to row statistics, the gradient pass recomputes it into dZ = softmax - onehot in its
epilogue, and dH = dZ @ W runs on the tcgen05 GEMM. Other dtypes: a matmul chunk of logits, then
the row kernel (qb_ce_rows) streams each row once and rewrites it with the gradient.
"""

import torch

from . import _common, _lib, ops  # noqa: F401 - ops registers the custom operators

IGNORE_INDEX = -100
CHUNK_ROWS = 4096           # rows per chunk of materialised logits (the matmul fallback)
# Rows per chunk on the tcgen05 path, where only dZ (bf16) is materialised: 16384 x 152064 is
# 5 GB, and the dH GEMM's 1792 output tiles of a 16384-row chunk fill 12.1 waves of the 148 SMs
# (a 4096-row chunk's 448 tiles: 3.03 waves, the last one nearly empty). Splitting dH's K (the
# vocabulary) to even out the last wave measured slower: the partial tiles' traffic costs more.
TC_CHUNK_ROWS = 16384
# Off the bf16 path dZ = softmax - onehot is stored in the matmul dtype before the dH matmul. In
# fp16 it is multiplied by GRAD_GAIN (a power of two, exact) so probabilities below fp16's
# smallest subnormal survive, with |dZ| <= GRAD_GAIN far below fp16's largest value, and
# divided back in fp32.
GRAD_GAIN = 1024.0


# False (the default): the logits exist only in TMEM - pass 1 reduces each tile to row
# statistics, and the gradient pass recomputes the tile and turns it into dZ in its epilogue
# (6 N H V flops executed for the algorithmic 4 N H V). True: pass 1 also stores the chunk's fp32
# logits (rows x vocab x 4 bytes, 2.5 GB at 4096 x 152064) and dZ comes from them in one
# streaming pass instead of the second logits GEMM. Same z, same arithmetic, same dZ.
STORE_LOGITS = False


def linear_ce_tc(h2, w, tgt, token_loss, entropy, pred, grad_h, scale_dev, chunk_rows,
                 store_logits=None):
    """The tcgen05 path for bf16 hidden states and head: per chunk of rows, pass 1 (logits in
    TMEM -> per-tile row statistics, and the fp32 logits when `store_logits`), the reduction,
    and with grad_h the dZ pass (dZ = (softmax - onehot) * scale_dev, from the stored logits or a
    second logits GEMM with dZ in its epilogue) followed by dH = dZ @ W into grad_h (fp32)."""
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


def tc_path_ok(h2, w):
    return (h2.is_cuda and w.is_cuda and h2.dtype == torch.bfloat16
            and w.dtype == torch.bfloat16 and h2.shape[1] % 8 == 0 and w.stride(-1) == 1
            and h2.stride(-1) == 1 and w.stride(0) % 8 == 0 and h2.stride(0) % 8 == 0)


def ce_rows_inplace(logits, target, token_loss, entropy, pred, grad_scale, write_grad):
    """Runs the row kernel on a [rows, vocab] logits chunk (rewritten in place with
    (softmax - onehot) * grad_scale when write_grad)."""
    rows, vocab = logits.shape
    _lib.call("qb_ce_rows", logits.data_ptr(), _lib.tag(logits.dtype), logits.stride(0),
              target.data_ptr(), rows, vocab, token_loss.data_ptr(), entropy.data_ptr(),
              _lib.ptr(pred), None, float(grad_scale), int(write_grad),
              _lib.stream(logits.device),
              work=(rows * vocab * logits.element_size() * (3 if write_grad else 1), 0))


def linear_ce_rows(hidden, weight, target, chunk_rows, with_grad):
    """The body of the custom op qlora_b200::linear_ce. hidden [n, H] and weight [V, H] in the
    matmul dtype, target [n] int64 (IGNORE_INDEX rows score nothing). Returns per row: the CE
    loss, the entropy of the softmax, the argmax (first index on ties), and with_grad the
    gradient of that row's loss w.r.t. its hidden state, (softmax - onehot) @ W in fp32 (zero
    for unlabelled rows; else an empty [0, H]). Only `chunk_rows` rows of logits exist at a time,
    on the tcgen05 path none at all (they stay in TMEM; it runs chunks of at least TC_CHUNK_ROWS
    rows, its bf16 dZ the one [rows, vocab] buffer)."""
    _lib.require_cuda(hidden, weight, target, what="fused linear CE")
    n, hdim = hidden.shape
    dev = hidden.device
    tgt = target.to(torch.int64).contiguous()
    token_loss = torch.empty(n, dtype=torch.float32, device=dev)
    entropy = torch.empty(n, dtype=torch.float32, device=dev)
    pred = torch.empty(n, dtype=torch.int64, device=dev)
    dh = torch.empty((n if with_grad else 0, hdim), dtype=torch.float32, device=dev)
    if n == 0:
        return token_loss, entropy, pred, dh
    h2 = hidden if hidden.stride(-1) == 1 else hidden.contiguous()
    if tc_path_ok(h2, weight):
        one = torch.ones(1, dtype=torch.float32, device=dev)   # dZ unscaled: bf16 keeps range
        linear_ce_tc(h2, weight, tgt, token_loss, entropy, pred, dh if with_grad else None, one,
                     max(chunk_rows, TC_CHUNK_ROWS))
        return token_loss, entropy, pred, dh
    # other dtypes: a matmul chunk of logits, then the row kernel streams each row once for the
    # statistics and rewrites it with (softmax - onehot) * gain, then dH_chunk = dZ W / gain
    gain = GRAD_GAIN if weight.dtype == torch.float16 else 1.0
    with torch.autocast(device_type=dev.type, enabled=False):
        for a in range(0, n, chunk_rows):
            b = min(a + chunk_rows, n)
            logits = h2[a:b] @ weight.t()
            ce_rows_inplace(logits, tgt[a:b], token_loss[a:b], entropy[a:b], pred[a:b], gain,
                            with_grad)
            if with_grad:
                dh[a:b] = (logits @ weight).float() * (1.0 / gain)
            del logits
    return token_loss, entropy, pred, dh


class FusedLinearCrossEntropy:
    """loss, per-token loss, entropy and argmax of CE(hidden @ W.T, target) with W frozen
    (cross_entropy.py:93-138): the custom op qlora_b200::linear_ce over the rows, whose
    registered backward scales each row's precomputed gradient by the incoming gradient of its
    loss; loss = sum of the per-token losses / denominator (a tensor or a number: no host
    read)."""

    @staticmethod
    def apply(hidden, weight, target, denominator, matmul_dtype, chunk_rows):
        _lib.require_cuda(hidden, weight, what="fused linear CE")
        shape = hidden.shape
        h2 = hidden.reshape(-1, shape[-1])
        h2 = h2 if h2.dtype == matmul_dtype else h2.to(matmul_dtype)
        w = weight if weight.dtype == matmul_dtype else weight.to(matmul_dtype)
        tgt = target.reshape(-1).to(device=hidden.device, dtype=torch.int64)
        with_grad = torch.is_grad_enabled() and hidden.requires_grad
        token_loss, entropy, pred, _ = torch.ops.qlora_b200.linear_ce(h2, w, tgt,
                                                                       int(chunk_rows),
                                                                       with_grad)
        loss = token_loss.sum() / denominator
        lead = shape[:-1]
        return loss, token_loss.view(lead), entropy.view(lead), pred.view(lead)


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


def _causal_lm_loss(hidden, head_weight, labels, attention_mask, kwargs):
    """The loss the causal-LM hook computes for cross_entropy.patch(): ForCausalLMLoss with its
    num_items_in_batch / shift_labels, and the ChunkedStep."""
    return fused_causal_lm_loss(hidden, head_weight, labels,
                                num_items_in_batch=kwargs.get("num_items_in_batch"),
                                shift_labels=kwargs.get("shift_labels"))


def patch():
    """Qwen2ForCausalLM.forward and trl.SFTTrainer.compute_loss on the fused loss
    (cross_entropy.py:190-321): the trainer arms it for one model forward, which returns the loss
    with logits=None; the ChunkedStep (per-token loss, entropy, argmax, counts, on the device) is
    left on the trainer. The trainer half is skipped when trl is not installed."""
    from . import hooks
    hooks.install_causal_lm()
    try:
        hooks.install_trainer(_causal_lm_loss)
    except ImportError:
        pass
