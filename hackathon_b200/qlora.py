"""A Qwen2.5-shaped QLoRA training step built from this package's ops.

The model is the Qwen2 decoder (RMSNorm -> q/k/v -> RoPE -> causal GQA attention -> o ->
residual -> RMSNorm -> gate/up -> SwiGLU -> down -> residual) with every linear a frozen NF4
(blocksize 64, double-quantised scales) base plus a trainable LoRA adapter, a final RMSNorm and a
frozen bf16 lm_head feeding the fused linear cross-entropy. Weights are random (N(0, 0.02)
before quantisation; LoRA A Kaiming-uniform, B N(0, 0.01)); there is no checkpoint to load.
Attention is torch's scaled_dot_product_attention (the reference never patches attention).

Per-rank data parallelism lives in dp.py; this module is single-device.
"""

import math
from dataclasses import dataclass, replace

import torch
import torch.nn.functional as F

from .cross_entropy import fused_causal_lm_loss
from .lora import DropoutCast, ScaledAdd
from .nf4 import NF4Linear, quantize_nf4
from .rmsnorm import rmsnorm
from .rope import CudaRoPE
from .swiglu import swiglu


@dataclass(frozen=True)
class QwenShape:
    name: str
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    tie_embeddings: bool
    theta: float = 1e6
    eps: float = 1e-6
    lora_r: int = 16
    lora_alpha: int = 32
    lora_dropout: float = 0.05


PRESETS = {
    # Qwen2.5-0.5B shapes, r=16 (the smallest benchmark configuration)
    "0.5b": QwenShape("qwen2.5-0.5b", 896, 4864, 24, 14, 2, 64, 151936, True),
    # Qwen2.5-1.5B shapes, r=16
    "1.5b": QwenShape("qwen2.5-1.5b", 1536, 8960, 28, 12, 2, 128, 151936, True),
    # Qwen2.5-7B shapes, r=64 alpha=128 (the headline benchmark configuration)
    "7b": QwenShape("qwen2.5-7b", 3584, 18944, 28, 28, 4, 128, 152064, False,
                    lora_r=64, lora_alpha=128),
}


def preset(name, **overrides):
    return replace(PRESETS[name], **overrides)


# Dropout masks of the current step, as bits, keyed by (projection, seed): drawn in the first
# forward, reused by the checkpoint recompute and the backward, dropped after the backward.
# QwenQLoRA.forward clears whatever a forward without backward left behind.
MASKS = {}

# Dropout masks drawn ahead on a side stream (one per device): the mask depends only on (seed,
# element index), so the next layer's masks are drawn while this layer's tensor-core GEMMs run
# (the Philox rounds load the integer pipes, which those GEMMs leave idle).
_SIDE_STREAMS = {}
MASK_CTAS_PER_SM = 2    # fixed grid beside the GEMMs' one CTA per SM (qb_dropout_bits)


def _side_stream(device):
    d = torch.device(device)
    if d not in _SIDE_STREAMS:
        _SIDE_STREAMS[d] = torch.cuda.Stream(device=d)
    return _SIDE_STREAMS[d]


def prefetch_masks(layer, seed, rows, device):
    """Draws the dropout masks of `layer`'s seven projections (seeds seed + 0 .. 6, the seeds
    DecoderLayer.forward gives them) into MASKS on the side stream and returns the event the
    consumer's stream must wait on before the layer runs (None: nothing drawn). The bits are
    allocated on the current stream and the side stream waits for it first, so memory reuse
    stays ordered on the current stream."""
    from .lora import dropout_bits
    main = torch.cuda.current_stream(device)
    todo = []
    for k, name in enumerate(_PROJ):
        mod = getattr(layer, name)
        key = (id(mod), seed + k)
        if (mod.training and mod.p > 0 and mod.fused and mod.in_features % 8 == 0
                and key not in MASKS):
            todo.append((key, mod, seed + k,
                         torch.empty((rows, (mod.in_features + 31) // 32), dtype=torch.int32,
                                     device=device)))
    if not todo:
        return None
    side = _side_stream(device)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        for key, mod, sd, bits in todo:
            dropout_bits(rows, mod.in_features, mod.p, sd, device, MASK_CTAS_PER_SM, out=bits)
            MASKS[key] = bits
        ev = torch.cuda.Event()
        ev.record(side)
    return ev


def recorded_mask(mod, seed, rows):
    """(bits, scale) of mod's dropout mask for `seed` when the step has it recorded for `rows`
    rows and mod's fused path will use it, else None."""
    if not (mod.training and mod.p > 0 and mod.fused and mod.in_features % 8 == 0):
        return None
    bits = MASKS.get((id(mod), seed))
    if bits is None or bits.shape[0] != rows:
        return None
    return bits, 1.0 / (1.0 - mod.p)


def shared_dropouts(x2, pairs):
    """The dropped-out inputs of projections that share x2, [(mod, seed)] -> [xd or None]: one
    pass over x2 (dropout_apply_multi) when every mask is recorded already, else all None (each
    projection then draws or applies its own)."""
    from .lora import dropout_apply_multi
    from .nf4 import fused_ok
    masks = [recorded_mask(mod, sd, x2.shape[0]) if fused_ok(x2, mod.quant_state) else None
             for mod, sd in pairs]
    if (len(pairs) < 2 or any(m is None for m in masks) or x2.shape[1] % 8
            or x2.stride(-1) != 1):
        return [None] * len(pairs)
    return dropout_apply_multi(x2, masks)


def gemm_mask_jobs(pairs, rows, device):
    """Allocates the bits of the (projection, seed) masks that are not drawn yet, enters them in
    MASKS and returns them as qb_mask_job tuples for the gate/up GEMM that draws them in its side
    warps (the GEMM runs on the current stream before any projection reads the bits)."""
    jobs = []
    for mod, sd in pairs:
        key = (id(mod), sd)
        if (mod.training and mod.p > 0 and mod.fused and mod.in_features % 8 == 0
                and key not in MASKS):
            bits = torch.empty((rows, (mod.in_features + 31) // 32), dtype=torch.int32,
                               device=device)
            MASKS[key] = bits
            jobs.append((bits, rows, mod.in_features, sd, mod.p))
    return jobs


def _mask_bits(x2, mod, p, seed):
    """The step's mask bits for (mod, seed) over x2's shape: drawn ahead (prefetch_masks) or
    drawn now (mask only, no data pass)."""
    from .lora import dropout_bits
    key = (id(mod), seed)
    bits = MASKS.get(key)
    if bits is None or bits.shape[0] != x2.shape[0]:
        bits = dropout_bits(x2.shape[0], x2.shape[1], p, seed, x2.device)
        MASKS[key] = bits
    return bits


# U = dropout(x) A^T in one kernel from x and the mask bits (qb_lora_xa) when True; False (the
# default) composes the dropout pass (xd to HBM: qb_dropout_mask, or qb_dropout_apply from
# recorded bits) with the tcgen05 GEMM - the same numbers up to accumulation order. qb_lora_xa
# entered the step together with the 2-SM GEMM and the side-stream masks, when runs of the 7B
# step began to stall; it stays opt-in until that is explained.
FUSED_ADAPTER_INPUT = False


# The rank-r products U = xd A^T of an activation checkpoint's first pass, kept for its
# recompute, keyed by (projection, seed) (the gate / up pair by ("pair", gate, seed)): the
# recompute forms the same xd from the same recorded mask and multiplies it by the same A (the
# adapters change only at the optimizer step), so it reuses U — [tokens, r], 2 MB a projection
# at 16384 tokens and r = 64 — and rebuilds only xd. Cleared with MASKS at every forward.
UPRODS = {}
KEEP_UPRODS = True


def _keep_uprod(keep_xd, graph):
    """True when this call is an activation checkpoint's first pass that a recompute follows:
    nothing saved is kept (keep_xd False) and the adapters take part in an autograd graph
    (`graph`: the autograd Function's needs_input_grad for them; grad mode itself is off inside
    a Function's forward)."""
    return KEEP_UPRODS and not keep_xd and graph


def _adapter_input(x2, mod, a16, p, seed, keep_xd, u_out=None, stash=False, xd=None):
    """(xd, U = xd a16^T, bits, scale) of one projection with xd = dropout(x2) * scale: U comes
    from x2 and the mask bits in one kernel (qb_lora_xa); xd is stored only when the backward
    will read it (keep_xd), else an empty placeholder stands in its saved slot. stash (the
    caller's graph flag of _keep_uprod): keep U of a checkpoint's first pass for its recompute
    (UPRODS); a recompute (keep_xd) takes it from there. xd: dropout(x2) already formed from the
    step's recorded mask (one pass over an input several projections share)."""
    key = (id(mod), seed)
    kept = UPRODS.pop(key, None) if keep_xd and u_out is None else None
    if kept is not None and kept.shape == (x2.shape[0], a16.shape[0]):
        xd, bits, scale = _dropped(x2, mod, p, seed, xd)
        return xd, kept, bits, scale
    xd, u, bits, scale = _adapter_product(x2, mod, a16, p, seed, keep_xd, u_out, xd)
    if u_out is None and _keep_uprod(keep_xd, stash):
        UPRODS[key] = u
    return xd, u, bits, scale


def _adapter_product(x2, mod, a16, p, seed, keep_xd, u_out, xd=None):
    """_adapter_input's computation: xd and U = xd a16^T."""
    from .gemm import gemm
    from .lora import lora_xa, lora_xa_ok
    if (xd is not None or not FUSED_ADAPTER_INPUT or not lora_xa_ok(x2, a16)
            or (p > 0 and x2.shape[1] % 8)):
        xd, bits, scale = _dropped(x2, mod, p, seed, xd)
        if u_out is not None and u_out.stride(-1) == 1 and u_out.stride(0) % 8 == 0:
            u = gemm(xd, a16, out=u_out)
        else:
            u = gemm(xd, a16)
            if u_out is not None:
                u = u_out.copy_(u)
        return xd, u, bits, scale
    if p <= 0:
        return x2, lora_xa(x2, a16, out=u_out), None, 1.0
    scale = 1.0 / (1.0 - p)
    bits = _mask_bits(x2, mod, p, seed)
    xd = torch.empty_like(x2) if keep_xd else x2.new_empty(0)
    u = lora_xa(x2, a16, bits, scale, out=u_out, xd_out=xd if keep_xd else None)
    return xd, u, bits, scale


def _dropped(x2, mod, p, seed, xd=None):
    """(dropout(x2) * scale, mask bits or None, scale) with the step's mask for (mod, seed): drawn
    once (Philox, the reference's stream) and replayed from the bits afterwards. xd: that
    product already formed from the recorded bits (dropout_apply_multi)."""
    from .lora import dropout_apply, dropout_mask
    if p <= 0:
        return x2, None, 1.0
    scale = 1.0 / (1.0 - p)
    key = (id(mod), seed)
    bits = MASKS.get(key)
    if xd is not None:
        if bits is None or bits.shape[0] != x2.shape[0] or xd.shape != x2.shape:
            raise RuntimeError("a dropped-out input was passed without its recorded mask")
        return xd, bits, scale
    if bits is None or bits.shape[0] != x2.shape[0]:
        xd, bits = dropout_mask(x2, p, seed, scale)
        MASKS[key] = bits
    else:
        xd = dropout_apply(x2, bits, scale)
    return xd, bits, scale


class GateUpSwiGLU(torch.autograd.Function):
    """The MLP's gate and up projections and the SwiGLU between them, long-token path:

        forward   xd_g, xd_u = dropout(x) (each projection's own mask); U_* = xd_* A_*^T
                  (qb_lora_xa, into the two halves of one [T, 2r] buffer)
                  h = silu(x W_g^T + U_g (s B_g)^T) * (x W_u^T + U_u (s B_u)^T)
                                        (one tcgen05 GEMM, SwiGLU in its epilogue; g and u are
                                         stored only when a backward will read them)
        backward  dg, du = SwiGLU'(dh; g, u)
                  dx = dg W_g + du W_u  (+= s mask_* .* (V_* A_*))      V_* = d* (s B_*)
                  dA_* = V_*^T xd_*, dB_* = s d*^T U_*   (tcgen05 GEMMs, split over the tokens)
    The recompute keeps the two rebuilt bf16 weights for the backward of the same layer."""

    @staticmethod
    def forward(ctx, x, a_g, b_g, a_u, b_u, gate, up, p, seed_g, seed_u, save_gu,
                mask_jobs=None):
        from .gemm import gemm_gateup_swiglu
        from .nf4 import _weight_workspace, dequantize_nf4
        x2 = x.reshape(-1, x.shape[-1])
        T, H = x2.shape
        I, r = gate.out_features, a_g.shape[0]
        a16_g, _ = gate.adapter16(x.dtype)
        a16_u, _ = up.adapter16(x.dtype)
        pair = ("pair", id(gate), seed_g)
        kept = UPRODS.pop(pair, None) if save_gu else None
        # both masks recorded: one pass over x forms the two dropouts
        dg, du = shared_dropouts(x2, [(gate, seed_g), (up, seed_u)]) if p > 0 else (None, None)
        if kept is not None and kept.shape == (T, 2 * r):
            # the recompute: [U_g | U_u] from the first pass, only xd_g / xd_u rebuilt
            lora_u = kept
            xd_g, bits_g, scale = _dropped(x2, gate, p, seed_g, dg)
            xd_u, bits_u, _ = _dropped(x2, up, p, seed_u, du)
            u_g, u_u = lora_u[:, :r], lora_u[:, r:]
        else:
            lora_u = torch.empty((T, 2 * r), dtype=x.dtype, device=x.device)   # [U_g | U_u]
            xd_g, u_g, bits_g, scale = _adapter_input(x2, gate, a16_g, p, seed_g, save_gu,
                                                      u_out=lora_u[:, :r], xd=dg)
            xd_u, u_u, bits_u, _ = _adapter_input(x2, up, a16_u, p, seed_u, save_gu,
                                                  u_out=lora_u[:, r:], xd=du)
            if _keep_uprod(save_gu, any(ctx.needs_input_grad[1:5])):
                UPRODS[pair] = lora_u
        if gate._shadow_b1 is not None and x.dtype == torch.bfloat16:
            b1_g, b1_u = gate._shadow_b1
        else:
            b1_g = torch.zeros((I, 2 * r), dtype=x.dtype, device=x.device)
            b1_u = torch.zeros_like(b1_g)
            b1_g[:, :r] = b_g * gate.scaling
            b1_u[:, r:] = b_u * up.scaling
        # Under activation checkpointing both passes must save the same tensors (the recompute's
        # are unpacked in the first pass's slots): what the first pass would keep for the
        # backward is an empty placeholder there, never None.
        keep_w = save_gu and ctx.needs_input_grad[0]
        ws = []
        for slot, mod in enumerate((gate, up)):
            w = torch.empty((I, H), dtype=torch.bfloat16, device=x.device) if keep_w \
                else _weight_workspace(x.device, I, H, slot)
            ws.append(dequantize_nf4(mod.packed, mod.quant_state, torch.bfloat16, out=w))
        empty = torch.empty(0, dtype=torch.bfloat16, device=x.device)
        kept = (ws[0], ws[1]) if keep_w else \
            ((empty, empty) if ctx.needs_input_grad[0] else (None, None))
        if save_gu:
            h, g, u = gemm_gateup_swiglu(x2, ws[0], ws[1], lora_u, b1_g, b1_u, save_gu=True,
                                         mask_jobs=mask_jobs)
        else:
            # the activation checkpoint's first pass: what it saves is discarded and the
            # recompute's tensors are unpacked in the same slots, so empty placeholders do
            h = gemm_gateup_swiglu(x2, ws[0], ws[1], lora_u, b1_g, b1_u, mask_jobs=mask_jobs)
            g = u = empty
        ctx.save_for_backward(xd_g, xd_u, u_g, u_u, a_g, b_g, a_u, b_u, bits_g, bits_u,
                              kept[0], kept[1], g, u)
        ctx.gate, ctx.up, ctx.p, ctx.scale = gate, up, p, scale
        ctx.seeds, ctx.shape = (seed_g, seed_u), x.shape
        return h.view(*x.shape[:-1], I)

    @staticmethod
    def backward(ctx, dh):
        from . import _lib
        from .gemm import gemm2, gemm_mask_acc, lora_products
        from .nf4 import _weight_workspace, dequantize_nf4
        (xd_g, xd_u, u_g, u_u, a_g, b_g, a_u, b_u, bits_g, bits_u, w_g, w_u, g, u) = \
            ctx.saved_tensors
        if g.numel() == 0:
            raise RuntimeError("GateUpSwiGLU: backward through a forward that kept no g/u")
        gate, up, p = ctx.gate, ctx.up, ctx.p
        dh2 = dh.reshape(-1, dh.shape[-1]).to(g.dtype).contiguous()
        dg, du = torch.empty_like(g), torch.empty_like(u)
        _lib.call("qb_swiglu_bwd", dh2.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(),
                  du.data_ptr(), _lib.tag(g.dtype), g.numel(), _lib.stream(g.device),
                  work=(5 * g.numel() * g.element_size(), 0))
        a16_g, sb16_g = gate.adapter16(g.dtype)
        a16_u, sb16_u = up.adapter16(g.dtype)
        need = ctx.needs_input_grad
        v_g, da_g, db_g = lora_products(dg, u_g, xd_g, sb16_g, a_g.shape, gate.scaling, need[1],
                                        need[2])
        v_u, da_u, db_u = lora_products(du, u_u, xd_u, sb16_u, a_u.shape, up.scaling, need[3],
                                        need[4])
        for mod, seed in zip((gate, up), ctx.seeds):
            MASKS.pop((id(mod), seed), None)
        dx = None
        if ctx.needs_input_grad[0]:
            I, H = dg.shape[1], xd_g.shape[1]
            if w_g is None or w_g.numel() == 0:
                w_g = dequantize_nf4(gate.packed, gate.quant_state, torch.bfloat16,
                                     out=_weight_workspace(dg.device, I, H, 0))
                w_u = dequantize_nf4(up.packed, up.quant_state, torch.bfloat16,
                                     out=_weight_workspace(dg.device, I, H, 1))
            dx = gemm2(dg, w_g.t(), du, w_u.t())                       # dg W_g + du W_u
            if p > 0:
                gemm_mask_acc(v_g, a16_g.t(), bits_g, ctx.scale, dx)
                gemm_mask_acc(v_u, a16_u.t(), bits_u, ctx.scale, dx)
            else:   # no mask: both adapter terms as one more tcgen05 GEMM over dx in place
                gemm2(v_g, a16_g.t(), v_u, a16_u.t(), out=dx, residual=dx)
            dx = dx.view(ctx.shape)
        return dx, da_g, db_g, da_u, db_u, None, None, None, None, None, None, None


class LoRANF4Proj(torch.autograd.Function):
    """The whole QLoRA projection (and the residual add it feeds) on this package's kernels:

        forward   xd = dropout(x)                      (mask drawn once per step, kept as bits)
                  U  = xd A^T            (qb_lora_xa: from x and the bits in one tcgen05 kernel;
                                          xd itself is stored only when the backward reads it)
                  y  = h + x deq(W)^T + b + U (s B)^T                   (one tcgen05 GEMM)
        backward  V  = g (s B)                                (skinny tcgen05 GEMM, 64-wide tiles)
                  dx = g deq(W)  [+= s mask .* (V A)]                   (tcgen05 GEMM, then the
                                                                         masked-accumulate GEMM;
                                                                         V A as extra K if p = 0)
                  dA = V^T xd,  dB = s g^T U,  dh = g   (fp32 adapter grads: tcgen05 GEMMs with the
                                                         tokens split across the SMs)
    Under activation checkpointing the recompute keeps xd and, on the long-token path, the bf16
    weight it rebuilt, so the backward of the same layer neither replays the mask on x nor
    rebuilds W (both live only from the layer's recompute to its backward). output_dead: the
    caller discards y (the recompute of a layer's last projection) - everything the backward
    reads is built, the output GEMM is not run. keep_saved=False: what this forward saves is
    discarded (an activation checkpoint's first pass), so xd is not stored (a placeholder keeps
    its slot)."""

    @staticmethod
    def forward(ctx, x, lora_a, lora_b, mod, p, seed, residual, rope, output_dead=False,
                keep_saved=True, dropped=None):
        from .nf4 import dequantize_nf4, nf4_linear_fwd, uses_dequant_path
        x2 = x.reshape(-1, x.shape[-1])
        a16, sb16 = mod.adapter16(x.dtype)
        graph = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        xd, u, bits, scale = _adapter_input(
            x2, mod, a16, p, seed, keep_saved, stash=graph,
            xd=None if dropped is None else dropped.reshape(x2.shape))
        w_keep = None
        if ctx.needs_input_grad[0] and uses_dequant_path(x2.shape[0]):
            w_keep = dequantize_nf4(mod.packed, mod.quant_state, torch.bfloat16,
                                    out=torch.empty((mod.out_features, mod.in_features),
                                                    dtype=torch.bfloat16, device=x.device))
        ctx.save_for_backward(xd, u, lora_a, lora_b, bits, w_keep)
        if output_dead:
            # a checkpoint recompute's last projection: torch keeps only the recompute's saved
            # tensors (and stops at the last of them), never its output
            y = torch.empty((x2.shape[0], mod.out_features), dtype=x.dtype, device=x.device)
        else:
            y = nf4_linear_fwd(x2, mod.packed, mod.quant_state, mod.bias, u, sb16,
                               residual=residual, weight=w_keep, rope=rope)
        ctx.mod, ctx.p, ctx.seed, ctx.scale, ctx.shape = mod, p, seed, scale, x.shape
        ctx.has_residual = residual is not None
        ctx.rope = rope     # the position tables (constants, not activations)
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, g):
        from .gemm import gemm_mask_acc, lora_products
        from .nf4 import nf4_linear_dgrad
        xd, u, lora_a, lora_b, bits, w_keep = ctx.saved_tensors
        mod, p = ctx.mod, ctx.p
        g2 = g.reshape(-1, g.shape[-1])
        if g2.dtype != xd.dtype:
            g2 = g2.to(xd.dtype)
        if ctx.rope is not None:      # through the RoPE first: its transpose
            from .rope import rope_rows
            g2 = rope_rows(g2, ctx.rope[0], ctx.rope[1], backward=True)
        a16, sb16 = mod.adapter16(xd.dtype)
        v, da, db = lora_products(g2, u, xd, sb16, lora_a.shape, mod.scaling,
                                  ctx.needs_input_grad[1], ctx.needs_input_grad[2])
        if p > 0:
            MASKS.pop((id(mod), ctx.seed), None)
        dx = None
        if not ctx.needs_input_grad[0]:
            pass                      # e.g. the first layer's q/k/v: x comes from the embedding
        elif p > 0:
            dx = nf4_linear_dgrad(g2, mod.packed, mod.quant_state, weight=w_keep)
            gemm_mask_acc(v, a16.t(), bits, ctx.scale, dx)         # dx += s mask .* (V A)
            dx = dx.view(ctx.shape)
        else:
            dx = nf4_linear_dgrad(g2, mod.packed, mod.quant_state, v, a16, weight=w_keep)
            dx = dx.view(ctx.shape)
        dres = g if ctx.has_residual and ctx.needs_input_grad[6] else None
        return dx, da, db, None, None, None, dres, None, None, None, None


class LoRANF4Linear(torch.nn.Module):
    """y = x @ deq(W).T + b + (alpha/r) * dropout(x) @ A.T @ B.T with W frozen in NF4."""

    def __init__(self, in_features, out_features, bias, shape, device, gen):
        super().__init__()
        w = torch.empty(out_features, in_features, device=device, dtype=torch.bfloat16)
        w.normal_(0.0, 0.02, generator=gen)
        self.packed, self.quant_state = quantize_nf4(w)
        del w
        self.bias = None
        if bias:
            b = torch.empty(out_features, device=device, dtype=torch.bfloat16)
            self.bias = b.normal_(0.0, 0.02, generator=gen)
        r = shape.lora_r
        a = torch.empty(r, in_features, device=device, dtype=torch.float32)
        bound = 1.0 / math.sqrt(in_features)    # kaiming_uniform_(a=sqrt(5)), as nn.Linear/peft
        a.uniform_(-bound, bound, generator=gen)
        b = torch.empty(out_features, r, device=device, dtype=torch.float32)
        b.normal_(0.0, 0.01, generator=gen)
        self.lora_A = torch.nn.Parameter(a)
        self.lora_B = torch.nn.Parameter(b)
        self.scaling = shape.lora_alpha / r
        self.p = shape.lora_dropout
        self.in_features, self.out_features = in_features, out_features
        self.fused = True
        self._shadow16 = None     # (A, s B) in bf16 from an attached lora.AdapterShadow
        self._shadow_b1 = None    # a gate/up pair's ([s B_g | 0], [0 | s B_u]) from the shadow

    def adapter16(self, dtype):
        """(A, s B) in `dtype` for the adapter GEMMs: the attached AdapterShadow's copies (bf16,
        rebuilt once per step) when there is one, else converted here."""
        if self._shadow16 is not None and dtype == torch.bfloat16:
            return self._shadow16
        return (self.lora_A.detach().to(dtype),
                (self.lora_B.detach() * self.scaling).to(dtype))

    def forward(self, x, seed, residual=None, rope=None, output_dead=False, keep_saved=True,
                dropped=None):
        """residual + this projection of x (the residual add of the decoder layer rides in the
        projection's epilogue on the fused path); rope = (cos, sin) [S, 128] applies the
        rotate-half RoPE to the output heads (fused path only); output_dead: the caller only
        needs what the backward saves (a checkpoint recompute), the result is left unwritten;
        keep_saved=False: the caller discards what the forward saves (a checkpoint's first
        pass); dropped: dropout(x) already formed from this step's recorded mask for `seed` (the
        fused path uses it in place of its own dropout pass; the reference composition redraws
        the same mask)."""
        from .nf4 import fused_ok
        p = self.p if self.training else 0.0
        if self.fused and fused_ok(x, self.quant_state):
            if residual is not None and (residual.dtype != torch.bfloat16
                                         or residual.shape[:-1] != x.shape[:-1]):
                raise ValueError("residual: bf16, one row per input row")
            return LoRANF4Proj.apply(x, self.lora_A, self.lora_B, self, p, seed, residual, rope,
                                     output_dead, keep_saved, dropped if p > 0 else None)
        if rope is not None:
            raise ValueError("rope: only on the fused path")
        # the reference's composition: NF4Linear + DropoutCast + adapter GEMMs + ScaledAdd
        base = NF4Linear.apply(x, self.packed, self.quant_state, self.bias)
        xd = DropoutCast.apply(x, p, seed, x.dtype) if p > 0 else x
        lo = F.linear(F.linear(xd, self.lora_A.to(x.dtype)), self.lora_B.to(x.dtype))
        out = ScaledAdd.apply(base, lo, self.scaling)
        return out if residual is None else residual + out


_PROJ = ("q", "k", "v", "o", "gate", "up", "down")


class DecoderLayer(torch.nn.Module):
    def __init__(self, shape, device, gen):
        super().__init__()
        s = shape
        H, I, D = s.hidden, s.intermediate, s.head_dim
        self.shape = s
        self.ln1 = torch.ones(H, device=device, dtype=torch.bfloat16)
        self.ln2 = torch.ones(H, device=device, dtype=torch.bfloat16)
        self.q = LoRANF4Linear(H, s.heads * D, True, s, device, gen)
        self.k = LoRANF4Linear(H, s.kv_heads * D, True, s, device, gen)
        self.v = LoRANF4Linear(H, s.kv_heads * D, True, s, device, gen)
        self.o = LoRANF4Linear(s.heads * D, H, False, s, device, gen)
        self.gate = LoRANF4Linear(H, I, False, s, device, gen)
        self.up = LoRANF4Linear(H, I, False, s, device, gen)
        self.down = LoRANF4Linear(I, H, False, s, device, gen)

    def rope_fused_ok(self, x, cos):
        """q and k take the RoPE in their GEMM epilogue: both on the fused path, heads of 128,
        one position table for the batch, bf16 tables with 16-byte rows."""
        from .nf4 import fused_ok
        return (self.q.fused and self.k.fused and fused_ok(x, self.q.quant_state)
                and fused_ok(x, self.k.quant_state) and self.shape.head_dim == 128
                and cos.shape[0] == 1 and cos.dtype == torch.bfloat16 and cos.is_contiguous())

    def mlp_fused_ok(self, x):
        """The gate/up pair runs as one GEMM with the SwiGLU in its epilogue on the long-token
        path (bf16, NF4 weights the fused kernels take, in_features a multiple of 64)."""
        from .nf4 import fused_ok, uses_dequant_path
        g, u = self.gate, self.up
        return (g.fused and u.fused and fused_ok(x, g.quant_state) and fused_ok(x, u.quant_state)
                and uses_dequant_path(x.numel() // x.shape[-1]) and g.in_features % 64 == 0
                and g.lora_A.shape == u.lora_A.shape and g.p == u.p)

    def forward(self, h, cos, sin, seed, ckpt_calls=None, prefetch=None, masks=None):
        """ckpt_calls: a one-element list the activation checkpoint passes to both of its calls;
        the first call's saved tensors are discarded, so it skips storing what only a backward
        reads; the second call (the recompute) has its output discarded, so the last
        projection, whose output is the layer's output, builds only what its backward reads.
        prefetch: called once, in the first pass only, as the o projection starts (the next
        layer's dropout masks then overlap this layer's o / gate / up / down GEMMs).
        masks: called once, in the first pass only, for the mask jobs the gate/up GEMM draws in
        its side warps (this layer's down mask and the next layer's six)."""
        first_of_checkpoint = recompute = False
        if ckpt_calls is not None:
            first_of_checkpoint = ckpt_calls[0] == 0
            recompute = ckpt_calls[0] == 1
            ckpt_calls[0] += 1
        s = self.shape
        B, S, _ = h.shape
        keep = not first_of_checkpoint    # the first pass's saved tensors are discarded
        x = rmsnorm(h, self.ln1, s.eps)
        # q / k / v share x: with their masks recorded, one pass forms the three dropouts
        dq, dk, dv = shared_dropouts(x.reshape(-1, x.shape[-1]),
                                     [(self.q, seed + 0), (self.k, seed + 1), (self.v, seed + 2)])
        if self.rope_fused_ok(x, cos):
            # RoPE in the q / k projections' epilogue (tables [S, 128] of this sequence)
            cs = (cos[0], sin[0])
            q = self.q(x, seed + 0, rope=cs, keep_saved=keep, dropped=dq).view(
                B, S, s.heads, s.head_dim).transpose(1, 2)
            k = self.k(x, seed + 1, rope=cs, keep_saved=keep, dropped=dk).view(
                B, S, s.kv_heads, s.head_dim).transpose(1, 2)
        else:
            q = self.q(x, seed + 0, keep_saved=keep, dropped=dq).view(
                B, S, s.heads, s.head_dim).transpose(1, 2)
            k = self.k(x, seed + 1, keep_saved=keep, dropped=dk).view(
                B, S, s.kv_heads, s.head_dim).transpose(1, 2)
            q, k = CudaRoPE.apply(q, k, cos, sin)
        v = self.v(x, seed + 2, keep_saved=keep, dropped=dv).view(
            B, S, s.kv_heads, s.head_dim).transpose(1, 2)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        a = a.transpose(1, 2).reshape(B, S, s.heads * s.head_dim)
        if prefetch is not None and not recompute:
            prefetch()
        h = self.o(a, seed + 3, residual=h, keep_saved=keep)
        x = rmsnorm(h, self.ln2, s.eps)
        if self.mlp_fused_ok(x):
            p = self.gate.p if self.training else 0.0
            jobs = masks() if masks is not None and not recompute else None
            m = GateUpSwiGLU.apply(x, self.gate.lora_A, self.gate.lora_B, self.up.lora_A,
                                   self.up.lora_B, self.gate, self.up, p, seed + 4, seed + 5,
                                   torch.is_grad_enabled() and not first_of_checkpoint, jobs)
        else:
            dg, du = shared_dropouts(x.reshape(-1, x.shape[-1]),
                                     [(self.gate, seed + 4), (self.up, seed + 5)])
            m = swiglu(self.gate(x, seed + 4, dropped=dg), self.up(x, seed + 5, dropped=du))
        return self.down(m, seed + 6, residual=h, output_dead=recompute, keep_saved=keep)


class QwenQLoRA(torch.nn.Module):
    """The full model: embedding -> layers -> final norm -> fused linear CE."""

    def __init__(self, shape, device="cuda", seed=0, checkpoint=True):
        super().__init__()
        self.shape = shape
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)
        emb = torch.empty(shape.vocab, shape.hidden, device=dev, dtype=torch.bfloat16)
        self.embed = emb.normal_(0.0, 0.02, generator=gen)
        self.layers = torch.nn.ModuleList(DecoderLayer(shape, dev, gen)
                                          for _ in range(shape.layers))
        self.norm = torch.ones(shape.hidden, device=dev, dtype=torch.bfloat16)
        if shape.tie_embeddings:
            self.lm_head = self.embed
        else:
            head = torch.empty(shape.vocab, shape.hidden, device=dev, dtype=torch.bfloat16)
            self.lm_head = head.normal_(0.0, 0.02, generator=gen)
        self.checkpoint = checkpoint
        # True: draw layer i+1's dropout masks on a side stream beside layer i's GEMMs. Off by
        # default: it entered the step together with the 2-SM GEMM and qb_lora_xa, when runs of
        # the 7B step began to stall, and stays opt-in until that is explained.
        self.mask_prefetch = False
        # True: each layer's gate/up GEMM draws its down projection's dropout mask and the next
        # layer's six in warps beside the GEMM's own (one kernel, one stream); the projections
        # then apply recorded bits instead of running the Philox rounds themselves.
        self.gemm_masks = True
        self._rope = {}
        self.step_seed = 0
        # the bf16 adapter operands of every projection, rebuilt by one launch per forward
        from .lora import AdapterShadow
        self.adapter_shadow = AdapterShadow(
            [m for m in self.modules() if isinstance(m, LoRANF4Linear)],
            [(layer.gate, layer.up) for layer in self.layers])

    def rope_tables(self, seq, device):
        key = (seq, device)
        if key not in self._rope:
            D = self.shape.head_dim
            inv = 1.0 / (self.shape.theta ** (torch.arange(0, D, 2, dtype=torch.float32,
                                                           device=device) / D))
            pos = torch.arange(seq, dtype=torch.float32, device=device)
            emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)[None]
            self._rope[key] = (emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16))
        return self._rope[key]

    def forward(self, input_ids, labels, num_items_in_batch=None):
        B, S = input_ids.shape
        dev = input_ids.device
        if MASKS and dev in _SIDE_STREAMS:   # masks a side stream may still be writing
            torch.cuda.current_stream(dev).wait_stream(_SIDE_STREAMS[dev])
        MASKS.clear()
        UPRODS.clear()
        if self.adapter_shadow is not None:   # the adapters changed since the last forward
            self.adapter_shadow.refresh()
        cos, sin = self.rope_tables(S, dev)
        h = F.embedding(input_ids, self.embed)
        seeds = [self.layer_seed(i) for i in range(len(self.layers))]
        ready = [None] * len(self.layers)       # events of masks drawn ahead

        def prefetcher(j):
            if not (self.mask_prefetch and self.training and torch.is_grad_enabled()
                    and j < len(self.layers)):
                return None

            def run():
                ready[j] = prefetch_masks(self.layers[j], seeds[j], B * S, dev)
            return run

        def mask_jobs(i):
            if not (self.gemm_masks and not self.mask_prefetch and self.training
                    and torch.is_grad_enabled()):
                return None
            pairs = [(self.layers[i].down, seeds[i] + 6)]
            if i + 1 < len(self.layers):
                nxt = self.layers[i + 1]
                pairs += [(getattr(nxt, n), seeds[i + 1] + k) for k, n in enumerate(_PROJ[:6])]
            return lambda: gemm_mask_jobs(pairs, B * S, dev)

        for i, layer in enumerate(self.layers):
            if ready[i] is not None:
                torch.cuda.current_stream(dev).wait_event(ready[i])
            if self.checkpoint and self.training:
                # the recompute replays the dropout masks from their bits, so it is
                # deterministic; the first pass saves placeholders where only the recompute's
                # tensors are ever read (shape check off for those)
                h = torch.utils.checkpoint.checkpoint(layer, h, cos, sin, seeds[i], [0],
                                                      prefetcher(i + 1), mask_jobs(i),
                                                      use_reentrant=False,
                                                      determinism_check="none")
            else:
                h = layer(h, cos, sin, seeds[i], None, prefetcher(i + 1), mask_jobs(i))
        h = rmsnorm(h, self.norm, self.shape.eps)
        return fused_causal_lm_loss(h, self.lm_head, labels, num_items_in_batch=num_items_in_batch)

    def layer_seed(self, i):
        """Per (step, layer) dropout seed; projection k of the layer draws with seed + k."""
        return (self.step_seed * 1_000_003 + i * 7919) & 0x7FFFFFFF

    def adapter_parameters(self):
        return [p for p in self.parameters() if p.requires_grad]


def synthetic_batch(shape, batch, seq, device, seed, ignore_frac=0.05):
    """Token ids uniform in [0, vocab), labels = ids with ~ignore_frac set to -100 (shifted
    inside the loss, as ForCausalLMLoss does)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    ids = torch.randint(0, shape.vocab, (batch, seq), device=device, generator=gen)
    labels = ids.clone()
    labels[torch.rand(batch, seq, device=device, generator=gen) < ignore_frac] = -100
    return ids, labels


def make_optimizer(model, lr=1e-4):
    """AdamW on the adapters only (the NF4 base, norms and head are frozen buffers)."""
    return torch.optim.AdamW(model.adapter_parameters(), lr=lr, betas=(0.9, 0.999),
                             weight_decay=0.0, fused=True)


def train_step(model, opt, input_ids, labels, grad_sync=None, num_items_in_batch=None):
    """One optimizer step; returns the loss tensor (on the device, not synchronised)."""
    model.train()
    loss, _ = model(input_ids, labels, num_items_in_batch=num_items_in_batch)
    loss.backward()
    if grad_sync is not None:
        grad_sync()
    opt.step()
    # with a gradient sync the .grad tensors are views into its flat buffer and stay; without
    # one, dropping them lets the next backward hand its fresh gradients over without an add
    opt.zero_grad(set_to_none=grad_sync is None)
    model.step_seed += 1
    return loss.detach()
