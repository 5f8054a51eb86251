"""LoRA dropout + cast and scaled add around peft's 4-bit LoRA layer (API of solution/lora.py).

peft's bnb.Linear4bit forward under autocast is
    result = base_layer(x); result = result + lora_B(lora_A(dropout(x))) * scaling
Here:
    xd  = DropoutCast(x)      one pass: Philox mask from a seed (no stored mask), 1/(1-p) scale,
                              cast to the compute dtype; backward = same kernel, same seed
    lo  = lora_B(lora_A(xd))  the adapter GEMMs (autograd gives dA, dB, dx)
    out = ScaledAdd(result, lo, scaling)
The mask stream is Philox-4x32-10 keyed by the seed at counter int32(row*cols + col): the one
Triton's tl.rand draws, so masks equal the reference kernel's for the same seed.
"""

import torch

from . import _common, _lib

TORCH_DROPOUT_RNG = False


def _rows(t):
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


def _dropout_scale(src, out_dtype, seed, p, scale):
    _lib.require_cuda(src, what="dropout_scale")
    s2 = _rows(src)
    out = torch.empty(s2.shape, dtype=out_dtype, device=src.device)
    M, N = s2.shape
    _lib.call("qb_dropout_scale", s2.data_ptr(), _lib.tag(s2.dtype), s2.stride(0), out.data_ptr(),
              _lib.tag(out_dtype), out.stride(0), M, N, int(seed) & 0xFFFFFFFFFFFFFFFF,
              float(p), float(scale), _lib.stream(src.device),
              work=(M * N * (s2.element_size() + out.element_size()), 0))
    return out.view(src.shape)


def dropout_mask(x2, p, seed, scale, out_dtype=None):
    """(dropout(x2) in out_dtype, mask bits int32 [rows, ceil(cols/32)]) — the same Philox mask
    as DropoutCast, recorded so a recompute or a backward can reuse it without random numbers."""
    _lib.require_cuda(x2, what="dropout_mask")
    rows, cols = x2.shape
    out = torch.empty((rows, cols), dtype=out_dtype or x2.dtype, device=x2.device)
    bits = torch.empty((rows, (cols + 31) // 32), dtype=torch.int32, device=x2.device)
    _lib.call("qb_dropout_mask", x2.data_ptr(), _lib.tag(x2.dtype), x2.stride(0), out.data_ptr(),
              _lib.tag(out.dtype), out.stride(0), bits.data_ptr(), rows, cols,
              int(seed) & 0xFFFFFFFFFFFFFFFF, float(p), float(scale), _lib.stream(x2.device),
              work=(rows * cols * (x2.element_size() + out.element_size()) + bits.numel() * 4, 0))
    return out, bits


def dropout_bits(rows, cols, p, seed, device, ctas_per_sm=0, out=None):
    """The mask bits dropout_mask records for a [rows, cols] input (int32 [rows, ceil(cols/32)]),
    drawn without the data: the mask depends on (seed, element index) only. ctas_per_sm caps
    the grid (1..8 blocks per SM) so the kernel can share the SMs with a GEMM on another
    stream; 0 fills the GPU."""
    if out is None:
        out = torch.empty((rows, (cols + 31) // 32), dtype=torch.int32, device=device)
    _lib.call("qb_dropout_bits", out.data_ptr(), rows, cols, int(seed) & 0xFFFFFFFFFFFFFFFF,
              float(p), int(ctas_per_sm), _lib.stream(torch.device(device)),
              work=(out.numel() * 4, rows * cols))
    return out


def lora_xa(x2, a16, bits=None, scale=1.0, out=None, xd_out=None):
    """U = dropout(x2) @ a16.T with the dropout taken from recorded mask bits inside the kernel
    (xd = bf16(x * scale) where kept, else 0 — what dropout_apply writes); bits None: U = x2 @
    a16.T. x2 [T, K] bf16, a16 [R, K] bf16 -> U [T, R] bf16 (into `out`, which may be a column
    slice of a wider buffer). xd_out [T, K]: also stores xd (with bits)."""
    _lib.require_cuda(x2, a16, what="lora_xa")
    T, K = x2.shape
    R = a16.shape[0]
    if x2.dtype != torch.bfloat16 or a16.dtype != torch.bfloat16:
        raise TypeError("lora_xa: bf16 input and adapter")
    if out is None:
        out = torch.empty((T, R), dtype=torch.bfloat16, device=x2.device)
    _lib.call("qb_lora_xa", x2.data_ptr(), x2.stride(0), a16.data_ptr(), a16.stride(0),
              _lib.ptr(bits), bits.stride(0) if bits is not None else 0, float(scale),
              out.data_ptr(), out.stride(0), _lib.ptr(xd_out),
              xd_out.stride(0) if xd_out is not None else 0, T, K, R, _lib.stream(x2.device),
              work=(T * K * 2 * (2 if xd_out is not None else 1) + T * R * 2
                    + (bits.numel() * 4 if bits is not None else 0), 0))
    return out


def lora_xa_ok(x2, a16):
    """The shapes and layouts qb_lora_xa takes (else the caller composes dropout + GEMM)."""
    R = a16.shape[0]
    return (x2.dtype == torch.bfloat16 and x2.dim() == 2 and x2.stride(1) == 1
            and x2.stride(0) % 8 == 0 and x2.data_ptr() % 16 == 0 and R % 32 == 0
            and 32 <= R <= 256 and a16.is_contiguous() and a16.shape[1] % 8 == 0)


def dropout_apply(x2, bits, scale, out=None, accumulate=False):
    """out = x2 * mask * scale (or out += ...) from recorded mask bits."""
    rows, cols = x2.shape
    if out is None:
        out = torch.empty_like(x2)
    _lib.call("qb_dropout_apply", x2.data_ptr(), _lib.tag(x2.dtype), x2.stride(0),
              bits.data_ptr(), out.data_ptr(), _lib.tag(out.dtype), out.stride(0), rows, cols,
              float(scale), int(accumulate), _lib.stream(x2.device),
              work=(rows * cols * (x2.element_size() + out.element_size() * (2 if accumulate else 1))
                    + bits.numel() * 4, 0))
    return out


class DropoutCast(torch.autograd.Function):
    """x -> dropout(x) cast to out_dtype, mask from (seed, flat index) (lora.py:84-93)."""

    @staticmethod
    def forward(ctx, x, p, seed, out_dtype):
        scale = 1.0 / (1.0 - p) if p > 0 else 1.0
        ctx.p, ctx.seed, ctx.scale, ctx.x_dtype = p, seed, scale, x.dtype
        return _dropout_scale(x, out_dtype, seed, p, scale)

    @staticmethod
    def backward(ctx, g):
        return _dropout_scale(g, ctx.x_dtype, ctx.seed, ctx.p, ctx.scale), None, None, None


class ScaledAdd(torch.autograd.Function):
    """out = base + lo * scaling in promote(base, lo) (lora.py:96-112)."""

    @staticmethod
    def forward(ctx, base, lo, scaling):
        _lib.require_cuda(base, lo, what="scaled_add")
        b2, l2 = _rows(base), _rows(lo)
        out_dtype = torch.promote_types(base.dtype, lo.dtype)
        out = torch.empty(b2.shape, dtype=out_dtype, device=base.device)
        M, N = b2.shape
        _lib.call("qb_scaled_add", b2.data_ptr(), _lib.tag(b2.dtype), b2.stride(0), l2.data_ptr(),
                  _lib.tag(l2.dtype), l2.stride(0), out.data_ptr(), _lib.tag(out_dtype),
                  out.stride(0), M, N, float(scaling), _lib.stream(base.device),
                  work=(M * N * (b2.element_size() + l2.element_size() + out.element_size()), 0))
        ctx.scaling, ctx.base_dtype, ctx.lo_dtype = scaling, base.dtype, lo.dtype
        return out.view(base.shape)

    @staticmethod
    def backward(ctx, g):
        d_base = g if g.dtype == ctx.base_dtype else g.to(ctx.base_dtype)
        d_lo = _dropout_scale(g, ctx.lo_dtype, 0, 0.0, ctx.scaling)  # g * scaling, cast
        return d_base, d_lo, None


class _Seeds:
    """Philox seeds from a private generator seeded by the run's torch seed, so no other random
    stream (data order, init) is disturbed and a run stays reproducible (lora.py:115-124)."""
    gen = None

    @classmethod
    def next(cls):
        if cls.gen is None:
            cls.gen = torch.Generator().manual_seed(torch.initial_seed() & 0xFFFF_FFFF)
        return int(torch.randint(0, 2**31 - 1, (1,), generator=cls.gen))


def _single_adapter(layer):
    """The one active plain-LoRA adapter of a peft layer, or None (lora.py:127-142)."""
    if layer.disable_adapters or layer.merged:
        return None
    active = [a for a in layer.active_adapters if a in layer.lora_A.keys()]
    if len(active) != 1:
        return None
    a = active[0]
    if a in getattr(layer, "lora_variant", {}):
        return None
    lora_a, lora_b = layer.lora_A[a], layer.lora_B[a]
    if not (type(lora_a) is torch.nn.Linear and type(lora_b) is torch.nn.Linear
            and lora_a.bias is None and lora_b.bias is None):
        return None
    if not isinstance(layer.lora_dropout[a], (torch.nn.Dropout, torch.nn.Identity)):
        return None
    return a


def patch():
    """Routes peft's lora.bnb.Linear4bit.forward through DropoutCast / ScaledAdd
    (lora.py:145-176). A no-op when peft is not installed."""
    try:
        from peft.tuners.lora import bnb as lora_bnb
    except ImportError:
        return
    cls = getattr(lora_bnb, "Linear4bit", None)
    if cls is None:
        return
    original = cls.forward
    if getattr(original, "_solution_patch", False):
        return

    def forward(self, x, *args, **kwargs):
        compute_dtype = _common.autocast_dtype()
        adapter = None
        if not args and not kwargs and compute_dtype is not None and _common.on_gpu(x) \
                and x.dtype in (torch.float32, torch.float16, torch.bfloat16):
            adapter = _single_adapter(self)
        if adapter is None:
            return original(self, x, *args, **kwargs)
        result = self.base_layer(x)
        drop = self.lora_dropout[adapter]
        p = float(drop.p) if isinstance(drop, torch.nn.Dropout) and drop.training else 0.0
        if TORCH_DROPOUT_RNG and p > 0:
            xd = DropoutCast.apply(drop(x), 0.0, 0, compute_dtype)
        else:
            xd = DropoutCast.apply(x, p, _Seeds.next() if p > 0 else 0, compute_dtype)
        lo = self.lora_B[adapter](self.lora_A[adapter](xd))
        return ScaledAdd.apply(result, lo, self.scaling[adapter])

    forward._solution_patch = True
    cls.forward = forward
