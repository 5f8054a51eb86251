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

from . import _common, _lib, ops  # noqa: F401 - ops registers the custom operators

TORCH_DROPOUT_RNG = False


def _rows(t):
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


def _seed64(seed):
    """A Philox key as the kernels take it (unsigned 64-bit)."""
    return int(seed) & 0xFFFFFFFFFFFFFFFF


def _seed_arg(seed):
    """The same key as a signed 64-bit int (what a custom op's int argument holds)."""
    s = _seed64(seed)
    return s - (1 << 64) if s >= (1 << 63) else s


def dropout_scale_into(src, out, p, seed, scale):
    """qb_dropout_scale: out = dropout(src) * scale in out's dtype, the mask from the
    reference's Philox stream keyed by `seed` (p = 0: no mask)."""
    _lib.require_cuda(src, out, what="dropout_scale")
    s2, o2 = _rows(src), out.view(-1, out.shape[-1])
    M, N = s2.shape
    _lib.call("qb_dropout_scale", s2.data_ptr(), _lib.tag(s2.dtype), s2.stride(0), o2.data_ptr(),
              _lib.tag(o2.dtype), o2.stride(0), M, N, _seed64(seed), float(p), float(scale),
              _lib.stream(src.device), work=(M * N * (s2.element_size() + o2.element_size()), 0))
    return out


def scaled_add_into(base, lo, out, scaling):
    """qb_scaled_add: out = base + lo * scaling in out's dtype."""
    _lib.require_cuda(base, lo, out, what="scaled_add")
    b2, l2, o2 = _rows(base), _rows(lo), out.view(-1, out.shape[-1])
    M, N = b2.shape
    _lib.call("qb_scaled_add", b2.data_ptr(), _lib.tag(b2.dtype), b2.stride(0), l2.data_ptr(),
              _lib.tag(l2.dtype), l2.stride(0), o2.data_ptr(), _lib.tag(o2.dtype), o2.stride(0),
              M, N, float(scaling), _lib.stream(base.device),
              work=(M * N * (b2.element_size() + l2.element_size() + o2.element_size()), 0))
    return out


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


def dropout_apply_multi(x2, masks, out_dtype=None):
    """[x2 * mask_j * scale_j] for masks = [(bits_j, scale_j)] (1..4 of them) from recorded mask
    bits, x2 read once (C-ABI qb_dropout_apply_multi); each result equals dropout_apply's."""
    import ctypes
    rows, cols = x2.shape
    n = len(masks)
    if not 1 <= n <= 4:
        raise ValueError("dropout_apply_multi: 1..4 masks")
    words = (cols + 31) // 32
    for bits, _ in masks:
        if bits.dtype != torch.int32 or not bits.is_contiguous() or bits.shape != (rows, words):
            raise ValueError("dropout_apply_multi: bits must be contiguous int32 "
                             "[rows, ceil(cols / 32)]")
    _lib.require_cuda(x2, *(b for b, _ in masks), what="dropout_apply_multi")
    dtype = out_dtype or x2.dtype
    outs = [torch.empty((rows, cols), dtype=dtype, device=x2.device) for _ in masks]
    bits_arr = (ctypes.c_void_p * n)(*(b.data_ptr() for b, _ in masks))
    outs_arr = (ctypes.c_void_p * n)(*(o.data_ptr() for o in outs))
    ld_arr = (ctypes.c_int64 * n)(*(o.stride(0) for o in outs))
    sc_arr = (ctypes.c_float * n)(*(float(sc) for _, sc in masks))
    _lib.call("qb_dropout_apply_multi", x2.data_ptr(), _lib.tag(x2.dtype), x2.stride(0), n,
              bits_arr, outs_arr, _lib.tag(dtype), ld_arr, sc_arr, rows, cols,
              _lib.stream(x2.device),
              work=(rows * cols * (x2.element_size() + n * outs[0].element_size())
                    + sum(b.numel() * 4 for b, _ in masks), 0))
    return outs


# The C layout of qb_pack_segment (include/qlora_b200.h): a table of these, built once, drives
# the one launch of qb_adapter_pack.
PACK_SEGMENT = [("src", "<u8"), ("dst", "<u8"), ("src_ld", "<i8"), ("dst_ld", "<i8"),
                ("rows", "<i4"), ("cols", "<i4"), ("scale", "<f4"), ("pad", "<i4"),
                ("first_chunk", "<i8")]
PACK_CHUNK = 2048


def pack_table(segments):
    """The qb_pack_segment table of (src fp32 [rows, cols] view, dst bf16 view of the same shape,
    scale) triples, as bytes, and the launch's chunk count."""
    import numpy as np
    table = np.zeros(len(segments), dtype=np.dtype(PACK_SEGMENT))
    chunks = 0
    for i, (src, dst, scale) in enumerate(segments):
        if src.dim() != 2 or src.shape != dst.shape:
            raise ValueError("pack_table: 2-D src and dst of one shape")
        if src.dtype != torch.float32 or dst.dtype != torch.bfloat16:
            raise TypeError("pack_table: fp32 src, bf16 dst")
        if src.stride(1) != 1 or dst.stride(1) != 1:
            raise ValueError("pack_table: rows with unit column stride")
        rows, cols = src.shape
        table[i] = (src.data_ptr(), dst.data_ptr(), src.stride(0), dst.stride(0), rows, cols,
                    scale, 0, chunks)
        chunks += (rows * cols + PACK_CHUNK - 1) // PACK_CHUNK
    return table.tobytes(), chunks


class AdapterShadow:
    """bf16 copies of a model's LoRA operands, rebuilt by one launch per step (qb_adapter_pack)
    instead of one conversion per projection per use (forward, checkpoint recompute and
    backward: the casts autocast makes of lora_A / lora_B's fp32 weights at every call of
    solution/lora.py:172, with the scaling of :173 folded into B).

    For every module: a16 = bf16(A) [r, in] and sb16 = bf16(s B) [out, r]; for every (gate, up)
    pair also the [I, 2r] extra-K operands of the fused gate/up GEMM, [s B_g | 0] and [0 | s B_u]
    (their zero halves written once). The modules read them through `adapter16` while the
    shadow is attached; refresh() must run after every change of the adapters (the model runs it
    at the start of each forward) - the optimizer updates them in place, without a version bump
    under fused AdamW, so nothing else tells the copies are stale."""

    def __init__(self, modules, pairs=()):
        mods = list(modules)
        if not mods:
            raise ValueError("AdapterShadow: no modules")
        dev = mods[0].lora_A.device
        sizes = [m.lora_A.numel() + m.lora_B.numel() for m in mods]
        pair_sizes = [2 * g.lora_B.shape[0] * 2 * g.lora_B.shape[1] for g, _ in pairs]
        self.buf = torch.zeros(sum(sizes) + sum(pair_sizes), dtype=torch.bfloat16, device=dev)
        segs, off = [], 0
        for m in mods:
            a, b = m.lora_A.detach(), m.lora_B.detach()
            a16 = self.buf[off: off + a.numel()].view(a.shape)
            off += a.numel()
            sb16 = self.buf[off: off + b.numel()].view(b.shape)
            off += b.numel()
            segs += [(a, a16, 1.0), (b, sb16, float(m.scaling))]
            m._shadow16 = (a16, sb16)
        for g, u in pairs:
            I, r = g.lora_B.shape
            b1 = []
            for k, mod in enumerate((g, u)):
                t = self.buf[off: off + I * 2 * r].view(I, 2 * r)
                off += I * 2 * r
                segs.append((mod.lora_B.detach(), t[:, k * r:(k + 1) * r], float(mod.scaling)))
                b1.append(t)
            g._shadow_b1 = u._shadow_b1 = tuple(b1)
        table, self.chunks = pack_table(segs)
        self.nseg = len(segs)
        self.elements = sum(src.numel() for src, _, _ in segs)
        self.table = torch.frombuffer(bytearray(table), dtype=torch.uint8).to(dev)
        self.modules, self.pairs = mods, list(pairs)

    def refresh(self):
        _lib.call("qb_adapter_pack", self.table.data_ptr(), self.nseg, self.chunks,
                  _lib.stream(self.buf.device), work=(self.elements * 6, 0))

    def detach(self):
        for m in self.modules:
            m._shadow16 = None
        for g, u in self.pairs:
            g._shadow_b1 = u._shadow_b1 = None


class DropoutCast:
    """x -> dropout(x) * 1/(1-p) cast to out_dtype, the mask a function of (seed, flat index) only
    (lora.py:84-93): the custom op qlora_b200::dropout_scale, whose registered backward applies
    the same mask and scale to the gradient."""

    @staticmethod
    def apply(x, p, seed, out_dtype):
        _lib.require_cuda(x, what="dropout_scale")
        scale = 1.0 / (1.0 - p) if p > 0 else 1.0
        return torch.ops.qlora_b200.dropout_scale(x, float(p), _seed_arg(seed), scale, out_dtype)


class ScaledAdd:
    """out = base + lo * scaling in promote(base, lo) (lora.py:96-112): the custom op
    qlora_b200::scaled_add; its backward is (g, g * scaling in lo's dtype)."""

    @staticmethod
    def apply(base, lo, scaling):
        _lib.require_cuda(base, lo, what="scaled_add")
        return torch.ops.qlora_b200.scaled_add(base, lo, float(scaling))


class SeedStream:
    """Philox keys for the patched peft layers: key i of a process is a SplitMix64 mix of
    (torch.initial_seed(), i), kept below 2^31 like the reference's. A run with a fixed torch
    seed draws the same keys, and no torch generator (data order, init) is advanced."""

    count = 0

    @classmethod
    def next(cls):
        cls.count += 1
        z = (torch.initial_seed() * 0x9E3779B97F4A7C15 + cls.count * 0xBF58476D1CE4E5B9)
        z &= 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return (z ^ (z >> 31)) & 0x7FFFFFFF


# The reference's name for the seed source.
_Seeds = SeedStream


def _plain_adapter(layer):
    """The name of the adapter this patch computes for a peft LoRA layer: the only active one,
    a plain one (no DoRA-style variant) made of bias-free nn.Linear A and B behind an
    nn.Dropout or nn.Identity, on a layer that is neither disabled nor merged. None sends the
    call to peft's own forward."""
    if layer.disable_adapters or layer.merged:
        return None
    names = [n for n in layer.active_adapters if n in layer.lora_A]
    if len(names) != 1 or names[0] in getattr(layer, "lora_variant", {}):
        return None
    n = names[0]
    plain = all(type(m) is torch.nn.Linear and m.bias is None
                for m in (layer.lora_A[n], layer.lora_B[n]))
    if not plain or not isinstance(layer.lora_dropout[n], (torch.nn.Dropout, torch.nn.Identity)):
        return None
    return n


def patch():
    """peft's lora.bnb.Linear4bit.forward as base(x) + ScaledAdd(B(A(DropoutCast(x)))), the
    reference's composition (lora.py:145-176), for calls this package takes: autocast on, a
    float CUDA input, no extra arguments, one plain adapter. A no-op when peft is absent."""
    try:
        from peft.tuners.lora import bnb as lora_bnb
    except ImportError:
        return
    if getattr(lora_bnb, "Linear4bit", None) is None:
        return

    def build(original):
        def forward(self, x, *args, **kwargs):
            dtype = _common.autocast_dtype()
            fits = (not args and not kwargs and dtype is not None and _common.on_gpu(x)
                    and x.dtype in (torch.float32, torch.float16, torch.bfloat16))
            name = _plain_adapter(self) if fits else None
            if name is None:
                return original(self, x, *args, **kwargs)
            drop = self.lora_dropout[name]
            p = float(drop.p) if isinstance(drop, torch.nn.Dropout) and drop.training else 0.0
            base = self.base_layer(x)
            if p > 0 and TORCH_DROPOUT_RNG:     # torch's own mask, then the cast
                xd = DropoutCast.apply(drop(x), 0.0, 0, dtype)
            else:
                xd = DropoutCast.apply(x, p, SeedStream.next() if p > 0 else 0, dtype)
            return ScaledAdd.apply(base, self.lora_B[name](self.lora_A[name](xd)),
                                   self.scaling[name])
        return forward

    _common.install(lora_bnb.Linear4bit, "forward", build)
