"""NF4 (4-bit NormalFloat) weights with double-quantised block scales, and the 4-bit linear.

Mirrors the API of solution/nf4.py:
  dequantize_nf4(packed, quant_state, dtype)  -> dense weight (nf4.py:71-92)
  supported(quant_state)                      -> admission check (nf4.py:65-68)
  NF4Linear.apply(x, packed, quant_state, bias) (nf4.py:95-112)
  linear4bit / patch_linear4bit / project     (nf4.py:115-176)
and adds the producer of the format, `quantize_nf4`, since bitsandbytes is not a dependency.

Format (bitsandbytes' 4-bit layout): weight i of the flattened [out, in] matrix is a 4-bit index
into the 16-entry NF4 table; byte j holds weights 2j (high nibble) and 2j+1 (low nibble). Each
block of `blocksize` (64) weights has a scale. With double quantisation ("nested") the scales are
themselves stored as uint8 indices into a 256-entry signed dynamic table (`state2.code`) with one
fp32 scale per `state2.blocksize` (256) of them, after subtracting their mean (`offset`).

Every op here runs on the GPU through libqlora_b200.so; there is no CPU path.
"""

import numpy as np
import torch

from . import _lib, ops  # noqa: F401 - ops registers the qlora_b200 custom operators

# The NF4 code book of the QLoRA paper (Dettmers et al., 2023, appendix E): quantiles of N(0,1)
# normalised to [-1, 1], with an exact zero.
NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


def signed_dynamic_code(exponent_bits=7):
    """The 256-entry signed dynamic-tree code book used for the second-level scales.

    Dynamic tree quantisation (Dettmers, "8-bit approximations for parallelism in deep
    learning", 2016): for decade e = 0..exponent_bits-1 the magnitudes 10^(e-exponent_bits+1)
    times the midpoints of 2^e + 1 evenly spaced points in [0.1, 1], with both signs; plus 0
    and 1. Sorted ascending (the quantiser searches it)."""
    vals = []
    for e in range(exponent_bits):
        pts = np.linspace(0.1, 1.0, 2 ** e + 1)
        mids = (pts[:-1] + pts[1:]) / 2.0
        mag = (10.0 ** (e - exponent_bits + 1)) * mids
        vals.extend(mag.tolist())
        vals.extend((-mag).tolist())
    vals += [0.0, 1.0]
    vals += [0.0] * (256 - len(vals))
    return torch.tensor(sorted(vals), dtype=torch.float32)


_NF4_TABLES = {}
_CODE2_TABLES = {}


def nf4_table(device):
    """The NF4 code book as fp32 on `device` (cached per device)."""
    key = torch.device(device)
    table = _NF4_TABLES.get(key)
    if table is None:
        table = torch.tensor(NF4_CODE, dtype=torch.float32, device=key)
        _NF4_TABLES[key] = table
    return table


def _code2_table(device):
    key = torch.device(device)
    table = _CODE2_TABLES.get(key)
    if table is None:
        table = signed_dynamic_code().to(key)
        _CODE2_TABLES[key] = table
    return table


class QuantState:
    """The attributes of bitsandbytes' QuantState that the kernels read (duck-type compatible):
    shape, dtype, blocksize, quant_type, code (the NF4 table), absmax, nested, offset, state2."""

    def __init__(self, absmax, shape=None, code=None, blocksize=None, quant_type="nf4",
                 dtype=None, offset=None, state2=None):
        self.absmax = absmax
        self.shape = shape
        self.code = code
        self.blocksize = blocksize
        self.quant_type = quant_type
        self.dtype = dtype
        self.offset = offset
        self.state2 = state2
        self.nested = state2 is not None

    def to(self, device):
        """Moves every tensor to `device` (like bitsandbytes' QuantState.to)."""
        self.absmax = self.absmax.to(device)
        if self.code is not None:
            self.code = self.code.to(device)
        if self.nested:
            if torch.is_tensor(self.offset):
                self.offset = self.offset.to(device)
            self.state2.absmax = self.state2.absmax.to(device)
            self.state2.code = self.state2.code.to(device)
        return self


def supported(quant_state):
    """True when the kernels handle this quant state: NF4, 2-D, even block sizes."""
    return (quant_state is not None and quant_state.quant_type == "nf4"
            and len(quant_state.shape) == 2 and quant_state.blocksize % 2 == 0
            and (not quant_state.nested or quant_state.state2.blocksize % 2 == 0))


def quantize_nf4(weight, blocksize=64, compress_statistics=True, blocksize2=256):
    """(packed uint8 [n/2, 1], QuantState) of a 2-D CUDA weight, in the layout that
    bitsandbytes' quantize_4bit(quant_type="nf4") produces: blockwise absmax, nearest NF4 code,
    high nibble first; with compress_statistics the block scales are double-quantised.
    One device->host read fetches the offset (a Python float in the returned state)."""
    _lib.require_cuda(weight, what="quantize_nf4")
    if weight.dim() != 2:
        raise ValueError("quantize_nf4: expects a 2-D weight")
    w = weight.contiguous()
    n = w.numel()
    if n % 2:
        raise ValueError("quantize_nf4: the weight must have an even number of elements")
    dev = w.device
    lut = nf4_table(dev)
    n_blocks = (n + blocksize - 1) // blocksize
    packed = torch.empty((n // 2, 1), dtype=torch.uint8, device=dev)
    absmax = torch.empty(n_blocks, dtype=torch.float32, device=dev)
    s = _lib.stream(dev)
    _lib.call("qb_nf4_quantize", w.data_ptr(), _lib.tag(w.dtype), n, blocksize, lut.data_ptr(),
              packed.data_ptr(), absmax.data_ptr(), s)
    state = QuantState(absmax=absmax, shape=torch.Size(w.shape), code=lut, blocksize=blocksize,
                       quant_type="nf4", dtype=w.dtype)
    if compress_statistics:
        code2 = _code2_table(dev)
        n2 = (n_blocks + blocksize2 - 1) // blocksize2
        q = torch.empty(n_blocks, dtype=torch.uint8, device=dev)
        absmax2 = torch.empty(n2, dtype=torch.float32, device=dev)
        offset = torch.empty(1, dtype=torch.float32, device=dev)
        ws = torch.empty(int(_lib.load().qb_nf4_double_quant_workspace(n_blocks)),
                         dtype=torch.uint8, device=dev)
        _lib.call("qb_nf4_double_quant", absmax.data_ptr(), n_blocks, blocksize2, code2.data_ptr(),
                  q.data_ptr(), absmax2.data_ptr(), offset.data_ptr(), ws.data_ptr(), s)
        state2 = QuantState(absmax=absmax2, code=code2, blocksize=blocksize2,
                            quant_type="dynamic", dtype=torch.float32)
        state = QuantState(absmax=q, shape=torch.Size(w.shape), code=lut, blocksize=blocksize,
                           quant_type="nf4", dtype=w.dtype, offset=float(offset.item()),
                           state2=state2)
    return packed, state


def _scale_args(qs):
    """(absmax, code2, absmax2, offset, blocksize2) of a quant state as the kernels take them:
    code2 / absmax2 None for a state without double quantisation."""
    if qs.nested:
        return (qs.absmax, qs.state2.code, qs.state2.absmax, float(qs.offset),
                int(qs.state2.blocksize))
    return qs.absmax, None, None, 0.0, 2


def state_of(absmax, code2, absmax2, offset, blocksize, blocksize2, rows, cols):
    """A QuantState over the tensors a custom op receives (the inverse of _scale_args)."""
    state2 = None
    if code2 is not None:
        state2 = QuantState(absmax=absmax2, code=code2, blocksize=blocksize2,
                            quant_type="dynamic", dtype=torch.float32)
    return QuantState(absmax=absmax, shape=torch.Size((rows, cols)), blocksize=blocksize,
                      quant_type="nf4", offset=offset if state2 is not None else None,
                      state2=state2)


def dequant_into(out, packed, absmax, code2, absmax2, offset, blocksize, blocksize2):
    """qb_nf4_dequant into `out` (any float dtype, out.numel() weights); code2 / absmax2 None for
    single-level scales (fp32 absmax)."""
    _lib.require_cuda(packed, out, what="dequantize_nf4")
    n = out.numel()
    nested = code2 is not None
    if nested:
        absmax = absmax.contiguous()
        code2 = code2.float().contiguous()
        absmax2 = absmax2.float().contiguous()
        c2p, a2p = code2.data_ptr(), absmax2.data_ptr()
    else:
        absmax = absmax.float().contiguous()
        offset, blocksize2, c2p, a2p = 0.0, 2, None, None
    lut = nf4_table(packed.device)
    packed = packed.reshape(-1)
    work = (n // 2 + n * out.element_size() + absmax.numel() * absmax.element_size()
            + (absmax2.numel() * 4 if nested else 0), 0)
    _lib.call("qb_nf4_dequant", packed.data_ptr(), n, absmax.data_ptr(), int(nested), c2p, a2p,
              float(offset), int(blocksize), int(blocksize2), lut.data_ptr(), out.data_ptr(),
              _lib.tag(out.dtype), _lib.stream(packed.device), work=work)
    return out


def dequantize_nf4(packed, quant_state, dtype=torch.float16, out=None):
    """The weight [out_features, in_features] in `dtype`, rebuilt from the packed NF4 bytes
    (the custom op qlora_b200::nf4_dequant; with `out`, written into that buffer directly).
    Bit-exact with the reference kernel: fp32 scale = code2[q]*absmax2 + offset (two roundings),
    w = nf4[nibble]*scale, rounded to nearest even in `dtype`."""
    _lib.require_cuda(packed, what="dequantize_nf4")
    absmax, code2, absmax2, offset, bs2 = _scale_args(quant_state)
    if out is not None:
        return dequant_into(out, packed, absmax, code2, absmax2, offset,
                            int(quant_state.blocksize), bs2)
    rows, cols = (int(d) for d in quant_state.shape)
    return torch.ops.qlora_b200.nf4_dequant(packed, absmax, code2, absmax2, offset,
                                            int(quant_state.blocksize), bs2, rows, cols, dtype)


def fused_ok(x, quant_state):
    """True when the tcgen05 NF4 GEMM takes this call: bf16 activations on CUDA, a 2-D nested
    NF4 state with blocksize 64 and feature counts that are multiples of 128."""
    if not (x.is_cuda and x.dtype == torch.bfloat16 and supported(quant_state)):
        return False
    out_f, in_f = quant_state.shape
    return (quant_state.nested and quant_state.blocksize == 64 and in_f % 128 == 0
            and out_f % 64 == 0)


def _nf4_args(packed, qs):
    lut = nf4_table(packed.device)
    return (packed.data_ptr(), qs.absmax.data_ptr(), qs.state2.code.data_ptr(),
            qs.state2.absmax.data_ptr(), float(qs.offset), int(qs.state2.blocksize),
            lut.data_ptr())


def _rows2d(t):
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


# Token count from which a projection runs as "rebuild W into a transient bf16 copy
# (qb_nf4_dequant), then the TMA-fed GEMM with the LoRA term as extra K (qb_gemm2_bf16)" instead
# of the fused kernel. The fused kernel reads 0.5 byte per weight but its thread-written operand
# caps it near 1 PFLOP/s; the TMA-fed GEMM runs at 1.1-1.4 PFLOP/s and the rebuild costs one
# streaming pass over the weight (tens of microseconds), so long token counts win by 10-40%.
# From this many rows on, a projection rebuilds W into a transient bf16 buffer and runs the
# TMA-fed GEMM; below, the fused kernel rebuilds W inside the GEMM. Measured (forward with the
# rank-64 LoRA term, `bench.py --kernel nf4_fwd_fused / nf4_fwd_dequant`): at 18944 x 3584 the
# fused kernel wins at 512 rows (79 against 103 us) and ties at 1024, the transient weight wins
# from 2048 on (0.25 against 0.30 ms; 1.29 against 1.00 PFLOP/s at 8192 rows); at 3584 x 3584
# the transient weight wins at every size measured.
DEQUANT_GEMM_MIN_TOKENS = 2048

_WEIGHT_WS = {}


def _weight_workspace(device, out_f, in_f, slot=0):
    """A bf16 [out_f, in_f] scratch for the transient weight, one per (device, stream, slot):
    every user of it is ordered on that stream, so one buffer serves all projections in turn
    (slot 1 for an op that needs two weights at once)."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream, slot)
    buf = _WEIGHT_WS.get(key)
    if buf is None or buf.numel() < out_f * in_f:
        buf = torch.empty(out_f * in_f, dtype=torch.bfloat16, device=device)
        _WEIGHT_WS[key] = buf
    return buf[:out_f * in_f].view(out_f, in_f)


def uses_dequant_path(tokens, path=None):
    """True when a projection over `tokens` rows runs as transient bf16 weight + TMA-fed GEMM."""
    if path not in (None, "fused", "dequant"):
        raise ValueError(f"unknown path {path!r}")
    return path == "dequant" or (path is None and tokens >= DEQUANT_GEMM_MIN_TOKENS)


def nf4_linear_fwd(x, packed, qs, bias=None, u=None, lora_b_scaled=None, path=None,
                   residual=None, weight_out=None, rope=None, weight=None):
    """y = residual + x @ deq(W).T (+ bias) (+ u @ lora_b_scaled.T), bf16 in and out, fp32
    accumulation. path "fused": the tcgen05 kernel that rebuilds the NF4 weight in registers inside
    the GEMM; "dequant": W rebuilt into a transient bf16 copy, then the TMA-fed GEMM (bias, LoRA
    term and residual in its one accumulation / epilogue); None picks by token count
    (DEQUANT_GEMM_MIN_TOKENS). On the dequant path the copy goes to `weight_out` (bf16
    [out, in]) when given — a caller keeps it for the backward — else to a shared scratch;
    `weight` is a copy the caller already rebuilt (dequant path, no rebuild here).
    rope = (cos, sin) [S, 128]: the output's heads get the rotate-half RoPE of their token's
    position (row m = position m % S), in the GEMM epilogue on the dequant path.
    x [..., in] -> y [..., out]."""
    out_f, in_f = qs.shape
    x2 = _rows2d(x)
    T = x2.shape[0]
    r = 0 if u is None else u.shape[-1]
    u2 = None if u is None else _rows2d(u)
    lb = None if lora_b_scaled is None else lora_b_scaled.contiguous()
    res2 = None if residual is None else _rows2d(residual)
    if weight is not None or uses_dequant_path(T, path):
        from .gemm import gemm2
        w = weight
        if w is None:
            w = weight_out if weight_out is not None else _weight_workspace(x.device, out_f, in_f)
            dequantize_nf4(packed, qs, torch.bfloat16, out=w)
        if rope is not None:
            if res2 is not None:
                raise ValueError("nf4_linear_fwd: rope and residual do not combine")
            from .gemm import gemm2_rope
            y = gemm2_rope(x2, w, u2, lb, rope[0], rope[1], bias=bias)
        else:
            y = gemm2(x2, w, u2, lb, bias=bias, residual=res2)
        return y.view(*x.shape[:-1], out_f)
    y = torch.empty((T, out_f), dtype=torch.bfloat16, device=x.device)
    b = None if bias is None else bias.to(torch.bfloat16).contiguous()
    _lib.call("qb_nf4_linear_fwd", x2.data_ptr(), x2.stride(0), *_nf4_args(packed, qs), T, in_f,
              out_f, _lib.ptr(b), _lib.ptr(u2), u2.stride(0) if u2 is not None else 0,
              _lib.ptr(lb), lb.stride(0) if lb is not None else 0, r, y.data_ptr(), y.stride(0),
              _lib.stream(x.device), work=(0, 2 * T * out_f * (in_f + r)))
    if rope is not None:
        from .rope import rope_rows
        y = rope_rows(y, rope[0], rope[1])
    if res2 is not None:
        y += res2
    return y.view(*x.shape[:-1], out_f)


def nf4_linear_dgrad(dy, packed, qs, v=None, lora_a=None, path=None, weight=None):
    """dx = dy @ deq(W) (+ v @ lora_a), bf16 in and out, fp32 accumulation; `path` as in
    nf4_linear_fwd (the fused kernel reads W transposed from the packed codes; the dequant path
    reads the transient copy MN-major). `weight`: the bf16 copy a forward kept (skips the
    rebuild). dy [..., out] -> dx [..., in]."""
    out_f, in_f = qs.shape
    d2 = _rows2d(dy)
    T = d2.shape[0]
    r = 0 if v is None else v.shape[-1]
    v2 = None if v is None else _rows2d(v)
    la = None if lora_a is None else lora_a.contiguous()
    if weight is not None or uses_dequant_path(T, path):
        from .gemm import gemm2
        w = weight
        if w is None:
            w = dequantize_nf4(packed, qs, torch.bfloat16,
                               out=_weight_workspace(dy.device, out_f, in_f))
        dx = gemm2(d2, w.t(), v2, None if la is None else la.t())
        return dx.view(*dy.shape[:-1], in_f)
    dx = torch.empty((T, in_f), dtype=torch.bfloat16, device=dy.device)
    _lib.call("qb_nf4_linear_dgrad", d2.data_ptr(), d2.stride(0), *_nf4_args(packed, qs), T,
              in_f, out_f, _lib.ptr(v2), v2.stride(0) if v2 is not None else 0, _lib.ptr(la),
              la.stride(0) if la is not None else 0, r, dx.data_ptr(), dx.stride(0),
              _lib.stream(dy.device), work=(0, 2 * T * in_f * (out_f + r)))
    return dx.view(*dy.shape[:-1], in_f)


class NF4Linear:
    """y = x @ W.T + b, W rebuilt from NF4 in forward and again in backward (nothing dense is kept
    between them); W and b are frozen, the backward gives dX only (nf4.py:95-112). The
    reference's autograd.Function name, over the custom op qlora_b200::nf4_linear (whose
    registered backward is qlora_b200::nf4_linear_dgrad)."""

    @staticmethod
    def apply(x, packed, quant_state, bias):
        absmax, code2, absmax2, offset, bs2 = _scale_args(quant_state)
        out_f, in_f = (int(d) for d in quant_state.shape)
        return torch.ops.qlora_b200.nf4_linear(x, packed, absmax, code2, absmax2, offset,
                                               int(quant_state.blocksize), bs2, out_f, in_f,
                                               bias)


def _prepare(module, x):
    """The part of bitsandbytes' Linear4bit.forward before the matmul: (x, bias, input dtype), or
    None when the layer must take the original path (nf4.py:115-138)."""
    try:
        from bitsandbytes.nn.modules import fix_4bit_weight_quant_state_from_module
    except ImportError:
        fix_4bit_weight_quant_state_from_module = None
    if fix_4bit_weight_quant_state_from_module is not None:
        fix_4bit_weight_quant_state_from_module(module)
    quant_state = getattr(module.weight, "quant_state", None)
    if (not x.is_cuda or not supported(quant_state) or module.weight.requires_grad
            or (module.bias is not None and module.bias.requires_grad)):
        return None
    if not getattr(module, "compute_type_is_set", True):
        module.set_compute_type(x)
        module.compute_type_is_set = True
    inp_dtype = x.dtype
    compute_dtype = getattr(module, "compute_dtype", None)
    if compute_dtype is not None:
        x = x.to(compute_dtype)
    if x.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        return None
    bias = module.bias
    if bias is not None:
        if bias.dtype != x.dtype:
            bias.data = bias.data.to(x.dtype)
        bias = bias.to(x.dtype)
    return x, bias, inp_dtype


def _upstream_forward(module):
    """bitsandbytes' own forward of the module's class (the one patch_linear4bit replaced)."""
    from ._common import PATCH_MARK
    fwd = type(module).forward
    return fwd.__wrapped__ if getattr(fwd, PATCH_MARK, False) else fwd


def linear4bit(module, x, keep_compute_dtype=False):
    """bitsandbytes' Linear4bit.forward on our kernels; a layer they do not take runs
    bitsandbytes' own forward. With keep_compute_dtype the output stays in the compute dtype
    instead of being cast back to the input dtype (nf4.py:141-149)."""
    prepared = _prepare(module, x)
    if prepared is None:
        return _upstream_forward(module)(module, x)
    x, bias, inp_dtype = prepared
    out = NF4Linear.apply(x, module.weight, module.weight.quant_state, bias)
    return out if keep_compute_dtype else out.to(inp_dtype)


def patch_linear4bit():
    """bitsandbytes' Linear4bit.forward through linear4bit (nf4.py:155-166)."""
    import bitsandbytes.nn.modules as bnb_modules

    from ._common import install
    install(bnb_modules.Linear4bit, "forward", lambda original: lambda self, x: linear4bit(self, x))


def project(layer, x):
    """An MLP projection that keeps its output in the compute dtype when it is a plain 4-bit
    layer; anything else runs as it is (nf4.py:169-176)."""
    try:
        import bitsandbytes.nn.modules as bnb_modules
        plain = (bnb_modules.Linear4bit, bnb_modules.LinearNF4)
    except ImportError:
        plain = ()
    if type(layer) in plain:
        return linear4bit(layer, x, keep_compute_dtype=True)
    return layer(x)
