"""bf16 GEMM on the tcgen05 kernel (C-ABI qb_gemm_bf16), for the contractions of the step."""

import ctypes

import torch

from . import _lib


def _operand(t):
    """(tensor, leading dim, mn_major) of a 2-D operand that is row-major or a transposed view.
    A tensor map needs a 16-byte aligned base and a leading dimension of whole 16-byte units (8
    bf16): other operands are copied into a row-major buffer with padded rows. A single row may
    take any leading dimension (only row 0 is read)."""
    rows, cols = t.shape
    if t.data_ptr() % 16 == 0:
        if t.stride(-1) == 1 or cols == 1:
            ld = t.stride(0) if rows > 1 else (cols + 7) // 8 * 8
            if ld % 8 == 0 and ld >= cols:
                return t, ld, False
        if t.stride(0) == 1 and rows > 1 and t.stride(1) % 8 == 0 and t.stride(1) >= rows:
            return t, t.stride(1), True
    ld = (cols + 7) // 8 * 8
    buf = torch.empty((rows, ld), dtype=t.dtype, device=t.device)[:, :cols]
    buf.copy_(t)
    return buf, ld, False


def gemm(a, b_t, out=None, out_dtype=torch.bfloat16, bias=None):
    """out[M, N] = a[M, K] @ b_t[N, K].T (+ bias) with fp32 accumulation.

    `a` and `b_t` are bf16; each may be row-major or the transpose view of a row-major tensor
    (read as MN-major, no copy)."""
    _lib.require_cuda(a, b_t, what="gemm")
    if a.dtype != torch.bfloat16 or b_t.dtype != torch.bfloat16:
        raise TypeError("gemm: bf16 operands only")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError(f"gemm: inner dimensions differ ({K} vs {K2})")
    a, lda, a_mn = _operand(a)
    b_t, ldb, b_mn = _operand(b_t)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if bias is not None:
        bias = bias.float().contiguous()
    _lib.call("qb_gemm_bf16", a.data_ptr(), lda, int(a_mn), b_t.data_ptr(), ldb, int(b_mn),
              out.data_ptr(), out.stride(0), _lib.tag(out.dtype), _lib.ptr(bias), M, N, K,
              _lib.stream(a.device), work=(0, 2 * M * N * K))
    return out


def gemm_acc_f32(a, b_t, out, alpha=1.0, accumulate=True):
    """out[M, N] (fp32, in place) = (out if accumulate else 0) + alpha * a[M, K] @ b_t[N, K].T
    on the tcgen05 GEMM (without accumulate, out is not read: it may hold anything), K split
    across the SMs when the output has too few tiles (C-ABI qb_gemm_bf16_acc_f32; the partial
    products meet in a workspace and are summed in a fixed order, so the result is the same on
    every run): the skinny LoRA weight gradients, whose K is the token count. Operands bf16,
    row-major or transposed views."""
    _lib.require_cuda(a, b_t, out, what="gemm_acc_f32")
    if a.dtype != torch.bfloat16 or b_t.dtype != torch.bfloat16 or out.dtype != torch.float32:
        raise TypeError("gemm_acc_f32: bf16 operands, fp32 output")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2 or out.shape != (M, N) or out.stride(-1) != 1:
        raise ValueError("gemm_acc_f32: shapes do not match")
    a, lda, a_mn = _operand(a)
    b_t, ldb, b_mn = _operand(b_t)
    nws = int(_lib.load().qb_gemm_bf16_acc_f32_workspace(M, N, K)) if M and N and K else 0
    ws = torch.empty(nws, dtype=torch.float32, device=a.device) if nws else None
    _lib.call("qb_gemm_bf16_acc_f32", a.data_ptr(), lda, int(a_mn), b_t.data_ptr(), ldb,
              int(b_mn), float(alpha), 1.0 if accumulate else 0.0, out.data_ptr(),
              out.stride(0), M, N, K, _lib.ptr(ws),
              nws, _lib.stream(a.device),
              work=((M + N) * K * 2 + M * N * 4 * (2 if accumulate else 1), 2 * M * N * K),
              kernels=2 if nws else 1)
    return out


def lora_products(g, u, xd, b_scaled, a_shape, scaling, need_a=True, need_b=True):
    """The LoRA branch's backward products for one projection, all on the tcgen05 GEMM:
    V = g (s B) [T, r] (bf16; the input gradient's term), and when wanted dA = V^T xd [r, in]
    and dB = s g^T U [out, r] (fp32, the tokens split across the SMs). g [T, out],
    u = xd A^T [T, r], xd [T, in], b_scaled = s B [out, r], all bf16 (row-major, or column
    slices of a wider buffer). Returns (V, dA or None, dB or None)."""
    v = gemm(g, b_scaled.t())
    da = db = None
    if need_a:
        da = torch.empty(a_shape, dtype=torch.float32, device=g.device)
        gemm_acc_f32(v.t(), xd.t(), da, accumulate=False)
    if need_b:
        db = torch.empty((g.shape[1], u.shape[1]), dtype=torch.float32, device=g.device)
        gemm_acc_f32(g.t(), u.t(), db, alpha=scaling, accumulate=False)
    return v, da, db


def gemm2(a0, b0_t, a1, b1_t, out=None, out_dtype=torch.bfloat16, bias=None, residual=None):
    """out[M, N] = residual + a0 @ b0_t.T + a1 @ b1_t.T (+ bias) in one fp32 accumulation and one
    rounding: the second term is extra K of the same tcgen05 GEMM (C-ABI qb_gemm2_bf16). a0/a1
    row-major; b0_t/b1_t both row-major or both transposed views of row-major tensors; a1 may be
    None; residual [M, N] in out_dtype with unit column stride."""
    if (a1 is None or a1.shape[-1] == 0) and residual is None:
        return gemm(a0, b0_t, out=out, out_dtype=out_dtype, bias=bias)
    tensors = (a0, b0_t) if a1 is None else (a0, b0_t, a1, b1_t)
    _lib.require_cuda(*tensors, what="gemm2")
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise TypeError("gemm2: bf16 operands only")
    M, K0 = a0.shape
    N, K0b = b0_t.shape
    if K0 != K0b:
        raise ValueError(f"gemm2: shapes {tuple(a0.shape)} {tuple(b0_t.shape)} do not match")
    a0 = a0 if a0.stride(-1) == 1 else a0.contiguous()
    b0_t, ldb0, b0_mn = _operand(b0_t)
    K1, a1p, lda1, b1p, ldb1 = 0, None, 0, None, 0
    if a1 is not None and a1.shape[-1] > 0:
        M1, K1 = a1.shape
        N1, K1b = b1_t.shape
        if K1 != K1b or M1 != M or N1 != N:
            raise ValueError(f"gemm2: shapes {tuple(a1.shape)} {tuple(b1_t.shape)} do not match "
                             f"[{M}, {N}]")
        a1 = a1 if a1.stride(-1) == 1 else a1.contiguous()
        b1_t, ldb1, b1_mn = _operand(b1_t)
        if b0_mn != b1_mn:   # the kernel takes both B operands in one layout
            b1_t = b1_t.t().contiguous().t() if b0_mn else b1_t.contiguous()
            b1_t, ldb1, b1_mn = _operand(b1_t)
        a1p, lda1, b1p = a1.data_ptr(), a1.stride(0), b1_t.data_ptr()
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a0.device)
    if bias is not None:
        bias = bias.float().contiguous()
    ldr = 0
    if residual is not None:
        if residual.shape != (M, N) or residual.dtype != out.dtype or residual.stride(-1) != 1:
            raise ValueError("gemm2: residual must be [M, N] in the output dtype, unit stride")
        ldr = residual.stride(0)
    _lib.call("qb_gemm2_bf16", a0.data_ptr(), a0.stride(0), 0, b0_t.data_ptr(), ldb0, int(b0_mn),
              K0, a1p, lda1, 0, b1p, ldb1, int(b0_mn), K1, out.data_ptr(), out.stride(0),
              _lib.tag(out.dtype), _lib.ptr(bias), _lib.ptr(residual), ldr, M, N,
              _lib.stream(a0.device), work=(0, 2 * M * N * (K0 + K1)))
    return out


def gemm2_rope(a0, b0_t, a1, b1_t, cos, sin, bias=None):
    """rope(bf16(a0 @ b0_t.T + a1 @ b1_t.T + bias)) for a q/k projection with heads of 128 dims
    (C-ABI qb_gemm2_rope_bf16): row m is the token at position m % S of cos/sin [S, 128]. All
    operands bf16 row-major; a1 may be None. Returns [M, N] bf16."""
    tensors = (a0, b0_t, cos, sin) if a1 is None else (a0, b0_t, a1, b1_t, cos, sin)
    _lib.require_cuda(*tensors, what="gemm2_rope")
    M, K0 = a0.shape
    N = b0_t.shape[0]
    for t in tensors:
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise TypeError("gemm2_rope: bf16 row-major operands")
    S = cos.shape[0]
    if cos.shape != sin.shape or cos.shape[1] != 128 or cos.stride() != sin.stride():
        raise ValueError("gemm2_rope: cos/sin [S, 128] with one layout")
    K1, a1p, lda1, b1p, ldb1 = 0, None, 0, None, 0
    if a1 is not None and a1.shape[1] > 0:
        K1 = a1.shape[1]
        a1p, lda1, b1p, ldb1 = a1.data_ptr(), a1.stride(0), b1_t.data_ptr(), b1_t.stride(0)
    if bias is not None:
        bias = bias.float().contiguous()
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a0.device)
    _lib.call("qb_gemm2_rope_bf16", a0.data_ptr(), a0.stride(0), b0_t.data_ptr(), b0_t.stride(0),
              K0, a1p, lda1, b1p, ldb1, K1, out.data_ptr(), out.stride(0), _lib.ptr(bias),
              cos.data_ptr(), sin.data_ptr(), cos.stride(0), S, 128, M, N,
              _lib.stream(a0.device), work=(0, 2 * M * N * (K0 + K1)))
    return out


class MaskJob(ctypes.Structure):
    """qb_mask_job: one dropout mask drawn as bits [rows, ceil(cols / 32)] int32 words."""
    _fields_ = [("bits", ctypes.c_void_p), ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("seed", ctypes.c_uint64), ("p", ctypes.c_float)]


MAX_MASK_JOBS = 8


def mask_jobs_array(jobs):
    """A qb_mask_job array of (bits, rows, cols, seed, p) tuples; bits an int32 CUDA tensor of
    [rows, ceil(cols / 32)] contiguous words."""
    if len(jobs) > MAX_MASK_JOBS:
        raise ValueError(f"at most {MAX_MASK_JOBS} mask jobs per launch")
    arr = (MaskJob * max(len(jobs), 1))()
    for i, (bits, rows, cols, seed, p) in enumerate(jobs):
        if (bits.dtype != torch.int32 or not bits.is_contiguous()
                or bits.shape != (rows, (cols + 31) // 32)):
            raise ValueError("mask job: bits must be contiguous int32 [rows, ceil(cols / 32)]")
        arr[i] = MaskJob(bits.data_ptr(), rows, cols, int(seed) & 0xFFFFFFFFFFFFFFFF, float(p))
    return arr


def gemm_gateup_swiglu(x, w_gate, w_up, lora_u=None, b1_gate=None, b1_up=None, save_gu=False,
                       mask_jobs=None):
    """h = silu(g) * u for the gate/up pair in one tcgen05 GEMM (C-ABI qb_gemm_gateup_swiglu):
    g = x @ w_gate.T (+ lora_u @ b1_gate.T), u = x @ w_up.T (+ lora_u @ b1_up.T), rounded to bf16
    before the SwiGLU. Returns h, or (h, g, u) with save_gu. All bf16, row-major.
    mask_jobs: up to 8 (bits, rows, cols, seed, p) dropout masks the same launch draws as bits
    in warps beside the GEMM's (qb_gemm_gateup_swiglu_masks); the bits equal dropout_bits'."""
    _lib.require_cuda(x, w_gate, w_up, what="gemm_gateup_swiglu")
    M, K0 = x.shape
    I, K0w = w_gate.shape
    if w_up.shape != w_gate.shape or K0w != K0 or w_up.stride(0) != w_gate.stride(0):
        raise ValueError("gemm_gateup_swiglu: gate and up weights must match x and each other")
    for t in (x, w_gate, w_up):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise TypeError("gemm_gateup_swiglu: bf16 row-major operands")
    K1, up_, ldu1, bg, bu, ldb1 = 0, None, 0, None, None, 0
    if lora_u is not None:
        K1 = lora_u.shape[1]
        if lora_u.shape[0] != M or b1_gate.shape != (I, K1) or b1_up.shape != (I, K1) or \
                b1_up.stride(0) != b1_gate.stride(0):
            raise ValueError("gemm_gateup_swiglu: LoRA operands do not match")
        up_, ldu1, bg, bu, ldb1 = (lora_u.data_ptr(), lora_u.stride(0), b1_gate.data_ptr(),
                                   b1_up.data_ptr(), b1_gate.stride(0))
    h = torch.empty((M, I), dtype=torch.bfloat16, device=x.device)
    g = u = None
    if save_gu:
        g, u = torch.empty_like(h), torch.empty_like(h)
    args = (x.data_ptr(), x.stride(0), w_gate.data_ptr(), w_up.data_ptr(), w_gate.stride(0), K0,
            up_, ldu1, bg, bu, ldb1, K1, h.data_ptr(), h.stride(0), _lib.ptr(g), _lib.ptr(u), I,
            M, I)
    if mask_jobs:
        _lib.require_cuda(*(j[0] for j in mask_jobs), what="gemm_gateup_swiglu")
        _lib.call("qb_gemm_gateup_swiglu_masks", *args, mask_jobs_array(mask_jobs),
                  len(mask_jobs), _lib.stream(x.device), work=(0, 2 * M * 2 * I * (K0 + K1)))
    else:
        _lib.call("qb_gemm_gateup_swiglu", *args, _lib.stream(x.device),
                  work=(0, 2 * M * 2 * I * (K0 + K1)))
    return (h, g, u) if save_gu else h


def gemm_mask_acc(a, b_t, bits, scale, out):
    """out[M, N] (bf16, in place) += scale * mask .* (a @ b_t.T), mask from the dropout bit words
    `bits` [M, ceil(N/32)] int32 (C-ABI qb_gemm_bf16_mask_acc). a row-major [M, K]; b_t row-major
    [N, K] or the transposed view of a row-major [K, N]."""
    _lib.require_cuda(a, b_t, bits, out, what="gemm_mask_acc")
    if a.dtype != torch.bfloat16 or b_t.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise TypeError("gemm_mask_acc: bf16 operands and output only")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2 or out.shape != (M, N) or bits.shape[0] != M or bits.shape[1] * 32 < N:
        raise ValueError("gemm_mask_acc: shapes do not match")
    a = a if a.stride(-1) == 1 else a.contiguous()
    b_t, ldb, b_mn = _operand(b_t)
    _lib.call("qb_gemm_bf16_mask_acc", a.data_ptr(), a.stride(0), b_t.data_ptr(), ldb, int(b_mn),
              bits.data_ptr(), bits.stride(0), float(scale), out.data_ptr(), out.stride(0), M, N,
              K, _lib.stream(a.device), work=(2 * M * N * out.element_size() + bits.numel() * 4
                                              + (M + N) * K * 2, 0))
    return out


def device_error():
    """Raises if a tensor-core kernel on this device gave up a bounded wait (synchronises)."""
    _lib.call("qb_device_error", _lib.stream())
