"""ctypes binding of libqlora_b200.so, the C-ABI over the sm_100a kernels (include/qlora_b200.h).

The library is built in-tree (`python -m hackathon_b200.csrc.build`, or `__graft_entry__.build()`)
and loaded once per process. There is no fallback: when the library is missing, or the op runs
on a tensor that is not a CUDA tensor, the call raises.
"""

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqlora_b200.so")

F32, F16, BF16 = 0, 1, 2
_TAGS = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> argtypes (every function returns int status unless listed in _RESTYPE)
_SIGNATURES = {
    "qb_abi_version": [],
    "qb_last_error": [],
    "qb_nf4_dequant": [_p, _i64, _p, _i32, _p, _p, _f32, _i32, _i32, _p, _p, _i32, _p],
    "qb_nf4_quantize": [_p, _i32, _i64, _i32, _p, _p, _p, _p],
    "qb_nf4_double_quant_workspace": [_i64],
    "qb_nf4_double_quant": [_p, _i64, _i32, _p, _p, _p, _p, _p, _p],
    "qb_nf4_double_quant_noalloc_max_blocks": [],
    "qb_nf4_double_quant_noalloc": [_p, _i64, _i32, _p, _p, _p, _p, _p],
    "qb_rmsnorm_fwd": [_p, _i32, _i64, _p, _i32, _p, _i32, _i64, _p, _i64, _i64, _f32, _p],
    "qb_rmsnorm_bwd": [_p, _i32, _i64, _p, _i32, _i64, _p, _i32, _p, _p, _i32, _i64, _i64, _i64,
                       _p],
    "qb_rope_qk": [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i64, _i64, _i64, _i64, _i64, _i64p,
                   _i64p, _i64p, _i64p, _i64, _i64, _i32, _p],
    "qb_swiglu_fwd": [_p, _p, _p, _i32, _i64, _p],
    "qb_swiglu_bwd": [_p, _p, _p, _p, _p, _i32, _i64, _p],
    "qb_dropout_scale": [_p, _i32, _i64, _p, _i32, _i64, _i64, _i64, _u64, _f32, _f32, _p],
    "qb_scaled_add": [_p, _i32, _i64, _p, _i32, _i64, _p, _i32, _i64, _i64, _i64, _f32, _p],
    "qb_dropout_mask": [_p, _i32, _i64, _p, _i32, _i64, _p, _i64, _i64, _u64, _f32, _f32, _p],
    "qb_dropout_apply": [_p, _i32, _i64, _p, _p, _i32, _i64, _i64, _i64, _f32, _i32, _p],
    "qb_dropout_apply_multi": [_p, _i32, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _i64, _p],
    "qb_dropout_bits": [_p, _i64, _i64, _u64, _f32, _i32, _p],
    "qb_lora_xa": [_p, _i64, _p, _i64, _p, _i64, _f32, _p, _i64, _p, _i64, _i64, _i64, _i64,
                   _p],
    "qb_ce_rows": [_p, _i32, _i64, _p, _i64, _i64, _p, _p, _p, _p, _f32, _i32, _p],
    "qb_device_error": [_p],
    "qb_monitor_report": [_i32, ctypes.c_char_p, _i64],
    "qb_gemm_bf16": [_p, _i64, _i32, _p, _i64, _i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _p],
    "qb_gemm_bf16_acc_f32": [_p, _i64, _i32, _p, _i64, _i32, _f32, _f32, _p, _i64, _i64, _i64,
                             _i64, _p, _i64, _p],
    "qb_gemm_bf16_acc_f32_workspace": [_i64, _i64, _i64],
    "qb_gemm2_bf16": [_p, _i64, _i32, _p, _i64, _i32, _i64, _p, _i64, _i32, _p, _i64, _i32, _i64,
                      _p, _i64, _i32, _p, _p, _i64, _i64, _i64, _p],
    "qb_selftest_bounded_wait": [_i64, _p],
    "qb_gemm2_rope_bf16": [_p, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _p, _i64, _p, _p,
                           _p, _i64, _i64, _i64, _i64, _i64, _p],
    "qb_gemm_gateup_swiglu": [_p, _i64, _p, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64, _p,
                              _i64, _p, _p, _i64, _i64, _i64, _p],
    "qb_gemm_gateup_swiglu_masks": [_p, _i64, _p, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64,
                                    _p, _i64, _p, _p, _i64, _i64, _i64, _p, _i32, _p],
    "qb_mask_job_size": [],
    "qb_gemm_bf16_mask_acc": [_p, _i64, _p, _i64, _i32, _p, _i64, _f32, _p, _i64, _i64, _i64,
                              _i64, _p],
    "qb_nf4_linear_fwd": [_p, _i64, _p, _p, _p, _p, _f32, _i32, _p, _i64, _i64, _i64, _p, _p,
                          _i64, _p, _i64, _i64, _p, _i64, _p],
    "qb_nf4_linear_dgrad": [_p, _i64, _p, _p, _p, _p, _f32, _i32, _p, _i64, _i64, _i64, _p,
                            _i64, _p, _i64, _i64, _p, _i64, _p],
    "qb_linear_ce_vocab_tiles": [_i64],
    "qb_linear_ce_stats": [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _p],
    "qb_linear_ce_stats_logits": [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p],
    "qb_ce_grad_from_logits": [_p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _p],
    "qb_ce_reduce": [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p],
    "qb_linear_ce_grad": [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p],
    "qb_pack_segment_size": [],
    "qb_adapter_pack": [_p, _i32, _i64, _p],
}
_RESTYPE = {"qb_last_error": ctypes.c_char_p, "qb_nf4_double_quant_workspace": ctypes.c_int64,
            "qb_nf4_double_quant_noalloc_max_blocks": ctypes.c_int64,
            "qb_linear_ce_vocab_tiles": ctypes.c_int64,
            "qb_gemm_bf16_acc_f32_workspace": ctypes.c_int64,
            "qb_pack_segment_size": ctypes.c_int64, "qb_mask_job_size": ctypes.c_int64}

_lock = threading.Lock()
_lib = None


def load():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m hackathon_b200.csrc.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPE.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def exported_symbols():
    """Names of the C-ABI functions this binding declares."""
    return list(_SIGNATURES)


class KernelTimer:
    """Brackets every C-ABI call with CUDA events on the current stream (the stream every op
    here launches on) while active, with the call's algorithmic bytes and flops, so a caller
    can turn device time into achieved GB/s or TFLOP/s per kernel."""

    def __init__(self):
        self.records = []   # (name, start event, end event, bytes, flops, kernels launched)

    def __enter__(self):
        global _timer
        self._prev, _timer = _timer, self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = self._prev

    def summary(self):
        """{name: {"launches" (calls), "kernels", "ms_total", "bytes", "flops"}}
        (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for name, s, e, nbytes, flops, kernels in self.records:
            d = out.setdefault(name, {"launches": 0, "kernels": 0, "ms_total": 0.0, "bytes": 0,
                                      "flops": 0})
            d["launches"] += 1
            d["kernels"] += kernels
            d["ms_total"] += s.elapsed_time(e)
            d["bytes"] += nbytes
            d["flops"] += flops
        return out


_timer = None


def call(name, *args, work=(0, 0), kernels=1):
    """Calls a C-ABI entry point; raises RuntimeError with the library's message on failure.
    `work` = (algorithmic bytes, flops) of the call and `kernels` the kernels it launches,
    recorded when a KernelTimer is active."""
    lib = load()
    timer = _timer
    if timer is not None:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        status = getattr(lib, name)(*args)
        e.record()
        timer.records.append((name, s, e, int(work[0]), int(work[1]), int(kernels)))
    else:
        status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.qb_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (status {status}): {msg}")


def tag(dtype):
    try:
        return _TAGS[dtype]
    except KeyError:
        raise TypeError(f"qlora_b200: unsupported dtype {dtype}") from None


def ptr(t):
    return t.data_ptr() if t is not None else None


def stream(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def strides3(t):
    s = t.stride()
    return (ctypes.c_int64 * 3)(s[0], s[1], s[2])


def require_cuda(*tensors, what="op"):
    for t in tensors:
        if t is not None and not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise RuntimeError(f"qlora_b200 {what}: expects CUDA tensors (there is no CPU path)")
