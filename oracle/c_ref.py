"""Loader of the C restatement (oracle/libnf4_ref.so) — TEST INFRASTRUCTURE ONLY."""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libnf4_ref.so")


def build():
    """Compiles libnf4_ref.so with the committed Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = ctypes.CDLL(LIB)
        p = ctypes.c_void_p
        lib.nf4_dequant_bf16.argtypes = [p, ctypes.c_int64, p, p, p, ctypes.c_float, ctypes.c_int,
                                         ctypes.c_int, p, p, ctypes.c_int]
        lib.nf4_dequant_bf16.restype = ctypes.c_int
        _lib = lib
    return _lib


def dequant_nf4_bf16(packed, n_weights, absmax_q, code2, absmax2, offset, blocksize=64,
                     blocksize2=256, lut=None, threads=1):
    """bf16 bit patterns (uint16) of a nested-NF4 tensor, computed in C."""
    from .nf4_ref import NF4_CODE
    lut = NF4_CODE if lut is None else np.asarray(lut, np.float32)
    arrs = [np.ascontiguousarray(a) for a in (packed, absmax_q, code2, absmax2, lut)]
    arrs[2] = arrs[2].astype(np.float32)
    arrs[3] = arrs[3].astype(np.float32)
    out = np.empty(n_weights, dtype=np.uint16)
    ptr = [a.ctypes.data_as(ctypes.c_void_p) for a in arrs]
    rc = _load().nf4_dequant_bf16(ptr[0], n_weights, ptr[1], ptr[2], ptr[3], float(offset),
                                  blocksize, blocksize2, ptr[4],
                                  out.ctypes.data_as(ctypes.c_void_p), threads)
    if rc != 0:
        raise ValueError("nf4_dequant_bf16: bad arguments")
    return out
