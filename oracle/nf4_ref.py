"""numpy restatements of the reference's integer/byte work — TEST INFRASTRUCTURE ONLY.

  dequant_nf4      solution/nf4.py:25-49 (nf4_dequant_kernel), all fp32 ops in numpy float32
                   (IEEE round-to-nearest-even, no fused multiply-add), output rounded RNE
  quantize_nf4     the first-level NF4 quantiser of bitsandbytes' quantize_4bit (used by
                   solution/test_kernels.py:48-49): blockwise absmax, nearest code, high nibble
                   first — restated from the format's published description
  double_quant     the second level: offset = mean(absmax), blocks of 256, nearest code2 entry
  philox_uniform   Triton's tl.rand(seed, offset) (Philox-4x32-10, Salmon et al. SC'11) as used
                   by solution/lora.py:41-42
  dropout_scale    solution/lora.py:29-46 (lora_dropout_scale_kernel)

bitsandbytes (unpinned: the reference has no lock file, and it is not installed) defines the
format; the dequant kernel reads the code book and code2 as inputs, so parity here does not
depend on their exact contents.
"""

import numpy as np

NF4_CODE = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)


def f32_to_bf16_bits(x):
    """fp32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays a quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), rounded)


def bf16_bits_to_f32(u):
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_nf4_f32(packed, n_weights, absmax, nested, code2, absmax2, offset, blocksize,
                    blocksize2, lut=NF4_CODE, start=0):
    """The fp32 weights [start, start + n_weights) before the output cast (nf4.py:25-49);
    `packed` and the scale arrays are the whole tensor's."""
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    idx = np.arange(start, start + n_weights, dtype=np.int64)
    byte = packed[idx // 2].astype(np.int64)
    nib = np.where(idx % 2 == 0, (byte >> 4) & 15, byte & 15)   # high nibble first (:30, :45-47)
    blk = idx // blocksize
    lut = np.asarray(lut, dtype=np.float32)
    if nested:
        q = np.asarray(absmax, dtype=np.uint8)[blk]
        scale = np.asarray(code2, dtype=np.float32)[q] * \
            np.asarray(absmax2, dtype=np.float32)[blk // blocksize2]      # rounded multiply
        scale = scale + np.float32(offset)                                 # rounded add (:38-42)
    else:
        scale = np.asarray(absmax, dtype=np.float32)[blk]
    return (lut[nib] * scale).astype(np.float32)


def dequant_nf4(packed, n_weights, absmax, nested, code2, absmax2, offset, blocksize, blocksize2,
                out="bf16", lut=NF4_CODE, start=0):
    """Dequantised weights: float32 / float16 arrays, or bf16 as uint16 bit patterns."""
    w = dequant_nf4_f32(packed, n_weights, absmax, nested, code2, absmax2, offset, blocksize,
                        blocksize2, lut, start)
    if out == "f32":
        return w
    if out == "f16":
        return w.astype(np.float16)   # numpy rounds to nearest even
    if out == "bf16":
        return f32_to_bf16_bits(w)
    raise ValueError(out)


def quantize_nf4(w, blocksize=64, lut=NF4_CODE):
    """(packed uint8 [n/2], absmax fp32 [nblocks]): per block absmax = max|w|, v = w * (1/absmax),
    index of the nearest code (first one on a tie), two per byte, high nibble first."""
    w = np.asarray(w, dtype=np.float32).reshape(-1)
    n = w.size
    nb = (n + blocksize - 1) // blocksize
    pad = np.zeros(nb * blocksize, dtype=np.float32)
    pad[:n] = w
    blocks = pad.reshape(nb, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    inv = np.where(absmax > 0, np.float32(1.0) / np.where(absmax > 0, absmax, 1), 0).astype(np.float32)
    v = (blocks * inv[:, None]).reshape(-1)[:n]
    d = np.abs(v[:, None] - np.asarray(lut, dtype=np.float32)[None, :])
    q = np.argmin(d, axis=1).astype(np.uint8)          # argmin returns the first minimum
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8)
    return packed, absmax


def double_quant(absmax, code2, blocksize2=256):
    """(codes uint8, absmax2 fp32, offset fp32) of the fp32 block scales."""
    a = np.asarray(absmax, dtype=np.float32)
    offset = np.float32(a.astype(np.float64).mean())
    c = a - offset
    nb = (a.size + blocksize2 - 1) // blocksize2
    code2 = np.asarray(code2, dtype=np.float32)
    q = np.empty(a.size, dtype=np.uint8)
    absmax2 = np.empty(nb, dtype=np.float32)
    for j in range(nb):
        blk = c[j * blocksize2:(j + 1) * blocksize2]
        m = np.float32(np.abs(blk).max())
        absmax2[j] = m
        inv = np.float32(1.0) / m if m > 0 else np.float32(0.0)
        v = blk * inv
        lo = np.searchsorted(code2, v, side="left").clip(0, 255)
        prev = (lo - 1).clip(0, 255)
        take_prev = (lo > 0) & (np.abs(v - code2[prev]) <= np.abs(code2[lo] - v))
        q[j * blocksize2:(j + 1) * blocksize2] = np.where(take_prev, prev, lo)
    return q, absmax2, offset


_M_A, _M_B = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W_A, _W_B = 0x9E3779B9, 0xBB67AE85
_MASK32 = np.uint64(0xFFFFFFFF)


def philox_first_word(seed, offsets, rounds=10):
    """First output word of Philox-4x32 with key (seed low, seed high) and counter
    (offset, 0, 0, 0)."""
    c0 = (np.asarray(offsets, dtype=np.int64) & 0xFFFFFFFF).astype(np.uint64)
    c1 = np.zeros_like(c0)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = int(seed) & 0xFFFFFFFF
    k1 = (int(seed) >> 32) & 0xFFFFFFFF
    for _ in range(rounds):
        pb = _M_B * c2
        pa = _M_A * c0
        n0 = (pb >> np.uint64(32)) ^ c1 ^ np.uint64(k0)
        n2 = (pa >> np.uint64(32)) ^ c3 ^ np.uint64(k1)
        c0, c1, c2, c3 = n0 & _MASK32, pb & _MASK32, n2 & _MASK32, pa & _MASK32
        k0 = (k0 + _W_A) & 0xFFFFFFFF
        k1 = (k1 + _W_B) & 0xFFFFFFFF
    return c0.astype(np.uint32)


def philox_uniform(seed, offsets):
    """tl.rand(seed, offsets): the word read as int32, x<0 -> -x-1, times 4.6566127342e-10 (fp32)."""
    x = philox_first_word(seed, offsets).view(np.int32)
    x = np.where(x < 0, ~x, x)
    return x.astype(np.float32) * np.float32(4.6566127342e-10)


def dropout_keep(seed, rows, cols, p, row_range=None):
    """Boolean keep mask [rows, cols] of the reference's dropout kernel (lora.py:40-43):
    offset = int32(row * cols + col), keep = rand > p. row_range=(lo, hi): only those rows of
    the [rows, cols] tensor's mask (offsets as in the whole tensor)."""
    lo, hi = (0, rows) if row_range is None else row_range
    r = np.arange(lo, hi, dtype=np.int64)[:, None]
    c = np.arange(cols, dtype=np.int64)[None, :]
    return philox_uniform(seed, r * cols + c) > np.float32(p)


def dropout_scale(x, p, seed, scale):
    """fp32 result of lora_dropout_scale_kernel on a 2-D float32 array."""
    x = np.asarray(x, dtype=np.float32)
    s = np.float32(scale)
    if p > 0:
        keep = dropout_keep(seed, x.shape[0], x.shape[1], p)
        return np.where(keep, x * s, np.float32(0.0)).astype(np.float32)
    return (x * s).astype(np.float32)
