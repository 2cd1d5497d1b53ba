"""Bit-level encodings of the 16-bit and 8-bit storage formats (oracle only).

numpy has float16 but neither bfloat16 nor float8_e4m3fn, so those two are
carried as raw integer bit patterns (``uint16`` / ``uint8``) and converted
here.  All roundings are round-to-nearest-even, which is what torch's
``Tensor.to(torch.bfloat16)`` and ``Tensor.to(torch.float8_e4m3fn)`` do; the
FP8 encoder only sees inputs already clamped to [-448, 448]
(``flashattn_tile/quant.py:125-127``), so it never needs the overflow rule.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("f32", "f16", "bf16")


# --------------------------------------------------------------------------- bf16
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    b = np.asarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round-to-nearest-even, NaN kept NaN."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


# --------------------------------------------------------------------------- e4m3
def _e4m3_table() -> np.ndarray:
    """float32 value of every e4m3fn code 0..255 (0x7F/0xFF are NaN)."""
    vals = np.zeros(256, dtype=np.float64)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 0xF and man == 0x7:
            vals[code] = np.nan
        elif exp == 0:
            vals[code] = sign * (man / 8.0) * 2.0 ** -6
        else:
            vals[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return vals.astype(np.float32)


E4M3_VALUES = _e4m3_table()
_E4M3_POS = E4M3_VALUES[:0x7F].astype(np.float64)  # codes 0x00..0x7E, ascending


def e4m3_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(bits, dtype=np.uint8)]


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """float32 (|x| <= 448) -> e4m3fn codes, round-to-nearest-even."""
    f = np.asarray(x, dtype=np.float32).astype(np.float64)
    mag = np.abs(f)
    if np.any(mag > 448.0):
        raise ValueError("f32_to_e4m3_bits expects inputs clamped to [-448, 448]")
    hi = np.searchsorted(_E4M3_POS, mag, side="left")
    hi = np.clip(hi, 0, len(_E4M3_POS) - 1)
    lo = np.clip(hi - 1, 0, len(_E4M3_POS) - 1)
    d_hi = np.abs(_E4M3_POS[hi] - mag)
    d_lo = np.abs(mag - _E4M3_POS[lo])
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & ((lo & 1) == 0))
    code = np.where(pick_lo, lo, hi).astype(np.uint8)
    # The sign survives rounding to zero (-0.0 encodes as 0x80), as in torch.
    return np.where(np.signbit(f), code | 0x80, code).astype(np.uint8)


# --------------------------------------------------------------------------- generic
def to_f32(data: np.ndarray, dtype: str) -> np.ndarray:
    """Decode a storage array of ``dtype`` ('f32'|'f16'|'bf16') to float32."""
    if dtype == "f32":
        return np.asarray(data, dtype=np.float32)
    if dtype == "f16":
        return np.asarray(data, dtype=np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(data)
    raise ValueError(f"unknown dtype {dtype!r}")


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 to the storage encoding of ``dtype``."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    raise ValueError(f"unknown dtype {dtype!r}")


def ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of ``dtype`` numbers at |x| (used for 1-ulp parity bounds)."""
    mant = {"f32": 23, "f16": 10, "bf16": 7}[dtype]
    min_exp = {"f32": -126, "f16": -14, "bf16": -126}[dtype]
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** min_exp)))
    return 2.0 ** (e - mant)
