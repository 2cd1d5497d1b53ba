"""Per-(page, KV-head) INT8 / FP8-e4m3 scales, restated in numpy (oracle only).

Follows ``flashattn_tile/quant.py:84-191``:

* scale = ``max(absmax / maxval, 1e-8)`` with absmax over (token, dim) of
  each (page, KV head) (``quant.py:114-117``);
* INT8: ``round_half_even(x / scale)`` clamped to [-127, 127]
  (``quant.py:122-124``);
* FP8 e4m3fn: ``x / scale`` clamped to [-448, 448], then cast with
  round-to-nearest-even (``quant.py:125-127``);
* dequantisation: ``q.float() * scale`` (``quant.py:159-161``).

FP8 codes are carried as ``uint8`` bit patterns (see ``oracle.numerics``).
"""

from __future__ import annotations

import numpy as np

from . import numerics

INT8_MAX = 127.0
FP8_MAX = 448.0
MIN_SCALE = 1e-8


def quantize_kv_pages(k_f32: np.ndarray, v_f32: np.ndarray, mode: str):
    """Returns ``(qk, qv, scale_k, scale_v)``; scales are fp32 ``[pages, Hkv]``."""
    if k_f32.shape != v_f32.shape:
        raise ValueError(f"k/v shape mismatch: {k_f32.shape} vs {v_f32.shape}")
    if k_f32.ndim != 4:
        raise ValueError("cache must be [num_pages, page_size, num_kv_heads, head_dim]")
    if mode not in ("int8", "float8_e4m3fn", "fp8"):
        raise ValueError(f"unknown quantisation mode {mode!r}; expected 'int8' or 'float8_e4m3fn'")
    max_val = np.float32(INT8_MAX if mode == "int8" else FP8_MAX)
    out = []
    for x in (np.asarray(k_f32, np.float32), np.asarray(v_f32, np.float32)):
        amax = np.abs(x).max(axis=(1, 3))
        scale = np.maximum(amax / max_val, np.float32(MIN_SCALE)).astype(np.float32)
        scaled = x / scale[:, None, :, None]
        if mode == "int8":
            qx = np.clip(np.round(scaled), -max_val, max_val).astype(np.int8)
        else:
            qx = numerics.f32_to_e4m3_bits(np.clip(scaled, -max_val, max_val))
        out.append((qx, scale))
    (qk, sk), (qv, sv) = out
    return qk, qv, sk, sv


def dequantize_kv_pages(qk, qv, scale_k, scale_v, mode: str):
    """fp32 ``q * scale`` (the caller rounds to its output dtype)."""
    if qk.shape != qv.shape:
        raise ValueError("quantised k/v shapes must match")
    if scale_k.shape != (qk.shape[0], qk.shape[2]):
        raise ValueError(f"scale_k shape {scale_k.shape} must be [{qk.shape[0]}, {qk.shape[2]}]")

    def deq(x, s):
        xf = x.astype(np.float32) if mode == "int8" else numerics.e4m3_bits_to_f32(x)
        return xf * s.astype(np.float32)[:, None, :, None]

    return deq(qk, scale_k), deq(qv, scale_v)


def append_tokens_quantized(qk, qv, scale_k, scale_v, page_table, seq_lens, new_k, new_v, page_size, mode):
    """Quantise-on-write append, in place (the semantics of ``fat_append_tokens``
    for 8-bit caches; no FlashAttnTile counterpart -- it extends
    ``paging.py:172-210`` to the format of ``quant.py:84-142``).

    For each sequence b, with pos = seq_lens[b], page = page_table[b, pos //
    page_size], slot = pos % page_size, and per KV head: the new scale is
    ``max(max(absmax_old, absmax_new) / maxval, 1e-8)`` where ``absmax_old =
    max|code| * scale`` over slots ``[0, slot)`` (0 when slot == 0); the old codes
    are requantised from ``code * old_scale`` when the scale changed; the new
    token is quantised with the new scale.  All arithmetic in float32, one
    rounding per operation.  ``new_k``/``new_v`` are float32 (the caller widens
    16-bit inputs exactly).  FP8 codes are uint8 bit patterns."""
    max_val = np.float32(INT8_MAX if mode == "int8" else FP8_MAX)
    min_scale = np.float32(MIN_SCALE)

    def decode(c):
        return c.astype(np.float32) if mode == "int8" else numerics.e4m3_bits_to_f32(c)

    def encode(v):
        v = np.asarray(v, np.float32)
        if mode == "int8":
            return np.clip(np.round(v), -max_val, max_val).astype(np.int8)
        return numerics.f32_to_e4m3_bits(np.clip(v, -max_val, max_val))

    for b in range(seq_lens.shape[0]):
        pos = int(seq_lens[b])
        page = int(page_table[b, pos // page_size])
        slot = pos % page_size
        for codes, scales, new in ((qk, scale_k, new_k), (qv, scale_v, new_v)):
            for h in range(codes.shape[2]):
                x = np.asarray(new[b, h], np.float32)
                amax_new = np.float32(np.abs(x).max())
                s_old = np.float32(scales[page, h])
                amax_old = np.float32(0.0)
                if slot > 0:
                    cmax = np.float32(np.abs(decode(codes[page, :slot, h])).max())
                    amax_old = np.float32(cmax * s_old)
                s_new = np.float32(max(np.float32(max(amax_old, amax_new) / max_val), min_scale))
                if slot > 0 and s_new != s_old:
                    old = (decode(codes[page, :slot, h]) * s_old).astype(np.float32)
                    codes[page, :slot, h] = encode(old / s_new)
                codes[page, slot, h] = encode(x / s_new)
                scales[page, h] = s_new
        seq_lens[b] += 1


def kv_bytes_per_token(num_kv_heads: int, head_dim: int, storage: str = "fp16", page_size: int = 16) -> float:
    """``kv_bytes_per_token`` (``quant.py:194-208``)."""
    elem = {"fp16": 2, "bf16": 2, "fp32": 4, "int8": 1, "fp8": 1}[storage]
    return float(2 * num_kv_heads * head_dim * elem + 2 * num_kv_heads * 4 / page_size)
