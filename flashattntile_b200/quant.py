"""INT8 / FP8-e4m3 KV cache with per-(page, KV-head) fp32 scales.

Same format and API as FlashAttnTile's ``quant.py`` (``quant.py:84-208``):

* scales ``[num_pages, num_kv_heads]`` fp32, ``scale = max(absmax / maxval, 1e-8)``
  with absmax over (token, dim) of each (page, KV head);
* INT8 codes ``clamp(round_half_even(x / scale), -127, 127)``;
* FP8 codes ``(x / scale).clamp(-448, 448)`` cast with round-to-nearest-even;
* dequantisation ``code * scale``.

These are format helpers (tensor ops on whatever device the cache lives on);
the decode kernel consumes the codes and scales directly and never
dequantises the cache in memory.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .paging import PagedKVCache, validate_cache

FP8_DTYPE = getattr(torch, "float8_e4m3fn", None)
FP8_MAX = 448.0
INT8_MAX = 127.0
FP8_MIN_SCALE = 1e-8
INT8_MIN_SCALE = 1e-8


@dataclass
class QuantScales:
    """Per-(page, KV-head) dequantisation scales (``quant.py:36-46``)."""

    k: torch.Tensor
    v: torch.Tensor
    mode: str
    granularity: str = "per_page_per_head"

    def as_dict(self) -> dict:
        return {"k": self.k, "v": self.v, "mode": self.mode, "granularity": self.granularity}


def available_quant_modes() -> list[str]:
    return (["float8_e4m3fn"] if FP8_DTYPE is not None else []) + ["int8"]


def default_quant_mode() -> str:
    """FP8 when the dtype exists and a CUDA device is present, else INT8 (``quant.py:56-65``)."""
    return "float8_e4m3fn" if FP8_DTYPE is not None and torch.cuda.is_available() else "int8"


def _resolve_mode(mode: str) -> tuple[str, torch.dtype, float]:
    if mode == "auto":
        mode = default_quant_mode()
    if mode == "int8":
        return mode, torch.int8, INT8_MAX
    if mode in ("float8_e4m3fn", "fp8"):
        if FP8_DTYPE is None:
            raise RuntimeError("this PyTorch build has no torch.float8_e4m3fn")
        return mode, FP8_DTYPE, FP8_MAX
    raise ValueError(f"unknown quantisation mode {mode!r}; expected 'int8' or 'float8_e4m3fn'")


def quantize_kv_pages(k_cache: torch.Tensor, v_cache: torch.Tensor, mode: str = "auto"):
    """Returns ``(qk, qv, scale_k, scale_v, info)``."""
    if k_cache.shape != v_cache.shape:
        raise ValueError(f"k/v shape mismatch: {tuple(k_cache.shape)} vs {tuple(v_cache.shape)}")
    if k_cache.dim() != 4:
        raise ValueError("cache must be [num_pages, page_size, num_kv_heads, head_dim]")
    if not k_cache.is_floating_point():
        raise ValueError(f"quantize_kv_pages expects a float cache, got {k_cache.dtype}")
    mode, dtype, max_val = _resolve_mode(mode)
    min_scale = INT8_MIN_SCALE if mode == "int8" else FP8_MIN_SCALE

    def one(x: torch.Tensor):
        xf = x.detach().float()
        # Divide by a tensor, not a Python number: torch's CUDA kernels turn a
        # division by a scalar into a multiplication by its reciprocal, which can
        # differ from the correctly rounded quotient in the last bit.  This way
        # the scales (and so the codes) are the same on every device.
        amax = xf.abs().amax(dim=(1, 3))
        scale = (amax / torch.full_like(amax, max_val)).clamp_min(min_scale)
        y = xf / scale[:, None, :, None]
        if mode == "int8":
            codes = y.round().clamp_(-max_val, max_val).to(dtype)
        else:
            codes = y.clamp_(-max_val, max_val).to(dtype)
        return codes, scale

    qk, sk = one(k_cache)
    qv, sv = one(v_cache)
    _, page_size, kv_heads, head_dim = k_cache.shape
    info = {
        "mode": mode,
        "dtype": str(qk.dtype),
        "max_representable": max_val,
        "granularity": "per_page_per_head",
        "page_size": int(page_size),
        "num_kv_heads": int(kv_heads),
        "head_dim": int(head_dim),
        "scale_dtype": str(sk.dtype),
        "scale_min": float(sk.min()),
        "scale_max": float(sk.max()),
        "rounding": "round-to-nearest" if mode == "int8" else "cast-to-fp8",
    }
    return qk, qv, sk, sv, info


def dequantize_kv_pages(qk, qv, scale_k, scale_v, out_dtype: torch.dtype = torch.float16):
    if qk.shape != qv.shape:
        raise ValueError("quantised k/v shapes must match")
    if scale_k.shape != (qk.shape[0], qk.shape[2]):
        raise ValueError(f"scale_k shape {tuple(scale_k.shape)} must be [{qk.shape[0]}, {qk.shape[2]}]")
    k = qk.float() * scale_k.float()[:, None, :, None]
    v = qv.float() * scale_v.float()[:, None, :, None]
    return k.to(out_dtype), v.to(out_dtype)


def quantize_cache(cache: PagedKVCache, mode: str = "auto") -> tuple[PagedKVCache, QuantScales]:
    validate_cache(cache)
    qk, qv, sk, sv, info = quantize_kv_pages(cache.k_cache, cache.v_cache, mode=mode)
    quantized = PagedKVCache(k_cache=qk, v_cache=qv, page_table=cache.page_table, seq_lens=cache.seq_lens,
                             page_size=cache.page_size)
    return quantized, QuantScales(k=sk, v=sv, mode=info["mode"])


def dequantize_cache(cache: PagedKVCache, scales, out_dtype: torch.dtype = torch.float16) -> PagedKVCache:
    sk = scales["k"] if isinstance(scales, dict) else scales.k
    sv = scales["v"] if isinstance(scales, dict) else scales.v
    k, v = dequantize_kv_pages(cache.k_cache, cache.v_cache, sk, sv, out_dtype=out_dtype)
    return PagedKVCache(k_cache=k, v_cache=v, page_table=cache.page_table, seq_lens=cache.seq_lens,
                        page_size=cache.page_size)


def kv_bytes_per_token(num_kv_heads: int, head_dim: int, storage: str = "fp16", page_size: int = 16) -> float:
    """K+V bytes per cached token including the scale overhead (``quant.py:194-208``)."""
    elem = {"fp16": 2, "bf16": 2, "fp32": 4, "int8": 1, "fp8": 1}[storage]
    return float(2 * num_kv_heads * head_dim * elem + 2 * num_kv_heads * 4 / page_size)


def append_tokens_quantized(cache: PagedKVCache, scales, new_k: torch.Tensor, new_v: torch.Tensor) -> None:
    """Append one token per sequence to an INT8 / FP8 cache, quantising on write (one CUDA kernel).

    No reference counterpart: FlashAttnTile appends only to 16-bit caches
    (``paging.py:172-210``) and quantises whole caches offline
    (``quant.py:84-142``).  This keeps that offline format exact on the fly:
    the page receiving a token gets the scale ``quantize_kv_pages`` would give
    the sequence's tokens on it (earlier ones dequantised as ``code * scale``,
    plus the new one), earlier codes are requantised when the scale changed,
    and the new token is quantised with it.  ``new_k``/``new_v`` are
    ``[batch, num_kv_heads, head_dim]`` fp16 / bf16 / fp32; ``scales`` is a
    ``QuantScales`` or a dict with ``k``/``v`` (updated in place, like the codes
    and ``cache.seq_lens``)."""
    from .kernels.append import launch_append
    from .paging import _assert, _check_append_values, validate_metadata
    from . import _config

    validate_metadata(cache)
    k_scale = scales["k"] if isinstance(scales, dict) else scales.k
    v_scale = scales["v"] if isinstance(scales, dict) else scales.v
    quant_dtypes = (torch.int8,) + ((FP8_DTYPE,) if FP8_DTYPE is not None else ())
    _assert(cache.k_cache.dtype in quant_dtypes, f"expected an int8/float8 cache, got {cache.k_cache.dtype}")
    shape = (cache.batch_size, cache.num_kv_heads, cache.head_dim)
    _assert(new_k.shape == shape, f"new_k must be [{shape[0]}, {shape[1]}, {shape[2]}], got {tuple(new_k.shape)}")
    _assert(new_v.shape == new_k.shape, f"new_v shape {tuple(new_v.shape)} != new_k shape {tuple(new_k.shape)}")
    _assert(new_k.dtype in (torch.float16, torch.bfloat16, torch.float32) and new_v.dtype == new_k.dtype,
            f"new_k/new_v must share a float dtype (fp16, bf16, fp32), got {new_k.dtype}/{new_v.dtype}")
    expected = (cache.num_pages, cache.num_kv_heads)
    _assert(tuple(k_scale.shape) == expected and tuple(v_scale.shape) == expected,
            f"scales must have shape {expected}, got {tuple(k_scale.shape)}")
    if cache.batch_size == 0:
        return
    if _config.validate_values():
        _check_append_values(cache)
    launch_append(cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, new_k, new_v, cache.page_size,
                  k_scale=k_scale, v_scale=v_scale)
