"""Launcher of the device-side KV append (``fat_append_tokens``).

One token per sequence goes to ``page_table[b, seq_lens[b] // page_size]``,
slot ``seq_lens[b] % page_size``; ``seq_lens`` is then incremented -- all in one
kernel, without host synchronisation.  For INT8 / FP8 caches the token is
quantised on write and the page's per-(page, KV-head) scale is maintained
(see ``flashattntile_b200.quant.append_tokens_quantized``).
"""

from __future__ import annotations

import torch

from .. import _lib

_QUANT = (torch.int8,) + ((torch.float8_e4m3fn,) if hasattr(torch, "float8_e4m3fn") else ())


def launch_append(k_cache, v_cache, page_table, seq_lens, new_k, new_v, page_size, k_scale=None, v_scale=None):
    for t in (k_cache, v_cache, page_table, seq_lens, new_k, new_v):
        if not t.is_cuda:
            raise RuntimeError("append_tokens: flashattntile_b200 runs on CUDA tensors only (no CPU path)")
    if k_cache.stride() != v_cache.stride() or k_cache.stride(3) != 1:
        raise ValueError("append_tokens: k_cache and v_cache need equal strides and a contiguous last dim")
    if new_k.stride() != new_v.stride() or new_k.stride(2) != 1:
        new_k, new_v = new_k.contiguous(), new_v.contiguous()
    if page_table.stride(1) != 1:
        page_table = page_table.contiguous()
    if not seq_lens.is_contiguous():
        raise ValueError("append_tokens: seq_lens must be contiguous (it is updated in place)")
    scale_stride = 0
    if k_cache.dtype in _QUANT:
        if k_scale is None or v_scale is None:
            raise ValueError("append_tokens: an int8/fp8 cache needs k and v scales")
        if k_scale.dtype != torch.float32 or v_scale.stride() != k_scale.stride() or k_scale.stride(1) != 1:
            raise ValueError("append_tokens: scales must be float32 [num_pages, num_kv_heads] with equal strides")
        scale_stride = k_scale.stride(0)
    dev = k_cache.device
    lib = _lib.load()
    err = _lib.error_word(dev)
    status = lib.fat_append_tokens(
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        k_cache.shape[0], page_table.data_ptr(), page_table.stride(0), page_table.shape[1], seq_lens.data_ptr(),
        new_k.data_ptr(), new_v.data_ptr(), new_k.stride(0), new_k.stride(1), _lib.ptr(k_scale), _lib.ptr(v_scale),
        scale_stride, seq_lens.shape[0], k_cache.shape[2], k_cache.shape[3], int(page_size),
        _lib.DTYPE_CODE[k_cache.dtype], _lib.DTYPE_CODE[new_k.dtype], err.data_ptr(), _lib.stream_handle(dev))
    _lib.check(status, "append_tokens")


__all__ = ["launch_append"]
