"""Launcher of the bit-exact page-table gather kernel (``fat_gather_paged``)."""

from __future__ import annotations

import torch

from .. import _lib


def _check_pages(page_table, seq_lens, page_size, num_pages):
    """Reference message for a bad page id (``flashattn_tile/paging.py:248-251``)."""
    if seq_lens.numel() == 0:
        return
    need = torch.div(seq_lens.long() + page_size - 1, page_size, rounding_mode="floor")
    cols = torch.arange(page_table.shape[1], device=page_table.device)
    used = cols[None, :] < need[:, None].to(page_table.device)
    bad = used & ((page_table < 0) | (page_table >= num_pages))
    rows = bad.any(dim=1).nonzero()
    if rows.numel():
        raise AssertionError(f"sequence {int(rows[0, 0])} page id outside [0, {num_pages})")


def gather_paged_cuda(k_cache, v_cache, page_table, seq_lens, page_size):
    if not (k_cache.is_cuda and v_cache.is_cuda and page_table.is_cuda and seq_lens.is_cuda):
        raise RuntimeError("gather_paged: flashattntile_b200 runs on CUDA tensors only (no CPU path)")
    batch = int(seq_lens.shape[0])
    max_len = int(seq_lens.max()) if batch else 0
    shape = (batch, max_len, k_cache.shape[2], k_cache.shape[3])
    out_k = torch.empty(shape, dtype=k_cache.dtype, device=k_cache.device)
    out_v = torch.empty(shape, dtype=v_cache.dtype, device=v_cache.device)
    if max_len == 0:
        return out_k, out_v
    capacity = int(page_table.shape[1]) * page_size
    if max_len > capacity:
        raise AssertionError(f"seq_len {max_len} exceeds page-table capacity {capacity}")
    _check_pages(page_table, seq_lens, page_size, int(k_cache.shape[0]))
    if k_cache.stride() != v_cache.stride() or k_cache.stride(3) != 1:
        raise ValueError("gather_paged: k_cache and v_cache need equal strides and a contiguous last dim")
    eb = k_cache.element_size()
    err = _lib.error_word(k_cache.device)
    lib = _lib.load()
    status = lib.fat_gather_paged(
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0) * eb, k_cache.stride(1) * eb,
        k_cache.stride(2) * eb, k_cache.shape[0], page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
        seq_lens.data_ptr(), out_k.data_ptr(), out_v.data_ptr(), max_len, batch, k_cache.shape[2], page_size,
        k_cache.shape[3] * eb, err.data_ptr(), _lib.stream_handle(k_cache.device))
    _lib.check(status, "gather_paged")
    return out_k, out_v


__all__ = ["gather_paged_cuda"]
