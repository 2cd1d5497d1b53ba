"""Page-table contract, restated in numpy (oracle only).

Layout (``flashattn_tile/paging.py:3-19``): K/V ``[num_pages, page_size,
num_kv_heads, head_dim]``; ``page_table`` int32 ``[batch, max_pages]``;
``seq_lens`` int32 ``[batch]``; logical token ``t`` of sequence ``b`` lives in
page ``page_table[b, t // page_size]`` at slot ``t % page_size``.

The functions operate on raw storage arrays (any element type -- the gather
is a byte copy) and raise ``AssertionError`` with the reference's messages.
"""

from __future__ import annotations

import math

import numpy as np


def _assert(cond: bool, message: str) -> None:
    if not cond:
        raise AssertionError(message)


def validate(k_cache, v_cache, page_table, seq_lens, page_size, check_pages=True) -> None:
    """``validate_cache`` (``flashattn_tile/paging.py:84-130``) on numpy arrays."""
    _assert(k_cache.ndim == 4, f"k_cache must be 4-D [pages, page_size, kv_heads, dim], got {k_cache.shape}")
    _assert(k_cache.shape == v_cache.shape, f"k_cache {k_cache.shape} and v_cache {v_cache.shape} must match")
    _assert(k_cache.dtype == v_cache.dtype, f"k_cache dtype {k_cache.dtype} != v_cache dtype {v_cache.dtype}")
    _assert(page_size > 0, "page_size must be positive")
    _assert(k_cache.shape[1] == page_size, f"k_cache page dim {k_cache.shape[1]} != page_size {page_size}")
    _assert(page_table.dtype == np.int32, f"page_table must be int32, got {page_table.dtype}")
    _assert(seq_lens.dtype == np.int32, f"seq_lens must be int32, got {seq_lens.dtype}")
    _assert(page_table.ndim == 2, "page_table must be [batch, max_pages_per_seq]")
    _assert(seq_lens.ndim == 1, "seq_lens must be [batch]")
    _assert(page_table.shape[0] == seq_lens.shape[0], "page_table and seq_lens batch dimensions disagree")
    _assert(int(seq_lens.min()) >= 0 if seq_lens.size else True, "seq_lens must be non-negative")
    capacity = page_table.shape[1] * page_size
    max_len = int(seq_lens.max()) if seq_lens.size else 0
    _assert(max_len <= capacity, f"seq_len {max_len} exceeds page-table capacity {capacity}")
    if check_pages and max_len > 0:
        used = page_table[:, : math.ceil(max_len / page_size)].astype(np.int64)
        _assert(int(used.min()) >= 0, "page_table contains a negative page id")
        _assert(
            int(used.max()) < k_cache.shape[0],
            f"page_table references page {int(used.max())} but cache has {k_cache.shape[0]} pages",
        )


def gather_paged(k_cache, v_cache, page_table, seq_lens, page_size):
    """Padded contiguous ``[B, max_len, Hkv, D]`` copy, zero past each length.

    Follows ``flashattn_tile/paging.py:213-256``: bit-exact copy of the
    addressed rows, including the per-sequence page-id bounds message.
    """
    _assert(k_cache.shape == v_cache.shape, "k_cache and v_cache shapes must match")
    _assert(page_table.dtype == np.int32, "page_table must be int32")
    _assert(seq_lens.dtype == np.int32, "seq_lens must be int32")
    _assert(page_table.ndim == 2 and seq_lens.ndim == 1, "expected page_table [B, P] and seq_lens [B]")
    _assert(page_table.shape[0] == seq_lens.shape[0], "page_table / seq_lens batch mismatch")
    _assert(k_cache.shape[1] == page_size, "k_cache page dim != page_size")
    batch = seq_lens.shape[0]
    max_len = int(seq_lens.max()) if batch else 0
    shape = (batch, max_len, k_cache.shape[2], k_cache.shape[3])
    out_k = np.zeros(shape, dtype=k_cache.dtype)
    out_v = np.zeros(shape, dtype=v_cache.dtype)
    if max_len == 0:
        return out_k, out_v
    capacity = page_table.shape[1] * page_size
    _assert(max_len <= capacity, f"seq_len {max_len} exceeds page-table capacity {capacity}")
    for b in range(batch):
        length = int(seq_lens[b])
        if length == 0:
            continue
        ids = page_table[b, : math.ceil(length / page_size)].astype(np.int64)
        _assert(
            int(ids.min()) >= 0 and int(ids.max()) < k_cache.shape[0],
            f"sequence {b} page id outside [0, {k_cache.shape[0]})",
        )
        out_k[b, :length] = k_cache[ids].reshape(-1, *k_cache.shape[2:])[:length]
        out_v[b, :length] = v_cache[ids].reshape(-1, *v_cache.shape[2:])[:length]
    return out_k, out_v


def sequence_kv(k_cache, v_cache, page_table, length, b, page_size):
    """K/V rows ``[length, Hkv, D]`` of sequence ``b`` (no padding)."""
    ids = page_table[b, : math.ceil(length / page_size)].astype(np.int64)
    k = k_cache[ids].reshape(-1, *k_cache.shape[2:])[:length]
    v = v_cache[ids].reshape(-1, *v_cache.shape[2:])[:length]
    return k, v


def append_tokens(k_cache, v_cache, page_table, seq_lens, page_size, new_k, new_v) -> None:
    """One-token append (``flashattn_tile/paging.py:172-210``), in place."""
    batch, kvh, dim = seq_lens.shape[0], k_cache.shape[2], k_cache.shape[3]
    _assert(new_k.shape == (batch, kvh, dim), f"new_k must be [{batch}, {kvh}, {dim}], got {new_k.shape}")
    _assert(new_v.shape == new_k.shape, f"new_v shape {new_v.shape} != new_k shape {new_k.shape}")
    _assert(new_k.dtype == k_cache.dtype, f"new_k dtype {new_k.dtype} != cache dtype {k_cache.dtype}")
    capacity = page_table.shape[1] * page_size
    pos = seq_lens.astype(np.int64)
    _assert(int(pos.max()) < capacity, f"append would exceed page-table capacity {capacity}")
    page_idx = pos // page_size
    phys = page_table[np.arange(batch), page_idx].astype(np.int64)
    _assert(
        int(phys.min()) >= 0 and int(phys.max()) < k_cache.shape[0],
        f"page_table maps to a page outside [0, {k_cache.shape[0]})",
    )
    slots = pos % page_size
    k_cache[phys, slots] = new_k
    v_cache[phys, slots] = new_v
    seq_lens += 1
