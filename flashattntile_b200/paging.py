"""Paged KV-cache contract (NHD layout), same as FlashAttnTile's ``paging.py``.

Layout (``flashattn_tile/paging.py:3-19``)
------------------------------------------
``k_cache`` / ``v_cache``
    ``[num_pages, page_size, num_kv_heads, head_dim]``: page ``p`` holds
    ``page_size`` consecutive tokens for every KV head.
``page_table``
    ``int32 [batch, max_pages_per_seq]``; entry ``[b, i]`` is the physical page
    of logical block ``i`` of sequence ``b``.  Entries past a sequence's length
    are never read.
``seq_lens``
    ``int32 [batch]``; token ``t`` of sequence ``b`` lives in page
    ``page_table[b, t // page_size]`` at slot ``t % page_size``.

``validate_cache`` keeps the reference's checks and ``AssertionError``
messages (``paging.py:84-130``).  ``gather_paged`` runs a CUDA copy kernel
(bit-exact, zero past each length) instead of the reference's per-sequence
Python loop.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _config, _lib


@dataclass
class PagedKVCache:
    """Paged K/V cache plus its page table (``flashattn_tile/paging.py:30-76``)."""

    k_cache: torch.Tensor
    v_cache: torch.Tensor
    page_table: torch.Tensor
    seq_lens: torch.Tensor
    page_size: int

    @property
    def batch_size(self) -> int:
        return int(self.seq_lens.shape[0])

    @property
    def num_pages(self) -> int:
        return int(self.k_cache.shape[0])

    @property
    def num_kv_heads(self) -> int:
        return int(self.k_cache.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.k_cache.shape[3])

    @property
    def max_pages_per_seq(self) -> int:
        return int(self.page_table.shape[1])

    @property
    def capacity(self) -> int:
        return self.max_pages_per_seq * self.page_size


def _assert(condition: bool, message: str) -> None:
    if not condition:
        raise AssertionError(message)


def validate_metadata(cache: PagedKVCache) -> None:
    """Shape / dtype / device checks only: never reads device memory.  Messages
    are built only when a check fails (this runs on every call)."""
    if not isinstance(cache, PagedKVCache):
        raise AssertionError("cache must be a PagedKVCache")
    k, v = cache.k_cache, cache.v_cache
    kshape = k.shape
    if len(kshape) != 4:
        raise AssertionError(f"k_cache must be 4-D [pages, page_size, kv_heads, dim], got {tuple(kshape)}")
    if kshape != v.shape:
        raise AssertionError(f"k_cache {tuple(kshape)} and v_cache {tuple(v.shape)} must match")
    if k.dtype != v.dtype:
        raise AssertionError(f"k_cache dtype {k.dtype} != v_cache dtype {v.dtype}")
    if k.device != v.device:
        raise AssertionError("k_cache and v_cache must live on the same device")
    if cache.page_size <= 0:
        raise AssertionError("page_size must be positive")
    if kshape[1] != cache.page_size:
        raise AssertionError(f"k_cache page dim {kshape[1]} != page_size {cache.page_size}")
    table, lens = cache.page_table, cache.seq_lens
    if table.dtype != torch.int32:
        raise AssertionError(f"page_table must be int32, got {table.dtype}")
    if lens.dtype != torch.int32:
        raise AssertionError(f"seq_lens must be int32, got {lens.dtype}")
    if table.dim() != 2:
        raise AssertionError("page_table must be [batch, max_pages_per_seq]")
    if lens.dim() != 1:
        raise AssertionError("seq_lens must be [batch]")
    if table.shape[0] != lens.shape[0]:
        raise AssertionError("page_table and seq_lens batch dimensions disagree")
    if table.device != lens.device:
        raise AssertionError("page_table and seq_lens must live on the same device")


def cache_value_stats(cache: PagedKVCache) -> tuple[int, int, int, int]:
    """``(min seq_len, max seq_len, min used page id, max used page id)`` in one
    device->host transfer.  "Used" entries are those a sequence's length reaches
    (the first ``ceil(max_len / page_size)`` columns, as the reference checks);
    with no used entry the page bounds are reported as ``(0, -1)``."""
    lens = cache.seq_lens
    table = cache.page_table
    if lens.is_cuda and table.is_cuda and lens.device == table.device:
        # One small kernel and one 16-byte read-back instead of a dozen torch reductions.
        from . import _lib

        lo, hi, umin, umax = _lib.cache_value_stats(lens, table, cache.page_size)
        return int(lo), int(hi), int(umin), int(umax)
    need = torch.div(lens.max().to(torch.int64) + cache.page_size - 1, cache.page_size, rounding_mode="floor")
    cols = torch.arange(table.shape[1], device=table.device)
    used = (cols < need.to(table.device))[None, :].expand_as(table)
    big = torch.iinfo(torch.int32).max
    pmin = torch.where(used, table, torch.full_like(table, big)).amin()
    pmax = torch.where(used, table, torch.full_like(table, -1)).amax()
    lo, hi = torch.aminmax(lens)
    stats = torch.stack([lo.to(torch.int64), hi.to(torch.int64), pmin.to(torch.int64).to(lo.device),
                         pmax.to(torch.int64).to(lo.device)]).tolist()
    if stats[2] == big:
        stats[2], stats[3] = 0, -1
    return int(stats[0]), int(stats[1]), int(stats[2]), int(stats[3])


def validate_cache(cache: PagedKVCache, *, check_pages: bool = True) -> tuple[int, int] | None:
    """All checks of ``flashattn_tile/paging.py:84-130``, including the value
    checks on ``seq_lens`` / ``page_table`` -- read back in a single device->host
    transfer.  Returns ``(min seq_len, max seq_len)`` (None for an empty batch)."""
    validate_metadata(cache)
    return validate_cache_values(cache, check_pages=check_pages)


def validate_cache_values(cache: PagedKVCache, *, check_pages: bool = True) -> tuple[int, int] | None:
    """The value half of :func:`validate_cache` (metadata already checked)."""
    if cache.seq_lens.numel() == 0:
        return None
    return check_value_stats(cache, cache_value_stats(cache), check_pages=check_pages)


def check_value_stats(cache: PagedKVCache, stats, *, check_pages: bool = True) -> tuple[int, int]:
    """The assertions of the value checks on ``cache_value_stats`` numbers."""
    return check_value_numbers(stats, cache.capacity, cache.num_pages, check_pages=check_pages)


def check_value_numbers(stats, capacity: int, num_pages: int, *, check_pages: bool = True) -> tuple[int, int]:
    """:func:`check_value_stats` on plain numbers (the cache's capacity and page count)."""
    lo, max_len, umin, umax = (int(x) for x in stats)
    _assert(lo >= 0, "seq_lens must be non-negative")
    _assert(max_len <= capacity, f"seq_len {max_len} exceeds page-table capacity {capacity}")
    if check_pages and max_len > 0:
        _assert(umin >= 0, "page_table contains a negative page id")
        _assert(umax < num_pages, f"page_table references page {umax} but cache has {num_pages} pages")
    return lo, max_len


def allocate(batch: int, max_seq_len: int, num_kv_heads: int, head_dim: int, page_size: int,
             dtype: torch.dtype = torch.float16, device: torch.device | str = "cuda") -> PagedKVCache:
    """Zeroed cache with a contiguous page mapping (``paging.py:133-169``)."""
    _assert(batch > 0, "batch must be positive")
    _assert(max_seq_len > 0, "max_seq_len must be positive")
    _assert(num_kv_heads > 0 and head_dim > 0, "num_kv_heads and head_dim must be positive")
    _assert(page_size > 0, "page_size must be positive")
    allowed = {torch.float16, torch.bfloat16, torch.float32, torch.int8}
    if hasattr(torch, "float8_e4m3fn"):
        allowed.add(torch.float8_e4m3fn)
    _assert(dtype in allowed, f"unsupported cache dtype {dtype}")
    pages_per_seq = math.ceil(max_seq_len / page_size)
    num_pages = batch * pages_per_seq
    k_cache = torch.zeros((num_pages, page_size, num_kv_heads, head_dim), dtype=dtype, device=device)
    cache = PagedKVCache(
        k_cache=k_cache,
        v_cache=torch.zeros_like(k_cache),
        page_table=torch.arange(num_pages, dtype=torch.int32, device=device).reshape(batch, pages_per_seq),
        seq_lens=torch.zeros(batch, dtype=torch.int32, device=device),
        page_size=page_size,
    )
    validate_cache(cache)
    return cache


def _check_append_values(cache: PagedKVCache) -> None:
    """The reference's value checks of an append (``paging.py:192-203``), read back in one transfer."""
    positions = cache.seq_lens.long()
    page_idx = torch.div(positions, cache.page_size, rounding_mode="floor").clamp_max(cache.max_pages_per_seq - 1)
    rows = torch.arange(cache.batch_size, device=cache.page_table.device)
    phys = cache.page_table[rows, page_idx.to(cache.page_table.device)].long()
    pmin, pmax = torch.aminmax(phys)
    stats = torch.stack([positions.max().to(pmin.device), pmin, pmax]).tolist()
    _assert(int(stats[0]) < cache.capacity, f"append would exceed page-table capacity {cache.capacity}")
    _assert(int(stats[1]) >= 0 and int(stats[2]) < cache.num_pages,
            f"page_table maps to a page outside [0, {cache.num_pages})")


def append_tokens(cache: PagedKVCache, new_k: torch.Tensor, new_v: torch.Tensor) -> None:
    """Append one token per sequence in place (``paging.py:172-210``), in one CUDA kernel.

    Checks and messages are the reference's; the value checks (capacity, page
    ids) read ``seq_lens``/``page_table`` back in one transfer when value
    checks are on, and are otherwise left to the kernel, which skips a bad
    sequence and records ``FAT_DEVERR_BAD_PAGE`` (``device_error()``)."""
    validate_metadata(cache)
    shape = (cache.batch_size, cache.num_kv_heads, cache.head_dim)
    _assert(new_k.shape == shape, f"new_k must be [{shape[0]}, {shape[1]}, {shape[2]}], got {tuple(new_k.shape)}")
    _assert(new_v.shape == new_k.shape, f"new_v shape {tuple(new_v.shape)} != new_k shape {tuple(new_k.shape)}")
    _assert(new_k.dtype == cache.k_cache.dtype, f"new_k dtype {new_k.dtype} != cache dtype {cache.k_cache.dtype}")
    _assert(new_v.dtype == cache.k_cache.dtype, f"new_v dtype {new_v.dtype} != cache dtype {cache.k_cache.dtype}")
    _assert(new_k.device == cache.k_cache.device, "new_k must be on the cache device")
    _assert(new_v.device == cache.k_cache.device, "new_v must be on the cache device")
    if cache.batch_size == 0:
        return
    if _config.validate_values():
        _check_append_values(cache)
    from .kernels.append import launch_append

    launch_append(cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, new_k, new_v, cache.page_size)


def gather_paged(k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor, seq_lens: torch.Tensor,
                 page_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Padded contiguous ``[batch, max_len, kv_heads, dim]`` copies, zero past each
    length (``paging.py:213-256``), produced by the CUDA gather kernel."""
    _assert(k_cache.shape == v_cache.shape, "k_cache and v_cache shapes must match")
    _assert(page_table.dtype == torch.int32, "page_table must be int32")
    _assert(seq_lens.dtype == torch.int32, "seq_lens must be int32")
    _assert(page_table.dim() == 2 and seq_lens.dim() == 1, "expected page_table [B, P] and seq_lens [B]")
    _assert(page_table.shape[0] == seq_lens.shape[0], "page_table / seq_lens batch mismatch")
    _assert(k_cache.shape[1] == page_size, "k_cache page dim != page_size")
    from .kernels.gather import gather_paged_cuda

    return gather_paged_cuda(k_cache, v_cache, page_table, seq_lens, page_size)


def gather_contiguous(cache: PagedKVCache) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather ``cache`` into padded contiguous K/V (``paging.py:259-262``)."""
    validate_cache(cache)
    return gather_paged(cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, cache.page_size)
