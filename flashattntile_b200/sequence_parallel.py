"""Long-context decode split across GPUs by page range, merged by log-sum-exp.

FlashAttnTile splits one sequence's pages only inside a GPU (split-K over
page ranges, then an LSE reduce: ``kernels/decode.py:8-16, 223-356``).  Here
the same split runs across GPUs, one process per GPU:

1. Rank ``r`` of ``R`` owns the contiguous logical page range
   ``page_range(max_pages, R, r)`` of every sequence (the same columns of the
   page table for every sequence), in its own page pool.  Its local
   ``seq_lens`` count only the tokens of that range (``local_lengths``).
2. ``decode_partial`` runs the paged-decode kernel over the local pages and
   writes fp32 partials into one packed buffer: the normalised output
   ``o [B, H, D]`` followed by the base-2 log-sum-exp ``lse [B, H]`` of the
   scaled scores (``-inf`` where the rank holds no token of a sequence).
3. ``exchange_partials`` gathers the packed buffers of all ranks with one
   ``all_gather_into_tensor`` (NCCL over NVLink on a GPU node), in rank order.
4. ``merge_partials`` combines them with the LSE-merge kernel:
   ``out = sum_r o_r 2^(lse_r - M) / sum_r 2^(lse_r - M)``.

Every rank ends up with the full ``[B, H, D]`` output.  The exchange moves
``B * H * (D + 1) * 4`` bytes per rank; the pages themselves never leave their
GPU.  ``shard_view`` builds rank ``r``'s view of a cache that holds all pages
in one pool (a single-GPU emulation of the ranks, and the way tests check the
split against the unsplit decode).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _config, _lib
from .kernels.decode import _require_cuda, launch_decode
from .paging import PagedKVCache, validate_cache, validate_metadata


def page_range(max_pages: int, world_size: int, rank: int) -> tuple[int, int]:
    """Logical pages ``[p0, p1)`` of every sequence that rank ``rank`` owns.

    Contiguous, equal-sized ranges (the last one may be shorter or empty)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world_size {world_size}")
    if max_pages < 0:
        raise ValueError(f"max_pages must be non-negative, got {max_pages}")
    per = math.ceil(max_pages / world_size) if max_pages else 0
    p0 = min(rank * per, max_pages)
    return p0, min(p0 + per, max_pages)


def local_lengths(seq_lens: torch.Tensor, page_size: int, p0: int, p1: int) -> torch.Tensor:
    """Tokens of each sequence that fall in logical pages ``[p0, p1)`` (int32, same device)."""
    start = p0 * page_size
    return (seq_lens.to(torch.int64) - start).clamp(0, (p1 - p0) * page_size).to(torch.int32)


def shard_view(cache: PagedKVCache, rank: int, world_size: int) -> PagedKVCache:
    """Rank ``rank``'s share of a cache whose pool holds every page.

    Shares the K/V pools; the page table is a column slice (no copy).  A rank
    with no pages gets one table column and zero lengths."""
    p0, p1 = page_range(cache.max_pages_per_seq, world_size, rank)
    if p1 == p0:
        table = cache.page_table[:, :1]
        lens = torch.zeros_like(cache.seq_lens)
    else:
        table = cache.page_table[:, p0:p1]
        lens = local_lengths(cache.seq_lens, cache.page_size, p0, p1)
    return PagedKVCache(cache.k_cache, cache.v_cache, table, lens, cache.page_size)


def packed_size(batch: int, num_heads: int, head_dim: int) -> int:
    """fp32 elements of one rank's packed partial: ``o [B, H, D]`` then ``lse [B, H]``."""
    return batch * num_heads * (head_dim + 1)


def unpack(packed: torch.Tensor, batch: int, num_heads: int, head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Views ``(o [B, H, D], lse [B, H])`` of a packed partial."""
    n = batch * num_heads * head_dim
    return packed[:n].view(batch, num_heads, head_dim), packed[n:n + batch * num_heads].view(batch, num_heads)


def decode_partial(q: torch.Tensor, cache: PagedKVCache, softmax_scale: float | None = None, scales=None,
                   packed: torch.Tensor | None = None) -> torch.Tensor:
    """Decode ``q [B, H, D]`` against this rank's pages; return the packed fp32 partial.

    ``scales``: per-(page, KV-head) ``k`` / ``v`` scales for an INT8 / FP8 cache
    (a dict or an object with ``.k`` / ``.v``), as ``paged_decode_attention_fp8``
    takes them.  Sequences with no local token get ``o = 0``, ``lse = -inf``."""
    if not isinstance(cache, PagedKVCache):
        raise TypeError("cache must be a PagedKVCache")
    if _config.validate_values():
        validate_cache(cache)
    else:
        validate_metadata(cache)
    if q.dim() != 3 or q.shape[0] != cache.batch_size or q.shape[2] != cache.head_dim:
        raise ValueError(f"q {tuple(q.shape)} does not match the cache (batch {cache.batch_size}, "
                         f"head_dim {cache.head_dim})")
    _require_cuda(q)
    batch, heads, dim = q.shape
    if packed is None:
        packed = torch.empty(packed_size(batch, heads, dim), dtype=torch.float32, device=q.device)
    elif packed.dtype != torch.float32 or packed.numel() != packed_size(batch, heads, dim) or not packed.is_contiguous():
        raise ValueError("packed must be a contiguous float32 tensor of packed_size(B, H, D) elements")
    o, lse = unpack(packed, batch, heads, dim)
    scale = float(softmax_scale) if softmax_scale is not None else dim ** -0.5
    k_scale = v_scale = None
    if scales is not None:
        k_scale = scales["k"] if isinstance(scales, dict) else scales.k
        v_scale = scales["v"] if isinstance(scales, dict) else scales.v
    launch_decode(q, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, cache.page_size, scale,
                  k_scale=k_scale, v_scale=v_scale, out=o, out_dtype=torch.float32, lse=lse)
    return packed


def exchange_partials(packed: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather every rank's packed partial into ``[world_size, n]`` (rank order)."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world, packed.numel()), dtype=packed.dtype, device=packed.device)
    # A flat output: gloo checks each rank's slice against the input's shape.
    dist.all_gather_into_tensor(out.view(-1), packed.view(-1), group=group)
    return out


def merge_partials(parts: torch.Tensor, batch: int, num_heads: int, head_dim: int,
                   out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None,
                   lse_out: torch.Tensor | None = None) -> torch.Tensor:
    """Combine packed partials ``[R, packed_size]`` into ``[B, H, D]`` of ``out_dtype`` (CUDA kernel)."""
    _require_cuda(parts)
    n = packed_size(batch, num_heads, head_dim)
    if parts.dim() != 2 or parts.shape[1] != n or parts.dtype != torch.float32 or not parts.is_contiguous():
        raise ValueError(f"parts must be a contiguous float32 [R, {n}] tensor, got {tuple(parts.shape)} {parts.dtype}")
    if out is None:
        out = torch.empty((batch, num_heads, head_dim), dtype=out_dtype, device=parts.device)
    elif out.dtype != out_dtype or tuple(out.shape) != (batch, num_heads, head_dim) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [B, H, D] tensor of out_dtype")
    if lse_out is not None and (lse_out.dtype != torch.float32 or lse_out.numel() != batch * num_heads
                                or not lse_out.is_contiguous()):
        raise ValueError("lse_out must be a contiguous float32 tensor of B * H elements")
    if out_dtype not in _lib.DTYPE_CODE or out_dtype in (torch.int8,):
        raise ValueError(f"unsupported out dtype {out_dtype}")
    lib = _lib.load()
    dev = parts.device
    lse_ptr = parts.data_ptr() + batch * num_heads * head_dim * parts.element_size()
    status = lib.fat_lse_merge(parts.data_ptr(), n, lse_ptr, n, parts.shape[0], batch * num_heads, head_dim,
                               out.data_ptr(), _lib.DTYPE_CODE[out_dtype], _lib.ptr(lse_out),
                               torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(status, "lse_merge")
    return out


def sequence_parallel_decode(q: torch.Tensor, local_cache: PagedKVCache, softmax_scale: float | None = None,
                             scales=None, group=None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Decode one step of long sequences whose pages are split across the ranks of ``group``.

    ``q [B, H, D]`` is the same on every rank; ``local_cache`` holds this rank's
    page range of every sequence (``page_range`` / ``local_lengths``).  Returns
    the full output ``[B, H, D]`` (``out_dtype``, default q's dtype) on every rank."""
    batch, heads, dim = q.shape
    packed = decode_partial(q, local_cache, softmax_scale, scales)
    parts = exchange_partials(packed, group)
    return merge_partials(parts, batch, heads, dim, out_dtype or q.dtype)
