"""vLLM-shaped attention backend (FlashAttnTile's ``flashattn_tile/backend.py``).

``get_kv_cache_shape`` returns ``(2, blocks, block_size, kv_heads, head_dim)``
(``backend.py:56-60``); ``forward`` routes prefill metadata to
``prefill_attention`` (always causal, ``backend.py:149-173``) and everything
else to ``paged_decode_attention`` (``backend.py:175``), squeezing a
``[B, 1, H, D]`` decode query (``backend.py:142-143``).  ``kv_cache`` may also
be one ``(2, blocks, block_size, kv_heads, head_dim)`` tensor, as a serving
engine holds it; its K/V halves are then used zero-copy.

Prefill without packed ``k``/``v`` in the metadata (the reference raises,
``backend.py:158-162``) reads K/V from the paged cache instead: chunked prefill
and prefix caching, where the new tokens' K/V are already in the cache and
``seq_lens`` counts every cached token of each sequence.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .kernels.decode import paged_decode_attention
from .kernels.prefill import prefill_attention, prefill_paged_attention
from .paging import PagedKVCache, allocate

KV_CACHE_NDIM = 4


@dataclass
class AttentionMetadata:
    """Per-step metadata passed to :meth:`FlashAttnTileBackend.forward` (``backend.py:37-53``)."""

    page_table: torch.Tensor | None = None
    seq_lens: torch.Tensor | None = None
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    is_prefill: bool = False
    max_seqlen_q: int | None = None
    max_seqlen_k: int | None = None
    k: torch.Tensor | None = None
    v: torch.Tensor | None = None
    softmax_scale: float | None = None


def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int):
    return (2, int(num_blocks), int(block_size), int(num_kv_heads), int(head_dim))


class FlashAttnTileBackend:
    """Routes prefill and decode to the sm_100a kernels (``backend.py:63-175``)."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                 dtype: torch.dtype | None = None, device: torch.device | str | None = None) -> None:
        if num_heads % num_kv_heads != 0:
            raise ValueError(f"num_heads {num_heads} must be divisible by num_kv_heads {num_kv_heads}")
        if page_size <= 0:
            raise ValueError("page_size must be positive")
        self.num_heads = int(num_heads)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        self.dtype = dtype
        self.device = device

    def get_name(self) -> str:
        return "flashattn_tile"

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int):
        return get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_dim)

    @staticmethod
    def get_kv_cache_shape_per_tensor(num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int):
        return (int(num_blocks), int(block_size), int(num_kv_heads), int(head_dim))

    def allocate_kv_cache(self, batch: int, max_seq_len: int, dtype: torch.dtype = torch.float16,
                          device: torch.device | str = "cuda") -> PagedKVCache:
        return allocate(batch=batch, max_seq_len=max_seq_len, num_kv_heads=self.num_kv_heads,
                        head_dim=self.head_dim, page_size=self.page_size, dtype=dtype, device=device)

    def _resolve_cache(self, kv_cache, attn_metadata: AttentionMetadata) -> PagedKVCache:
        if isinstance(kv_cache, torch.Tensor):
            if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
                raise ValueError("a tensor kv_cache must be (2, blocks, block_size, kv_heads, head_dim)")
            if attn_metadata.page_table is None or attn_metadata.seq_lens is None:
                raise ValueError("a tensor kv_cache needs attn_metadata.page_table and seq_lens")
            return PagedKVCache(k_cache=kv_cache[0], v_cache=kv_cache[1], page_table=attn_metadata.page_table,
                                seq_lens=attn_metadata.seq_lens, page_size=int(kv_cache.shape[2]))
        if not isinstance(kv_cache, PagedKVCache):
            raise TypeError("kv_cache must be a PagedKVCache")
        if attn_metadata.page_table is None and attn_metadata.seq_lens is None:
            return kv_cache
        return PagedKVCache(
            k_cache=kv_cache.k_cache,
            v_cache=kv_cache.v_cache,
            page_table=kv_cache.page_table if attn_metadata.page_table is None else attn_metadata.page_table,
            seq_lens=kv_cache.seq_lens if attn_metadata.seq_lens is None else attn_metadata.seq_lens,
            page_size=kv_cache.page_size,
        )

    def forward(self, query: torch.Tensor, kv_cache, attn_metadata: AttentionMetadata) -> torch.Tensor:
        if not isinstance(kv_cache, (PagedKVCache, torch.Tensor)):
            raise TypeError("kv_cache must be a PagedKVCache")
        if not attn_metadata.is_prefill and query.dim() == 4:
            query = query.squeeze(1)
        if query.dim() != 3:
            raise ValueError(f"query must be 3-D, got {tuple(query.shape)}")
        if query.shape[1] != self.num_heads:
            raise ValueError(f"query has {query.shape[1]} heads, backend expects {self.num_heads}")
        if attn_metadata.is_prefill:
            paged = (attn_metadata.k is None or attn_metadata.v is None) and (
                isinstance(kv_cache, torch.Tensor) or attn_metadata.page_table is not None)
            if attn_metadata.cu_seqlens_q is None or (attn_metadata.cu_seqlens_k is None and not paged):
                raise ValueError("prefill routing requires cu_seqlens_q and cu_seqlens_k")
            max_q = attn_metadata.max_seqlen_q
            max_k = attn_metadata.max_seqlen_k
            if max_q is None:
                max_q = int((attn_metadata.cu_seqlens_q[1:] - attn_metadata.cu_seqlens_q[:-1]).max())
            if max_k is None and not paged:
                max_k = int((attn_metadata.cu_seqlens_k[1:] - attn_metadata.cu_seqlens_k[:-1]).max())
            if attn_metadata.k is None or attn_metadata.v is None:
                if paged:
                    # K/V through the page table (the cache already holds the new tokens).
                    cache = self._resolve_cache(kv_cache, attn_metadata)
                    return prefill_paged_attention(query, cache, attn_metadata.cu_seqlens_q, int(max_q),
                                                   causal=True, softmax_scale=attn_metadata.softmax_scale)
                raise ValueError("prefill routing requires attn_metadata.k and attn_metadata.v "
                                 "(packed [total_k, num_kv_heads, head_dim]), or a page table for paged prefill")
            return prefill_attention(query, attn_metadata.k, attn_metadata.v, attn_metadata.cu_seqlens_q,
                                     attn_metadata.cu_seqlens_k, int(max_q), int(max_k), causal=True,
                                     softmax_scale=attn_metadata.softmax_scale)
        cache = self._resolve_cache(kv_cache, attn_metadata)
        return paged_decode_attention(query, cache, softmax_scale=attn_metadata.softmax_scale)
