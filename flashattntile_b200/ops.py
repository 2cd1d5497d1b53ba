"""``torch.library`` custom ops, drop-in for FlashAttnTile's ``flashattn_tile/ops.py``.

Registered in the ``flashattn_tile`` namespace with the reference's schemas:

``flashattn_tile::paged_decode``     (``ops.py:35-55``)
    ``(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k) -> [B, H, D]``
``flashattn_tile::prefill_varlen``   (``ops.py:76-99``)
    ``(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal, softmax_scale) -> [T, H, D]``

plus one op the reference lacks (its quantised decode had no op):

``flashattn_tile::paged_decode_quant``
    ``(q, k_cache, v_cache, k_scale, v_scale, page_table, seq_lens, page_size, softmax_scale, split_k)``

Real kernels are registered for CUDA only; a CPU call raises (there is no CPU
kernel) instead of computing something slowly.  Fake kernels only read
metadata (``ops.py:58-73``, ``102-118``), so ``torch.compile(fullgraph=True)``
traces the ops without graph breaks.
"""

from __future__ import annotations

import torch

from .kernels.decode import _fast_decode, _fast_key, paged_decode_attention, paged_decode_attention_fp8
from .kernels.prefill import prefill_attention
from .paging import PagedKVCache

__all__ = ["paged_decode", "prefill_varlen", "paged_decode_quant", "ops_available", "PAGED_DECODE_OP",
           "PREFILL_OP", "PAGED_DECODE_QUANT_OP"]


# Registered through ``torch.library.Library`` (schema + CUDA kernel + fake)
# rather than ``torch.library.custom_op``: the same op names, schemas and
# no-mutation contract, without custom_op's Python wrapper layers (about 9 us
# per call of host time, which a decode step's GPU otherwise waits out).
_LIB = torch.library.Library("flashattn_tile", "DEF")
_LIB.define("paged_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor page_table, Tensor seq_lens, "
            "int page_size, float softmax_scale, int split_k) -> Tensor")
_LIB.define("paged_decode_quant(Tensor q, Tensor k_cache, Tensor v_cache, Tensor k_scale, Tensor v_scale, "
            "Tensor page_table, Tensor seq_lens, int page_size, float softmax_scale, int split_k) -> Tensor")
_LIB.define("prefill_varlen(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens_q, Tensor cu_seqlens_k, "
            "int max_seqlen_q, int max_seqlen_k, bool causal, float softmax_scale) -> Tensor")


def _paged_decode_cuda(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
                       seq_lens: torch.Tensor, page_size: int, softmax_scale: float, split_k: int) -> torch.Tensor:
    # Steps after the first with the same tensors skip the structural checks (_fast_decode).
    out = _fast_decode(_fast_key(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k))
    if out is not None:
        return out
    cache = PagedKVCache(k_cache=k_cache, v_cache=v_cache, page_table=page_table, seq_lens=seq_lens,
                         page_size=int(page_size))
    return paged_decode_attention(q, cache, softmax_scale=softmax_scale, config={"split_k": int(split_k)})


def _paged_decode_quant_cuda(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                             v_scale: torch.Tensor, page_table: torch.Tensor, seq_lens: torch.Tensor, page_size: int,
                             softmax_scale: float, split_k: int) -> torch.Tensor:
    out = _fast_decode(_fast_key(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k,
                                 k_scale, v_scale))
    if out is not None:
        return out
    cache = PagedKVCache(k_cache=k_cache, v_cache=v_cache, page_table=page_table, seq_lens=seq_lens,
                         page_size=int(page_size))
    return paged_decode_attention_fp8(q, cache, {"k": k_scale, "v": v_scale}, softmax_scale=softmax_scale,
                                      config={"split_k": int(split_k)})


def _prefill_varlen_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                         cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, causal: bool,
                         softmax_scale: float) -> torch.Tensor:
    return prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), int(max_seqlen_k),
                             causal=bool(causal), softmax_scale=softmax_scale)


_LIB.impl("paged_decode", _paged_decode_cuda, "CUDA")
_LIB.impl("paged_decode_quant", _paged_decode_quant_cuda, "CUDA")
_LIB.impl("prefill_varlen", _prefill_varlen_cuda, "CUDA")


@torch.library.register_fake("flashattn_tile::paged_decode")
def _paged_decode_fake(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k):
    torch._check(q.dim() == 3, lambda: f"q must be 3-D, got {q.dim()}")
    torch._check(q.shape[0] == seq_lens.shape[0], lambda: "q batch must match seq_lens")
    torch._check(q.shape[2] == k_cache.shape[3], lambda: "q head_dim must match cache")
    torch._check(q.shape[1] % k_cache.shape[2] == 0, lambda: "heads must be divisible by KV heads")
    return q.new_empty(q.shape)


@torch.library.register_fake("flashattn_tile::paged_decode_quant")
def _paged_decode_quant_fake(q, k_cache, v_cache, k_scale, v_scale, page_table, seq_lens, page_size, softmax_scale,
                             split_k):
    torch._check(q.dim() == 3, lambda: f"q must be 3-D, got {q.dim()}")
    torch._check(q.shape[0] == seq_lens.shape[0], lambda: "q batch must match seq_lens")
    torch._check(q.shape[2] == k_cache.shape[3], lambda: "q head_dim must match cache")
    torch._check(q.shape[1] % k_cache.shape[2] == 0, lambda: "heads must be divisible by KV heads")
    torch._check(k_scale.shape == (k_cache.shape[0], k_cache.shape[2]), lambda: "k_scale must be [pages, kv_heads]")
    return q.new_empty(q.shape)


@torch.library.register_fake("flashattn_tile::prefill_varlen")
def _prefill_varlen_fake(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal, softmax_scale):
    torch._check(q.dim() == 3, lambda: f"q must be 3-D, got {q.dim()}")
    torch._check(k.shape == v.shape, lambda: "k and v shapes must match")
    torch._check(q.shape[2] == k.shape[2], lambda: "q and k head_dim must match")
    torch._check(q.shape[1] % k.shape[1] == 0, lambda: "heads must be divisible by KV heads")
    return q.new_empty(q.shape)


paged_decode = torch.ops.flashattn_tile.paged_decode
paged_decode_quant = torch.ops.flashattn_tile.paged_decode_quant
prefill_varlen = torch.ops.flashattn_tile.prefill_varlen


PAGED_DECODE_OP = "flashattn_tile::paged_decode"
PREFILL_OP = "flashattn_tile::prefill_varlen"
PAGED_DECODE_QUANT_OP = "flashattn_tile::paged_decode_quant"


def ops_available() -> bool:
    """True when the ops are registered in this process (``ops.py:125-130``)."""
    ns = torch.ops.flashattn_tile
    return hasattr(ns, "paged_decode") and hasattr(ns, "prefill_varlen") and hasattr(ns, "paged_decode_quant")
