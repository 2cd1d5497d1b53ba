"""Packed varlen causal/non-causal prefill attention on B200.

Python API of FlashAttnTile's ``flashattn_tile/kernels/prefill.py``:
``prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
max_seqlen_k, causal=True, softmax_scale=None, config=None)``
(``prefill.py:236-326``) and ``DEFAULT_CONFIG`` (``prefill.py:145-150``).

The launch goes to the sm_100a kernel ``fat_prefill_varlen`` (tcgen05 MMAs
with accumulators in tensor memory, TMA-fed K/V).  ``config`` keys are
validated as in the reference and otherwise ignored.
"""

from __future__ import annotations

import contextlib

import torch

from .. import _config, _lib

DEFAULT_CONFIG = {"BLOCK_M": 64, "BLOCK_N": 64, "num_warps": 4, "num_stages": 3}
HAS_TRITON = False
HAS_CUDA_KERNELS = _lib.available()

# How P enters the P.V product (``fat_set_prefill_p_split``).  The reference
# kernel rounds P to the input dtype once (``prefill.py:128``); with bf16 that
# alone moves outputs by up to ~4e-3 where a row has few keys or a few keys
# dominate it.  By default bf16 feeds a key tile as a 16-bit head plus a 16-bit
# remainder (a second P.V pass over that tile) whenever one of its keys holds
# more than 1/16 of its row's probability sum so far ("adaptive"): every key
# left rounded then weighs at most 1/16 in the output.
P_SPLIT_MODES = {"auto": -1, "rounded": 0, "adaptive": 1, "all_tiles": 2, "fp16_pv": 3}


def set_p_precision(mode: str) -> str:
    """Set the P.V precision mode for later prefill launches; returns the previous one.

    ``"auto"`` (default: bf16 ``"fp16_pv"``, paged bf16 ``"adaptive"``, fp16
    ``"rounded"``), ``"rounded"`` (the reference's arithmetic), ``"adaptive"``,
    ``"all_tiles"``, ``"fp16_pv"`` (bf16, packed K/V: P.V in fp16 against a
    scaled fp16 copy of V)."""
    if mode not in P_SPLIT_MODES:
        raise ValueError(f"unknown P precision mode {mode!r}; expected one of {sorted(P_SPLIT_MODES)}")
    prev = _lib.load().fat_set_prefill_p_split(P_SPLIT_MODES[mode])
    return {v: k for k, v in P_SPLIT_MODES.items()}[prev]


@contextlib.contextmanager
def p_precision(mode: str):
    """Context manager form of :func:`set_p_precision`."""
    prev = set_p_precision(mode)
    try:
        yield
    finally:
        set_p_precision(prev)


SCHEDULES = {"persistent": 0, "per_item": 1}


def set_schedule(mode: str) -> str:
    """Set the prefill grid for later launches; returns the previous one.

    ``"persistent"`` (default: one CTA per SM claiming (head, sequence,
    256-row query pair) items from a per-stream counter) or ``"per_item"``
    (one CTA per item).  Outputs are bitwise identical."""
    if mode not in SCHEDULES:
        raise ValueError(f"unknown prefill schedule {mode!r}; expected one of {sorted(SCHEDULES)}")
    prev = _lib.load().fat_set_prefill_schedule(SCHEDULES[mode])
    return {v: k for k, v in SCHEDULES.items()}[prev]


@contextlib.contextmanager
def schedule(mode: str):
    """Context manager form of :func:`set_schedule`."""
    prev = set_schedule(mode)
    try:
        yield
    finally:
        set_schedule(prev)


def _resolve_config(config: dict | None) -> dict:
    """``prefill.py:167-191`` without the persisted tuning lookup."""
    resolved = dict(DEFAULT_CONFIG)
    if config is not None:
        unknown = set(config) - set(DEFAULT_CONFIG)
        if unknown:
            raise ValueError(f"unknown prefill config keys: {sorted(unknown)}")
        resolved.update(config)
    for key in ("BLOCK_M", "BLOCK_N"):
        if resolved[key] <= 0 or resolved[key] & (resolved[key] - 1):
            raise ValueError(f"{key} must be a positive power of two, got {resolved[key]}")
    if resolved["num_warps"] not in (1, 2, 4, 8, 16, 32):
        raise ValueError(f"num_warps must be a power of two <= 32, got {resolved['num_warps']}")
    if resolved["num_stages"] < 1:
        raise ValueError(f"num_stages must be >= 1, got {resolved['num_stages']}")
    return resolved


def _validate_inputs(q, k, v, cu_seqlens_q, cu_seqlens_k, causal) -> None:
    """``prefill.py:194-233``: same checks, order and messages."""
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be 3-D [tokens, heads, head_dim]")
    if k.shape != v.shape:
        raise ValueError(f"k shape {tuple(k.shape)} != v shape {tuple(v.shape)}")
    if q.shape[-1] != k.shape[-1]:
        raise ValueError(f"q head_dim {q.shape[-1]} != k head_dim {k.shape[-1]}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"dtype mismatch: q {q.dtype}, k {k.dtype}, v {v.dtype}")
    if not q.is_floating_point():
        raise ValueError(f"expected floating point inputs, got {q.dtype}")
    if q.device != k.device or k.device != v.device:
        raise ValueError("q, k, v must live on the same device")
    if cu_seqlens_q.dim() != 1 or cu_seqlens_k.dim() != 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be 1-D")
    if cu_seqlens_q.shape[0] != cu_seqlens_k.shape[0]:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must have the same batch dimension")
    if cu_seqlens_q.numel() < 2:
        raise ValueError("cu_seqlens must contain at least batch + 1 entries")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be int32")
    if cu_seqlens_q.device != q.device or cu_seqlens_k.device != q.device:
        raise ValueError("cu_seqlens must live on the same device as q")
    if _config.validate_values():
        cq = cu_seqlens_q.tolist()
        ck = cu_seqlens_k.tolist()
        if cq[0] != 0 or ck[0] != 0:
            raise ValueError("cu_seqlens must start at 0")
        if cq[-1] != q.shape[0]:
            raise ValueError("cu_seqlens_q[-1] must equal q.shape[0]")
        if ck[-1] != k.shape[0]:
            raise ValueError("cu_seqlens_k[-1] must equal k.shape[0]")
        if any(b < a for a, b in zip(cq, cq[1:])):
            raise ValueError("cu_seqlens_q must be non-decreasing")
        if any(b < a for a, b in zip(ck, ck[1:])):
            raise ValueError("cu_seqlens_k must be non-decreasing")
        if causal and any((k1 - k0) < (q1 - q0) for q0, q1, k0, k1 in zip(cq, cq[1:], ck, ck[1:])):
            raise ValueError("causal bottom-right alignment requires kv_len >= q_len per sequence")
    if q.shape[1] % k.shape[1] != 0:
        raise ValueError(f"num_heads ({q.shape[1]}) must be divisible by num_kv_heads ({k.shape[1]})")


def launch_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal, softmax_scale,
                   out=None, out_dtype=None):
    """Run ``fat_prefill_varlen`` on the current stream (no host sync)."""
    for t in (q, k, v, cu_seqlens_q, cu_seqlens_k):
        if not t.is_cuda:
            raise RuntimeError("flashattntile_b200 runs on CUDA tensors only; it has no CPU path")
    lib = _lib.load()
    dev = q.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()

    def aligned(t):
        eb = t.element_size()
        ok = (t.stride(2) == 1 and t.data_ptr() % 16 == 0 and (t.stride(0) * eb) % 16 == 0
              and (t.stride(1) * eb) % 16 == 0)
        return t if ok else t.contiguous()

    q, k, v = aligned(q), aligned(k), aligned(v)
    cu_seqlens_q = cu_seqlens_q.contiguous()
    cu_seqlens_k = cu_seqlens_k.contiguous()
    if out is not None:
        # A given output fixes the dtype the kernel writes.
        if out_dtype is not None and out_dtype != out.dtype:
            raise ValueError(f"out_dtype {out_dtype} does not match out's dtype {out.dtype}")
        if out.shape != q.shape or not out.is_cuda:
            raise ValueError(f"out must be a CUDA tensor of q's shape {tuple(q.shape)}, got {tuple(out.shape)}")
        out_dtype = out.dtype
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=dev)
    with torch.cuda.device(idx):
        err = _lib.error_word(dev)
        status = lib.fat_prefill_varlen(
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
            v.stride(0), v.stride(1), out.data_ptr(), out.stride(0), out.stride(1), cu_seqlens_q.data_ptr(),
            cu_seqlens_k.data_ptr(), cu_seqlens_q.numel() - 1, q.shape[0], k.shape[0], q.shape[1], k.shape[1],
            q.shape[2], int(max_seqlen_q), int(max_seqlen_k), int(bool(causal)), float(softmax_scale),
            _lib.DTYPE_CODE[q.dtype], _lib.DTYPE_CODE[out_dtype], err.data_ptr(), _lib.stream_handle(dev))
    _lib.check(status, "prefill_varlen")
    return out


def prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int, max_seqlen_k: int,
                      causal: bool = True, softmax_scale: float | None = None, config: dict | None = None):
    """Fused varlen prefill -> ``[total_q, num_heads, head_dim]`` in q's dtype."""
    _validate_inputs(q, k, v, cu_seqlens_q, cu_seqlens_k, causal)
    scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
    if max_seqlen_q <= 0:
        raise ValueError(f"max_seqlen_q must be positive, got {max_seqlen_q}")
    if max_seqlen_k <= 0:
        raise ValueError(f"max_seqlen_k must be positive, got {max_seqlen_k}")
    _resolve_config(config)
    if not q.is_cuda:
        raise RuntimeError("flashattntile_b200 runs on CUDA tensors only; it has no CPU path")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError(f"prefill has fp16/bf16 kernels only, got {q.dtype}")
    return launch_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), int(max_seqlen_k), bool(causal),
                          scale)


def prefill_paged_attention(q, cache, cu_seqlens_q, max_seqlen_q: int, causal: bool = True,
                            softmax_scale: float | None = None, out_dtype=None):
    """Prefill / chunked prefill over a paged cache -> ``[total_q, num_heads, head_dim]``.

    No reference counterpart (FlashAttnTile's prefill needs packed K/V,
    ``backend.py:158-162``): the keys of sequence b are its ``cache.seq_lens[b]``
    cached tokens, read through ``cache.page_table``; its ``q_len`` queries (from
    ``cu_seqlens_q``) are the last ``q_len`` of those positions (bottom-right
    causal alignment, as ``prefill_attention``).  The new tokens' K/V must
    already be in the cache (``append_tokens`` or the engine's own writer)."""
    from ..paging import PagedKVCache, validate_metadata

    if not isinstance(cache, PagedKVCache):
        raise TypeError("cache must be a PagedKVCache")
    validate_metadata(cache)
    if q.dim() != 3 or q.shape[2] != cache.head_dim:
        raise ValueError(f"q must be [total_q, num_heads, {cache.head_dim}], got {tuple(q.shape)}")
    if q.shape[1] % cache.num_kv_heads != 0:
        raise ValueError(f"num_heads {q.shape[1]} must be divisible by num_kv_heads {cache.num_kv_heads}")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_q.dim() != 1 or cu_seqlens_q.numel() != cache.batch_size + 1:
        raise ValueError("cu_seqlens_q must be int32 [batch + 1]")
    if q.dtype != cache.k_cache.dtype:
        raise ValueError(f"q dtype {q.dtype} must match the cache dtype {cache.k_cache.dtype}")
    for t in (q, cache.k_cache, cache.page_table, cache.seq_lens, cu_seqlens_q):
        if not t.is_cuda:
            raise RuntimeError("flashattntile_b200 runs on CUDA tensors only; it has no CPU path")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError(f"prefill has fp16/bf16 kernels only, got {q.dtype}")
    if max_seqlen_q <= 0:
        raise ValueError(f"max_seqlen_q must be positive, got {max_seqlen_q}")
    if _config.validate_values() and cache.batch_size:
        q_lens = (cu_seqlens_q[1:] - cu_seqlens_q[:-1]).to(cache.seq_lens.device)
        lo, hi, over = torch.stack([q_lens.min(), q_lens.max(), (q_lens - cache.seq_lens).max()]).tolist()
        if lo < 0 or hi > max_seqlen_q:
            raise ValueError(f"q lengths must lie in [0, max_seqlen_q={max_seqlen_q}]")
        if causal and over > 0:
            raise ValueError("causal paged prefill needs q_len <= cached length for every sequence")
        from ..paging import validate_cache

        validate_cache(cache)
    scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
    if cache.k_cache.stride() != cache.v_cache.stride() or cache.k_cache.stride(3) != 1:
        raise ValueError("k_cache and v_cache need equal strides and a contiguous head_dim")
    page_table = cache.page_table if cache.page_table.stride(1) == 1 else cache.page_table.contiguous()
    dev = q.device
    out_dtype = out_dtype or q.dtype
    out = torch.empty(q.shape, dtype=out_dtype, device=dev)
    if q.stride(2) != 1 or (q.stride(0) * q.element_size()) % 16 or (q.stride(1) * q.element_size()) % 16:
        q = q.contiguous()
    lib = _lib.load()
    k = cache.k_cache
    with torch.cuda.device(dev):
        err = _lib.error_word(dev)
        status = lib.fat_prefill_paged(
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), cache.v_cache.data_ptr(), k.stride(0), k.stride(1),
            k.stride(2), k.shape[0], page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
            cu_seqlens_q.contiguous().data_ptr(), cache.seq_lens.contiguous().data_ptr(), out.data_ptr(),
            out.stride(0), out.stride(1), cache.batch_size, q.shape[0], q.shape[1], cache.num_kv_heads,
            cache.head_dim, cache.page_size, int(max_seqlen_q), int(bool(causal)), scale,
            _lib.DTYPE_CODE[q.dtype], _lib.DTYPE_CODE[out_dtype], err.data_ptr(), _lib.stream_handle(dev))
    _lib.check(status, "prefill_paged")
    return out
