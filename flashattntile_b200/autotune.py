"""Algorithmic work accounting (the analytic half of FlashAttnTile's ``autotune.py``).

Every throughput this library reports divides one of these counts by a
measured time, as the reference does (``flashattn_tile/autotune.py:31-112``):

* ``flops_attention``: ``4 * batch * H * D * pairs`` with bottom-right causal
  pairs ``q(kv - q) + q(q + 1)/2`` (``autotune.py:31-55``);
* ``bytes_attention``: decode = Q + K + V + O, prefill = Q + K + V + O
  (``autotune.py:76-106``); scores never reach HBM.

``bytes_decode_paged`` extends the decode count to ragged batches and to
8-bit caches with their fp32 scales (one scale per (page, KV head) for K and
for V), the per-token accounting of ``quant.py:194-208``.

The reference's Triton knob tuner is not part of this library: the decode
kernel splits work over the SMs on the device and the prefill kernel has one
tile shape per head dimension.
"""

from __future__ import annotations

import math


def _causal_pairs(q_len: int, kv_len: int) -> int:
    if q_len <= 0 or kv_len <= 0:
        return 0
    if kv_len < q_len:
        raise ValueError("causal accounting requires kv_len >= q_len")
    return q_len * (kv_len - q_len) + q_len * (q_len + 1) // 2


def flops_attention(num_heads: int, head_dim: int, q_len: int, kv_len: int, causal: bool = False,
                    batch: int = 1) -> int:
    pairs = _causal_pairs(q_len, kv_len) if causal else q_len * kv_len
    return int(4 * batch * num_heads * head_dim * pairs)


def flops_attention_varlen(num_heads: int, head_dim: int, q_lens, kv_lens, causal: bool = False) -> int:
    if len(q_lens) != len(kv_lens):
        raise ValueError("q_lens and kv_lens must have the same length")
    return int(sum(flops_attention(num_heads, head_dim, int(q), int(k), causal=causal)
                   for q, k in zip(q_lens, kv_lens)))


def bytes_attention(mode: str, batch: int, q_len: int, kv_len: int, num_heads: int, num_kv_heads: int,
                    head_dim: int, elem_bytes: int = 2) -> int:
    if mode == "decode":
        if q_len != 1:
            raise ValueError("decode accounting assumes q_len == 1")
        q_bytes = batch * num_heads * head_dim * elem_bytes
        return int(2 * q_bytes + batch * kv_len * num_kv_heads * head_dim * 2 * elem_bytes)
    if mode == "prefill":
        q_bytes = batch * q_len * num_heads * head_dim * elem_bytes
        return int(2 * q_bytes + batch * kv_len * num_kv_heads * head_dim * 2 * elem_bytes)
    raise ValueError(f"unknown mode {mode!r}")


def bytes_decode_paged(seq_lens, num_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                       q_bytes: int = 2, kv_bytes: int = 2, scale_bytes: int = 0) -> int:
    """Q + O + the K/V rows of every cached token (+ 2 scales per used page per KV head)."""
    lens = [int(x) for x in seq_lens]
    batch = len(lens)
    qo = 2 * batch * num_heads * head_dim * q_bytes
    kv = sum(lens) * num_kv_heads * head_dim * 2 * kv_bytes
    scales = sum(math.ceil(n / page_size) for n in lens) * num_kv_heads * 2 * scale_bytes
    return int(qo + kv + scales)


def arithmetic_intensity(flops: float, nbytes: float) -> float:
    return float("inf") if nbytes <= 0 else float(flops) / float(nbytes)
