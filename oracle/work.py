"""Algorithmic FLOP / byte counts (oracle copy of the accounting contract).

Restates ``flashattn_tile/autotune.py:31-112``.  The library keeps its own
copy in ``flashattntile_b200.autotune``; tests check the two agree and
reproduce the reference's own known answers (``tests/test_autotune.py:13-52``
of the reference).
"""

from __future__ import annotations


def causal_pairs(q_len: int, kv_len: int) -> int:
    if q_len <= 0 or kv_len <= 0:
        return 0
    if kv_len < q_len:
        raise ValueError("causal accounting requires kv_len >= q_len")
    return q_len * (kv_len - q_len) + q_len * (q_len + 1) // 2


def flops_attention(num_heads, head_dim, q_len, kv_len, causal=False, batch=1) -> int:
    pairs = causal_pairs(q_len, kv_len) if causal else q_len * kv_len
    return int(4 * batch * num_heads * head_dim * pairs)


def flops_attention_varlen(num_heads, head_dim, q_lens, kv_lens, causal=False) -> int:
    if len(q_lens) != len(kv_lens):
        raise ValueError("q_lens and kv_lens must have the same length")
    return int(sum(flops_attention(num_heads, head_dim, int(q), int(k), causal=causal)
                   for q, k in zip(q_lens, kv_lens)))


def bytes_attention(mode, batch, q_len, kv_len, num_heads, num_kv_heads, head_dim, elem_bytes=2) -> int:
    if mode == "decode":
        if q_len != 1:
            raise ValueError("decode accounting assumes q_len == 1")
        q_bytes = batch * num_heads * head_dim * elem_bytes
        kv_bytes = batch * kv_len * num_kv_heads * head_dim * 2 * elem_bytes
        return int(2 * q_bytes + kv_bytes)
    if mode == "prefill":
        q_bytes = batch * q_len * num_heads * head_dim * elem_bytes
        kv_bytes = batch * kv_len * num_kv_heads * head_dim * 2 * elem_bytes
        return int(2 * q_bytes + kv_bytes)
    raise ValueError(f"unknown mode {mode!r}")


def bytes_decode_paged(seq_lens, num_heads, num_kv_heads, head_dim, page_size, q_bytes=2, kv_bytes=2,
                       scale_bytes=0) -> int:
    """Decode bytes of a ragged batch: Q + O, the K/V rows of every cached token,
    and for 8-bit caches two fp32 scales per used (page, KV head) -- the decode
    count of ``autotune.py:76-106`` summed per sequence, with the per-token scale
    accounting of ``quant.py:194-208``."""
    import math

    lens = [int(x) for x in seq_lens]
    qo = 2 * len(lens) * num_heads * head_dim * q_bytes
    kv = sum(lens) * num_kv_heads * head_dim * 2 * kv_bytes
    scales = sum(math.ceil(n / page_size) for n in lens) * num_kv_heads * 2 * scale_bytes
    return int(qo + kv + scales)
