"""fp32 attention, restated in numpy (oracle only).

Follows ``flashattn_tile/reference.py``:

* ``attention_varlen``  -- ``reference.py:50-142``: per sequence, scores
  ``einsum(q, k) * scale`` in fp32, bottom-right causal mask
  (``j <= i + kv_len - q_len``), fp32 softmax, ``probs @ v``, result cast to
  the input dtype.  GQA maps query head ``h`` to KV head ``h // G``
  (``reference.py:126-128``).
* ``attention_paged``   -- ``reference.py:145-194``: gather each sequence's
  pages, then one query per sequence through the varlen path.
* ``attention_dense``   -- ``reference.py:197-219``.
* ``decode_split_partials`` / ``lse_merge`` -- the split-K partials and the
  log-sum-exp merge of ``flashattn_tile/kernels/decode.py:223-356``
  (``m* = max m_s; l* = sum l_s e^(m_s-m*); o = sum acc_s e^(m_s-m*) / l*``).

Arrays are raw storage (``numerics.DTYPES``); every function takes the dtype
tag and returns the output in that encoding, or fp32 with ``out_f32=True``.
"""

from __future__ import annotations

import contextlib
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import numerics
from .paging import gather_paged, sequence_kv

_ROW_CHUNK = 256


def _as_int_list(cu, name):
    values = [int(x) for x in np.asarray(cu).reshape(-1).tolist()]
    if len(values) < 2:
        raise ValueError(f"{name} must have at least 2 entries (batch + 1)")
    if values[0] != 0:
        raise ValueError(f"{name} must start at 0, got {values[0]}")
    if any(b < a for a, b in zip(values, values[1:])):
        raise ValueError(f"{name} must be non-decreasing, got {values}")
    return values


@contextlib.contextmanager
def blas_single_thread():
    """Pin the BLAS / OpenMP pools to one thread while a thread pool of ours runs
    (``threads`` workers each calling a multi-threaded BLAS oversubscribe the
    cores several times over).  No-op when threadpoolctl is absent."""
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover - threadpoolctl ships with this image
        yield
        return
    with threadpool_limits(limits=1):
        yield


def _split_heads(qf, kf, vf):
    q_len, heads, dim = qf.shape
    kv_heads = kf.shape[1]
    group = heads // kv_heads
    qh = qf.reshape(q_len, kv_heads, group, dim).transpose(1, 2, 0, 3)  # [Hkv, G, q, D]
    kh = np.ascontiguousarray(kf.transpose(1, 2, 0))[:, None]  # [Hkv, 1, D, kv]
    vh = np.ascontiguousarray(vf.transpose(1, 0, 2))[:, None]  # [Hkv, 1, kv, D]
    return qh, kh, vh


def _attend_rows(qh, kh, vh, r0, r1, offset, causal, scale):
    """Rows ``[r0, r1)`` of one sequence -> ``[Hkv, G, rows, D]`` fp32 (reference.py:126-140)."""
    kv_len = kh.shape[-1]
    s = np.matmul(qh[:, :, r0:r1], kh) * np.float32(scale)  # [Hkv, G, rows, kv]
    if causal:
        qi = np.arange(r0, r1)[:, None] + offset
        kj = np.arange(kv_len)[None, :]
        s = np.where(kj <= qi, s, np.float32(-np.inf))
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    p = e / e.sum(axis=-1, keepdims=True)
    return np.matmul(p, vh)


def attend(qf, kf, vf, causal, scale):
    """One sequence: ``qf [q_len, H, D]``, ``kf/vf [kv_len, Hkv, D]`` fp32 -> fp32."""
    q_len, heads, dim = qf.shape
    kv_len, kv_heads, _ = kf.shape
    qh, kh, vh = _split_heads(qf, kf, vf)
    out = np.empty((kv_heads, heads // kv_heads, q_len, dim), dtype=np.float32)
    offset = kv_len - q_len
    for r0 in range(0, q_len, _ROW_CHUNK):
        r1 = min(q_len, r0 + _ROW_CHUNK)
        out[:, :, r0:r1] = _attend_rows(qh, kh, vh, r0, r1, offset, causal, scale)
    return out.transpose(2, 0, 1, 3).reshape(q_len, heads, dim)


def _check_qkv(q, k, v):
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("q, k, v must be 3-D [tokens, heads, head_dim]")
    if q.shape[-1] != k.shape[-1] or k.shape != v.shape:
        raise ValueError(f"shape mismatch: q {q.shape}, k {k.shape}, v {v.shape}")
    if q.shape[1] % k.shape[1] != 0:
        raise ValueError(f"num_heads ({q.shape[1]}) must be divisible by num_kv_heads ({k.shape[1]})")


def attention_varlen(q, k, v, cu_q, cu_k, causal=True, scale=None, dtype="f32", out_f32=False, threads=1):
    """``ref_attention_varlen`` (``reference.py:50-142``) on storage arrays.

    ``threads > 1`` computes the (sequence, row chunk) blocks on a thread pool
    with BLAS pinned to one thread per worker; every block's arithmetic is the
    one of the serial loop, so the result is bitwise the same.
    """
    _check_qkv(q, k, v)
    cq = _as_int_list(cu_q, "cu_seqlens_q")
    ck = _as_int_list(cu_k, "cu_seqlens_k")
    if len(cq) != len(ck):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must have the same length")
    if cq[-1] != q.shape[0]:
        raise ValueError(f"cu_seqlens_q ends at {cq[-1]} but q has {q.shape[0]} tokens")
    if ck[-1] != k.shape[0]:
        raise ValueError(f"cu_seqlens_k ends at {ck[-1]} but k has {k.shape[0]} tokens")
    scale = float(scale) if scale is not None else q.shape[-1] ** -0.5
    qf = numerics.to_f32(q, dtype)
    kf = numerics.to_f32(k, dtype)
    vf = numerics.to_f32(v, dtype)
    out = np.zeros(q.shape, dtype=np.float32)
    blocks = []
    for b in range(len(cq) - 1):
        q0, q1, k0, k1 = cq[b], cq[b + 1], ck[b], ck[b + 1]
        q_len, kv_len = q1 - q0, k1 - k0
        if q_len == 0:
            continue
        if kv_len == 0:
            raise ValueError(f"sequence {b} has {q_len} queries but no keys")
        if causal and kv_len < q_len:
            raise ValueError(
                f"causal bottom-right alignment requires kv_len >= q_len (sequence {b}: {kv_len} < {q_len})"
            )
        if threads <= 1:
            out[q0:q1] = attend(qf[q0:q1], kf[k0:k1], vf[k0:k1], causal, scale)
            continue
        split = _split_heads(qf[q0:q1], kf[k0:k1], vf[k0:k1])
        blocks += [(q0, split, r0, min(q_len, r0 + _ROW_CHUNK), kv_len - q_len)
                   for r0 in range(0, q_len, _ROW_CHUNK)]

    def one(block):
        q0, (qh, kh, vh), r0, r1, offset = block
        rows = _attend_rows(qh, kh, vh, r0, r1, offset, causal, scale)  # [Hkv, G, rows, D]
        out[q0 + r0:q0 + r1] = rows.transpose(2, 0, 1, 3).reshape(r1 - r0, -1, rows.shape[-1])

    if blocks:
        # Largest blocks first so the pool finishes together.
        blocks.sort(key=lambda blk: -(blk[1][1].shape[-1] * (blk[3] - blk[2])))
        with blas_single_thread(), ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(one, blocks))
    return out if out_f32 else numerics.from_f32(out, dtype)


def attention_paged(q, k_cache, v_cache, page_table, seq_lens, page_size, scale=None,
                    dtype="f32", out_f32=False, threads=1):
    """``ref_attention_paged`` (``reference.py:145-194``): one query per sequence.

    ``threads > 1`` runs sequences on a thread pool (numpy releases the GIL in
    its copies and matmuls); the arithmetic per sequence is unchanged.
    """
    if q.ndim != 3:
        raise ValueError(f"q must be [batch, heads, head_dim], got {q.shape}")
    if q.shape[0] != seq_lens.shape[0]:
        raise ValueError(f"q batch {q.shape[0]} != seq_lens batch {seq_lens.shape[0]}")
    if q.shape[-1] != k_cache.shape[-1]:
        raise ValueError(f"q head_dim {q.shape[-1]} != cache head_dim {k_cache.shape[-1]}")
    if q.shape[1] % k_cache.shape[2] != 0:
        raise ValueError(f"num_heads {q.shape[1]} not divisible by num_kv_heads {k_cache.shape[2]}")
    batch = q.shape[0]
    lengths = [int(x) for x in seq_lens.tolist()]
    if batch == 0 or sum(lengths) == 0:
        raise ValueError("ref_attention_paged requires at least one cached token")
    for b, length in enumerate(lengths):
        if length == 0:
            raise ValueError(f"sequence {b} has 1 queries but no keys")
    scale = float(scale) if scale is not None else q.shape[-1] ** -0.5
    qf = numerics.to_f32(q, dtype)
    out = np.empty(q.shape, dtype=np.float32)

    def one(b):
        k, v = sequence_kv(k_cache, v_cache, page_table, lengths[b], b, page_size)
        out[b] = attend(qf[b : b + 1], numerics.to_f32(k, dtype), numerics.to_f32(v, dtype),
                        True, scale)[0]

    if threads > 1:
        with blas_single_thread(), ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(one, range(batch)))
    else:
        for b in range(batch):
            one(b)
    return out if out_f32 else numerics.from_f32(out, dtype)


def attention_dense(q, k, v, causal=True, scale=None, dtype="f32"):
    """``ref_attention_dense`` (``reference.py:197-219``): ``[B, H, S, D]`` tensors."""
    batch, heads, q_len, dim = q.shape
    kv_len = k.shape[2]
    qt = q.transpose(0, 2, 1, 3).reshape(batch * q_len, heads, dim)
    kt = k.transpose(0, 2, 1, 3).reshape(batch * kv_len, k.shape[1], dim)
    vt = v.transpose(0, 2, 1, 3).reshape(batch * kv_len, v.shape[1], dim)
    cq = [b * q_len for b in range(batch + 1)]
    ck = [b * kv_len for b in range(batch + 1)]
    out = attention_varlen(qt, kt, vt, cq, ck, causal, scale, dtype)
    return out.reshape(batch, q_len, heads, dim).transpose(0, 2, 1, 3)


def decode_split_partials(q, k_cache, v_cache, page_table, seq_lens, page_size, split_k,
                          scale=None, dtype="f32"):
    """Per-split ``(acc, m, l)`` of ``decode.py:258-313`` (natural-log domain).

    Split ``s`` covers pages ``[s*pps, min(n, (s+1)*pps))`` with
    ``pps = ceil(n / split_k)``; an empty split yields ``m=-inf, l=0, acc=0``.
    """
    batch, heads, dim = q.shape
    kv_heads = k_cache.shape[2]
    group = heads // kv_heads
    scale = float(scale) if scale is not None else dim ** -0.5
    qf = numerics.to_f32(q, dtype)
    acc = np.zeros((batch, heads, split_k, dim), dtype=np.float32)
    m = np.full((batch, heads, split_k), -np.inf, dtype=np.float32)
    l = np.zeros((batch, heads, split_k), dtype=np.float32)
    for b in range(batch):
        length = int(seq_lens[b])
        n = math.ceil(length / page_size)
        pps = math.ceil(n / split_k)
        k, v = sequence_kv(k_cache, v_cache, page_table, length, b, page_size)
        kf, vf = numerics.to_f32(k, dtype), numerics.to_f32(v, dtype)
        for s in range(split_k):
            t0, t1 = s * pps * page_size, min(length, (s + 1) * pps * page_size)
            if t1 <= t0:
                continue
            for h in range(heads):
                sc = (kf[t0:t1, h // group] @ qf[b, h]) * np.float32(scale)
                mm = sc.max()
                p = np.exp(sc - mm)
                m[b, h, s] = mm
                l[b, h, s] = p.sum()
                acc[b, h, s] = p @ vf[t0:t1, h // group]
    return acc, m, l


def lse_merge(acc, m, l):
    """Merge ``[..., S, D]`` partials with their ``[..., S]`` maxima and sums."""
    gm = m.max(axis=-1, keepdims=True)
    w = np.where(np.isneginf(m), 0.0, np.exp(m - np.where(np.isneginf(gm), 0.0, gm)))
    gl = (l * w).sum(axis=-1)
    return (acc * w[..., None]).sum(axis=-2) / gl[..., None]


def default_threads() -> int:
    return os.cpu_count() or 1


__all__ = [
    "attend",
    "attention_varlen",
    "attention_paged",
    "attention_dense",
    "blas_single_thread",
    "decode_split_partials",
    "lse_merge",
    "gather_paged",
    "default_threads",
]
