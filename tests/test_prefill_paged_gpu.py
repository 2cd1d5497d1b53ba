"""Paged prefill (K/V through the page table) against the oracle's varlen attention.

The oracle gathers each sequence's first seq_lens[b] tokens out of the pages
and runs the reference's varlen attention (``reference.py:97-142`` restated)
with the queries aligned to the last q_len positions.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import paging as opaging
from tests.helpers import TAG, assert_close_f32, assert_parity_16bit, to_np

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _case(seed, kv_lens, q_lens, heads, kvh, dim, ps, dtype, nan_pool=False):
    gen = torch.Generator().manual_seed(seed)
    batch = len(kv_lens)
    max_pages = max(1, max(math.ceil(n / ps) for n in kv_lens)) + 1
    pool = batch * max_pages + 3
    k = torch.randn(pool, ps, kvh, dim, generator=gen).to(dtype)
    v = torch.randn(pool, ps, kvh, dim, generator=gen).to(dtype)
    if nan_pool:  # stale slots past every sequence end hold NaN
        k_nan = torch.full_like(k, float("nan"))
        v_nan = torch.full_like(v, float("nan"))
    table = torch.randperm(pool, generator=gen)[: batch * max_pages].view(batch, max_pages).to(torch.int32)
    if nan_pool:
        kn, vn = k_nan.clone(), v_nan.clone()
        for b, n in enumerate(kv_lens):
            for t in range(n):
                pg, sl = int(table[b, t // ps]), t % ps
                kn[pg, sl], vn[pg, sl] = k[pg, sl], v[pg, sl]
        k, v = kn, vn
    q = torch.randn(sum(q_lens), heads, dim, generator=gen).to(dtype)
    cu_q = torch.tensor([0] + np.cumsum(q_lens).tolist(), dtype=torch.int32)
    return q, k, v, table, torch.tensor(kv_lens, dtype=torch.int32), cu_q


def _oracle(q, k, v, table, lens, cu_q, ps, dtype, causal=True, out_f32=False):
    ks, vs = [], []
    for b, n in enumerate(lens.tolist()):
        kb, vb = opaging.sequence_kv(to_np(k), to_np(v), to_np(table), n, b, ps)
        ks.append(kb)
        vs.append(vb)
    kp, vp = np.concatenate(ks), np.concatenate(vs)
    cu_k = np.array([0] + np.cumsum(lens.tolist()).tolist(), np.int32)
    return oatt.attention_varlen(to_np(q), kp, vp, to_np(cu_q), cu_k, causal=causal, dtype=TAG[dtype],
                                 out_f32=out_f32)


def _run(q, k, v, table, lens, cu_q, ps, causal=True, out_dtype=None):
    from flashattntile_b200.kernels.prefill import prefill_paged_attention
    from flashattntile_b200.paging import PagedKVCache

    cache = PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps)
    q_lens = (cu_q[1:] - cu_q[:-1]).tolist()
    out = prefill_paged_attention(q.to(DEV), cache, cu_q.to(DEV), max(q_lens), causal=causal, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out


CASES = [
    # kv_lens, q_lens, heads, kv_heads, dim, page_size
    ([100, 300, 17], [100, 300, 17], 4, 2, 128, 16),     # full prefill, ragged
    ([1000, 257, 64], [50, 257, 1], 8, 2, 128, 32),      # chunked: last q_len of the cached tokens
    ([513, 128], [513, 128], 4, 4, 64, 8),               # MHA, page 8
    ([700, 260], [300, 5], 8, 1, 128, 128),              # MQA, page 128
    ([640, 1030], [640, 200], 4, 2, 128, 256),           # page larger than a tile
    ([300, 129], [300, 40], 4, 2, 256, 16),              # head_dim 256 (one query tile per CTA)
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_paged_prefill_matches_oracle(case, dtype):
    kv_lens, q_lens, heads, kvh, dim, ps = CASES[case]
    q, k, v, table, lens, cu_q = _case(20 + case, kv_lens, q_lens, heads, kvh, dim, ps, dtype)
    out = _run(q, k, v, table, lens, cu_q, ps)
    want = _oracle(q, k, v, table, lens, cu_q, ps, dtype)
    atol = 2e-3  # both dtypes: bf16 feeds heavy key tiles' P as head + remainder (adaptive mode)
    assert_parity_16bit(out, want, dtype, atol=atol)
    out32 = _run(q, k, v, table, lens, cu_q, ps, out_dtype=torch.float32)
    want32 = _oracle(q, k, v, table, lens, cu_q, ps, dtype, out_f32=True)
    assert_close_f32(out32, want32, atol=atol)
    import flashattntile_b200

    assert flashattntile_b200.device_error() == 0


@pytest.mark.parametrize("ps", [16, 128])
def test_paged_prefill_ignores_nan_past_sequence_ends(ps):
    kv_lens, q_lens = [77, 200, 129], [77, 60, 129]
    q, k, v, table, lens, cu_q = _case(5, kv_lens, q_lens, 4, 2, 128, ps, torch.float16, nan_pool=True)
    out = _run(q, k, v, table, lens, cu_q, ps)
    assert torch.isfinite(out).all()
    want = _oracle(q, k, v, table, lens, cu_q, ps, torch.float16)
    assert_parity_16bit(out, want, torch.float16)


@pytest.mark.parametrize("mode", ["adaptive", "rounded"])
def test_paged_equals_packed_prefill_bitwise(mode):
    """Same keys, read packed or through pages, same P precision mode: identical
    outputs.  (bf16's default differs between the two: packed K/V runs P.V in
    fp16 against a scaled fp16 copy of V, which a paged cache does not get.)"""
    from flashattntile_b200.kernels.prefill import launch_prefill, p_precision

    kv_lens = [384, 1024, 256]
    q, k, v, table, lens, cu_q = _case(9, kv_lens, kv_lens, 8, 2, 128, 16, torch.bfloat16)
    with p_precision(mode):
        paged = _run(q, k, v, table, lens, cu_q, 16)
    ks, vs = [], []
    for b, n in enumerate(kv_lens):
        kb, vb = opaging.sequence_kv(to_np(k), to_np(v), to_np(table), n, b, 16)
        ks.append(kb)
        vs.append(vb)
    from tests.helpers import from_np

    kp = from_np(np.concatenate(ks), torch.bfloat16).to(DEV)
    vp = from_np(np.concatenate(vs), torch.bfloat16).to(DEV)
    with p_precision(mode):
        packed = launch_prefill(q.to(DEV), kp, vp, cu_q.to(DEV), cu_q.to(DEV), max(kv_lens), max(kv_lens), True,
                                128 ** -0.5)
        torch.cuda.synchronize()
    assert torch.equal(paged, packed)


def test_backend_routes_prefill_without_packed_kv_to_pages():
    from flashattntile_b200.backend import AttentionMetadata, FlashAttnTileBackend

    kv_lens, q_lens = [300, 90], [40, 90]
    q, k, v, table, lens, cu_q = _case(3, kv_lens, q_lens, 8, 2, 128, 16, torch.float16)
    kv = torch.stack([k, v]).to(DEV)  # the (2, blocks, block, Hkv, D) tensor a serving engine holds
    backend = FlashAttnTileBackend(8, 2, 128, 16)
    md = AttentionMetadata(page_table=table.to(DEV), seq_lens=lens.to(DEV), cu_seqlens_q=cu_q.to(DEV),
                           is_prefill=True, max_seqlen_q=90)
    out = backend.forward(q.to(DEV), kv, md)
    torch.cuda.synchronize()
    want = _oracle(q, k, v, table, lens, cu_q, 16, torch.float16)
    assert_parity_16bit(out, want, torch.float16)


def test_backend_decode_and_packed_prefill_routing():
    """``backend.forward`` decode (3-D and [B, 1, H, D] queries) and packed prefill
    equal the oracle (``tests/test_ops.py:111-143`` of the reference, on the GPU)."""
    from flashattntile_b200.backend import AttentionMetadata, FlashAttnTileBackend
    from flashattntile_b200.paging import PagedKVCache
    from tests.helpers import paged_case, varlen_case

    backend = FlashAttnTileBackend(num_heads=8, num_kv_heads=2, head_dim=128, page_size=16)
    q, k, v, table, lens = paged_case(31, [5, 40, 129], 8, 2, 128, 16, torch.float16)
    cache = PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), 16)
    md = AttentionMetadata(page_table=cache.page_table, seq_lens=cache.seq_lens, softmax_scale=0.35)
    out = backend.forward(q.to(DEV), cache, md)
    out4 = backend.forward(q.to(DEV).unsqueeze(1), cache, md)
    torch.cuda.synchronize()
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), 16, scale=0.35, dtype="f16")
    assert_parity_16bit(out, want, torch.float16)
    assert torch.equal(out, out4)

    qp, kp, vp, cu_q, cu_k = varlen_case(32, [3, 70], [3, 70], 8, 2, 128, torch.float16)
    mdp = AttentionMetadata(cu_seqlens_q=cu_q.to(DEV), cu_seqlens_k=cu_k.to(DEV), is_prefill=True, max_seqlen_q=70,
                            max_seqlen_k=70, k=kp.to(DEV), v=vp.to(DEV), softmax_scale=0.35)
    outp = backend.forward(qp.to(DEV), cache, mdp)
    torch.cuda.synchronize()
    wantp = oatt.attention_varlen(to_np(qp), to_np(kp), to_np(vp), to_np(cu_q), to_np(cu_k), causal=True, scale=0.35,
                                  dtype="f16")
    assert_parity_16bit(outp, wantp, torch.float16)


def test_paged_prefill_head_dim_256_rejects_small_pages():
    """One producer lane per (page, column block): head_dim 256 needs 16-token pages."""
    q, k, v, table, lens, cu_q = _case(31, [40], [40], 4, 2, 256, 8, torch.float16)
    with pytest.raises(RuntimeError, match="page_size"):
        _run(q, k, v, table, lens, cu_q, 8)
