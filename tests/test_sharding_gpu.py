"""Head-first sharded decode on one GPU (ranks emulated as cache slices) against the oracle.

Every rank's shard is decoded by the CUDA kernel from a compact copy of its
KV-head slice (what a rank holding only its slice stores) or from a strided
view; page-range splits go through ``decode_partial``, the rows each owner
would receive from ``exchange_to_owners`` (sliced here in rank order) and the
LSE-merge kernel (``merge_owned``).  Ragged lengths, empty sequences on a
rank, GQA / MQA, fp16 / bf16 and an INT8 cache.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import TAG, assert_close_f32, paged_case, to_np

from oracle import attention as oatt
from oracle import quant as oquant

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _cache(q, k, v, table, lens, ps):
    from flashattntile_b200.paging import PagedKVCache

    return q.to(DEV), PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("world,kvh,heads", [(2, 8, 32), (4, 8, 32), (8, 8, 64), (3, 2, 8), (4, 1, 8)])
def test_sequence_sharded_decode(dtype, world, kvh, heads):
    from flashattntile_b200 import sharding

    lens = [1, 900, 17, 4000, 256, 33, 2048]
    q, k, v, table, lens_t = paged_case(101, lens, heads, kvh, 128, 16, dtype)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), 16, dtype=TAG[dtype],
                                out_f32=True)
    qd, cache = _cache(q, k, v, table, lens_t, 16)
    plan = sharding.plan_shards(kvh, world, "sequence")
    got = torch.full((len(lens), heads, 128), float("nan"), device=DEV)
    for r in range(world):
        sh = plan.shard(r, len(lens))
        if sh.seq1 == sh.seq0:
            continue
        local = sharding.shard_cache(cache, plan, r, copy=(r % 2 == 0))
        h0, h1 = sh.query_heads(heads, kvh)
        got[sh.seq0:sh.seq1, h0:h1] = sharding.sharded_decode(
            sharding.shard_query(qd, plan, r).contiguous(), local, plan, r, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert_close_f32(got, want, atol=1e-4)


@pytest.mark.parametrize("kind", ["f16", "int8"])
@pytest.mark.parametrize("world", [2, 3, 5])
def test_page_split_owner_merge(kind, world):
    from flashattntile_b200 import sharding
    from flashattntile_b200 import sequence_parallel as sp

    lens = [3000, 1, 0, 700, 64]  # a zero-length sequence; short ones leave later ranks empty
    heads, kvh, dim, ps = 16, 4, 128, 32
    q, k, v, table, lens_t = paged_case(103, lens, heads, kvh, dim, ps, torch.float32)
    scales = None
    if kind == "int8":
        qk, qv, sk, sv = oquant.quantize_kv_pages(k.numpy(), v.numpy(), "int8")
        dk, dv = oquant.dequantize_kv_pages(qk, qv, sk, sv, "int8")
        k, v = torch.from_numpy(qk), torch.from_numpy(qv)
        scales = {"k": torch.from_numpy(sk).to(DEV), "v": torch.from_numpy(sv).to(DEV)}
        kf, vf = dk, dv
    else:
        k, v = k.half(), v.half()
        kf, vf = to_np(k).astype(np.float32), to_np(v).astype(np.float32)
    q = q.half()
    nz = [b for b, n in enumerate(lens) if n > 0]
    want = oatt.attention_paged(to_np(q)[nz].astype(np.float32), kf, vf, to_np(table)[nz], to_np(lens_t)[nz], ps,
                                dtype="f32", out_f32=True)
    qd, cache = _cache(q, k, v, table, lens_t, ps)
    plan = sharding.plan_shards(kvh, world, "page", head_groups=1)
    packs = [sp.decode_partial(qd, sharding.shard_cache(cache, plan, r), scales=scales) for r in range(world)]
    rows = len(lens) * heads
    merged = torch.empty((rows, dim), dtype=torch.float32, device=DEV)
    for r0, r1 in sharding.owner_rows(rows, world):
        if r1 == r0:
            continue
        o = [sp.unpack(p, len(lens), heads, dim)[0].reshape(rows, dim)[r0:r1] for p in packs]
        lse = [sp.unpack(p, len(lens), heads, dim)[1].reshape(rows)[r0:r1] for p in packs]
        parts = torch.cat([torch.stack(o).view(world, -1), torch.stack(lse)], dim=1)
        merged[r0:r1] = sharding.merge_owned(parts, r1 - r0, dim, torch.float32)
    torch.cuda.synchronize()
    got = merged.view(len(lens), heads, dim)
    assert_close_f32(got[nz], want, atol=2e-3 if kind == "int8" else 1e-4)
    assert float(got[2].abs().max()) == 0.0  # no token anywhere: zeros, as the unsplit kernel gives
