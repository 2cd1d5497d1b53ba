"""Host logic of the head-first multi-GPU decode plan, on the CPU.

* ``plan_shards`` picks KV-head groups first (the largest divisor of the KV
  head count that divides the world size) and puts the rest of the ranks on
  sequences or page ranges; every rank's shard is disjoint and together they
  tile every (sequence, KV head, page) exactly once.
* ``shard_cache`` / ``shard_query`` slice a whole cache and query the way each
  rank holds them; computing every rank's shard with the oracle and putting
  the pieces back together reproduces the unsplit oracle attention.
* ``exchange_to_owners`` over ``gloo`` (world sizes 2 and 3) delivers each row
  of the fp32 partials to the rank that outputs it, in rank order; merged by
  log-sum-exp they equal the unsplit attention.

The CUDA paths (decode on a shard, the LSE-merge kernel) are covered by
``test_sharding_gpu.py``.
"""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashattntile_b200 import sharding
from flashattntile_b200 import sequence_parallel as sp
from flashattntile_b200.paging import PagedKVCache
from oracle import attention as oatt
from tests.helpers import paged_case, to_np

LN2 = math.log(2.0)


@pytest.mark.parametrize("kvh,world,groups", [(8, 1, 1), (8, 2, 2), (8, 4, 4), (8, 8, 8), (8, 16, 8),
                                              (8, 3, 1), (8, 6, 2), (1, 4, 1), (4, 8, 4), (2, 2, 2)])
def test_plan_is_head_first(kvh, world, groups):
    plan = sharding.plan_shards(kvh, world)
    assert plan.head_groups == groups and plan.splits == world // groups


@pytest.mark.parametrize("kvh,world,batch", [(8, 4, 32), (8, 16, 5), (2, 6, 7), (1, 3, 2)])
def test_sequence_shards_tile_units(kvh, world, batch):
    plan = sharding.plan_shards(kvh, world, "sequence")
    seen = np.zeros((batch, kvh), dtype=int)
    for r in range(world):
        sh = plan.shard(r, batch)
        seen[sh.seq0:sh.seq1, sh.kv_h0:sh.kv_h1] += 1
        assert plan.split_group_ranks(r)[sh.split] == r
    assert (seen == 1).all()


def test_page_shards_tile_pages():
    plan = sharding.plan_shards(2, 6, "page")  # 2 head groups x 3 page splits
    assert (plan.head_groups, plan.splits) == (2, 3)
    pages = 10
    seen = np.zeros((2, pages), dtype=int)
    for r in range(6):
        sh = plan.shard(r)
        p0, p1 = sp.page_range(pages, plan.splits, sh.split)
        seen[sh.kv_h0:sh.kv_h1, p0:p1] += 1
    assert (seen == 1).all()


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        sharding.plan_shards(8, 0)
    with pytest.raises(ValueError):
        sharding.plan_shards(8, 4, "token")
    with pytest.raises(ValueError):
        sharding.plan_shards(8, 4, head_groups=3)
    with pytest.raises(ValueError):
        sharding.plan_shards(8, 4).shard(4, 8)
    with pytest.raises(ValueError):
        sharding.plan_shards(8, 4, "sequence").shard(0)  # a sequence split needs the batch


def test_owner_rows_tile():
    for rows, world in ((512, 8), (7, 3), (3, 5), (64, 1)):
        spans = sharding.owner_rows(rows, world)
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _oracle_out(q, cache):
    return oatt.attention_paged(to_np(q), to_np(cache.k_cache), to_np(cache.v_cache), to_np(cache.page_table),
                                to_np(cache.seq_lens), cache.page_size, dtype="f16", out_f32=True)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_first_sequence_shards_reassemble(world):
    lens = [1, 40, 300, 77, 129]
    q, k, v, table, lens_t = paged_case(81, lens, 16, 8, 64, 16)
    cache = PagedKVCache(k, v, table, lens_t, 16)
    want = _oracle_out(q, cache)
    plan = sharding.plan_shards(8, world, "sequence")
    got = np.full(want.shape, np.nan, dtype=np.float32)
    for r in range(world):
        sh = plan.shard(r, len(lens))
        local = sharding.shard_cache(cache, plan, r, copy=True)
        assert local.k_cache.shape[2] == sh.kv_h1 - sh.kv_h0 and local.k_cache.is_contiguous()
        ql = sharding.shard_query(q, plan, r)
        h0, h1 = sh.query_heads(16, 8)
        if sh.seq1 > sh.seq0:
            got[sh.seq0:sh.seq1, h0:h1] = _oracle_out(ql.contiguous(), local)
    np.testing.assert_allclose(got, want, atol=1e-6, rtol=0)


def _merge_rows(o_parts, lse_parts):
    """Base-2 LSE merge of [R, rows, D] / [R, rows] partials (numpy, -inf aware)."""
    m = lse_parts.max(axis=0)
    w = np.where(np.isneginf(lse_parts), 0.0, np.exp2(lse_parts - np.where(np.isneginf(m), 0.0, m)))
    return (o_parts * w[..., None]).sum(axis=0) / w.sum(axis=0)[..., None]


def _partial(q, cache):
    """Oracle fp32 partial of one rank: normalised o [B,H,D] and base-2 lse [B,H]."""
    acc, m, l = oatt.decode_split_partials(to_np(q), to_np(cache.k_cache), to_np(cache.v_cache),
                                           to_np(cache.page_table), to_np(cache.seq_lens), cache.page_size, 1,
                                           dtype="f16")
    acc, m, l = acc[:, :, 0], m[:, :, 0], l[:, :, 0]
    with np.errstate(divide="ignore", invalid="ignore"):
        o = np.where(l[..., None] > 0, acc / l[..., None], 0.0).astype(np.float32)
        lse = np.where(l > 0, (m + np.log(l)) / LN2, -np.inf).astype(np.float32)
    return o, lse


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _owner_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = [700, 5, 1000]
        heads, kvh, dim, ps = 8, 2, 64, 16
        q, k, v, table, lens_t = paged_case(91, lens, heads, kvh, dim, ps)
        cache = PagedKVCache(k, v, table, lens_t, ps)
        plan = sharding.plan_shards(kvh, world, "page", head_groups=1)
        local = sharding.shard_cache(cache, plan, rank)
        o, lse = _partial(q, local)
        packed = torch.from_numpy(np.concatenate([o.reshape(-1), lse.reshape(-1)]))
        parts = sharding.exchange_to_owners(packed, len(lens), heads, dim)
        rows_total = len(lens) * heads
        r0, r1 = sharding.owner_rows(rows_total, world)[rank]
        n = r1 - r0
        po = parts[:, :n * dim].reshape(world, n, dim).numpy()
        pl = parts[:, n * dim:].reshape(world, n).numpy()
        merged = _merge_rows(po, pl)
        want = _oracle_out(q, cache).reshape(rows_total, dim)[r0:r1]
        result_q.put((rank, float(np.abs(merged - want).max()), tuple(parts.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_to_owners_over_gloo(world):
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_owner_worker, args=(r, world, port, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [result_q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rows_total = 3 * 8
    for rank, err, shape in results:
        r0, r1 = sharding.owner_rows(rows_total, world)[rank]
        assert shape == (world, (r1 - r0) * 65)
        assert err < 2e-6, (rank, err)
