"""Host logic of the sequence-parallel (page-range split) decode, on the CPU.

The split, the local lengths, the packed partial layout and the rank order of
the exchange are checked against the oracle: partials computed by the oracle
on every rank's share, exchanged over ``gloo`` (world size 2 and 3), merged by
log-sum-exp, must equal the unsplit oracle attention.  The CUDA decode and
merge kernels are covered by ``test_sequence_parallel_gpu.py``.
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

from flashattntile_b200 import sequence_parallel as sp
from flashattntile_b200.paging import PagedKVCache
from oracle import attention as oatt
from tests.helpers import paged_case, to_np

LN2 = math.log(2.0)


@pytest.mark.parametrize("max_pages", [0, 1, 5, 7, 64, 2048])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_page_ranges_tile_the_table(max_pages, world):
    ranges = [sp.page_range(max_pages, world, r) for r in range(world)]
    covered = []
    for p0, p1 in ranges:
        assert 0 <= p0 <= p1 <= max_pages
        covered.extend(range(p0, p1))
    assert covered == list(range(max_pages))
    sizes = [p1 - p0 for p0, p1 in ranges]
    per = math.ceil(max_pages / world) if max_pages else 0
    assert max(sizes) == per
    # ranges are filled in rank order: every non-empty one but the last is full
    nonempty = [s for s in sizes if s]
    assert all(s == per for s in nonempty[:-1])


def test_page_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sp.page_range(8, 2, 2)
    with pytest.raises(ValueError):
        sp.page_range(8, 0, 0)


@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_local_lengths_partition_each_sequence(world):
    ps = 16
    lens = torch.tensor([0, 1, 15, 16, 17, 100, 160], dtype=torch.int32)
    max_pages = math.ceil(int(lens.max()) / ps)
    total = torch.zeros_like(lens)
    for r in range(world):
        p0, p1 = sp.page_range(max_pages, world, r)
        loc = sp.local_lengths(lens, ps, p0, p1)
        assert loc.dtype == torch.int32
        assert int(loc.min()) >= 0 and int(loc.max()) <= (p1 - p0) * ps
        total += loc
    assert torch.equal(total, lens)


def test_shard_view_slices_without_copy():
    q, k, v, table, lens = paged_case(3, [5, 40, 64], 4, 2, 64, 16)
    cache = PagedKVCache(k, v, table, lens, 16)
    view = sp.shard_view(cache, 1, 2)
    assert view.k_cache.data_ptr() == k.data_ptr()
    assert view.page_table.data_ptr() == table[:, 2:].data_ptr()
    assert view.page_table.stride(1) == 1
    assert view.seq_lens.tolist() == [0, 8, 32]
    empty = sp.shard_view(cache, 7, 8)  # 4 pages over 8 ranks: rank 7 holds none
    assert empty.page_table.shape[1] == 1 and empty.seq_lens.tolist() == [0, 0, 0]


def test_packed_layout():
    packed = torch.arange(sp.packed_size(2, 3, 4), dtype=torch.float32)
    o, lse = sp.unpack(packed, 2, 3, 4)
    assert o.shape == (2, 3, 4) and lse.shape == (2, 3)
    assert float(o[1, 2, 3]) == 23.0 and float(lse[0, 0]) == 24.0 and float(lse[1, 2]) == 29.0


def test_kernels_have_no_cpu_path():
    q, k, v, table, lens = paged_case(3, [5, 40], 4, 2, 64, 16)
    cache = PagedKVCache(k, v, table, lens, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        sp.decode_partial(q, cache)
    with pytest.raises(RuntimeError, match="CUDA"):
        sp.merge_partials(torch.zeros(2, sp.packed_size(2, 4, 64)), 2, 4, 64)


# ------------------------------------------------------------------ oracle partials
def _oracle_packed(q, view: PagedKVCache) -> torch.Tensor:
    """Packed (o, base-2 lse) partial of one rank's share, from the oracle."""
    acc, m, l = oatt.decode_split_partials(to_np(q), to_np(view.k_cache), to_np(view.v_cache),
                                           to_np(view.page_table), to_np(view.seq_lens), view.page_size, 1)
    acc, m, l = acc[:, :, 0], m[:, :, 0], l[:, :, 0]
    has = l > 0
    o = np.where(has[..., None], acc / np.where(has, l, 1.0)[..., None], 0.0).astype(np.float32)
    lse = np.where(has, (m + np.log(np.where(has, l, 1.0))) / LN2, -np.inf).astype(np.float32)
    return torch.from_numpy(np.concatenate([o.ravel(), lse.ravel()]))


def _merge_np(parts: np.ndarray, batch, heads, dim) -> np.ndarray:
    n = batch * heads * dim
    o = parts[:, :n].reshape(-1, batch, heads, dim).astype(np.float64)
    lse = parts[:, n:].reshape(-1, batch, heads).astype(np.float64)
    top = lse.max(axis=0)
    w = np.where(np.isneginf(lse), 0.0, np.exp2(lse - np.where(np.isneginf(top), 0.0, top)))
    return (o * w[..., None]).sum(axis=0) / w.sum(axis=0)[..., None]


CASE = dict(lens=[1, 63, 64, 65, 300, 17], heads=8, kv_heads=2, dim=64, page_size=16)


def _rank_main(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, table, lens = paged_case(21, CASE["lens"], CASE["heads"], CASE["kv_heads"], CASE["dim"],
                                          CASE["page_size"])
        cache = PagedKVCache(k, v, table, lens, CASE["page_size"])
        packed = _oracle_packed(q, sp.shard_view(cache, rank, world))
        parts = sp.exchange_partials(packed)
        np.save(os.path.join(result_dir, f"parts{rank}.npy"), parts.numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_exchange_and_merge_equal_unsplit_attention(world, tmp_path):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    q, k, v, table, lens = paged_case(21, CASE["lens"], CASE["heads"], CASE["kv_heads"], CASE["dim"],
                                      CASE["page_size"])
    cache = PagedKVCache(k, v, table, lens, CASE["page_size"])
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), CASE["page_size"],
                                out_f32=True)
    expected_parts = np.stack([_oracle_packed(q, sp.shard_view(cache, r, world)).numpy() for r in range(world)])
    for r in range(world):
        parts = np.load(tmp_path / f"parts{r}.npy")
        np.testing.assert_array_equal(parts, expected_parts)  # every rank, rank order
        got = _merge_np(parts, len(CASE["lens"]), CASE["heads"], CASE["dim"])
        np.testing.assert_allclose(got, want, atol=2e-5, rtol=0)
