"""Sequence-parallel decode on the GPU: the LSE-returning decode and the merge kernel.

Ranks are emulated on one GPU (each rank's share is a column slice of one page
table, ``shard_view``); their packed partials, stacked in rank order, are
merged by ``fat_lse_merge`` and compared with the oracle's unsplit attention
and with the unsplit decode kernel.  ``test_nccl_two_ranks`` runs the real
exchange (NCCL, one process per GPU) when the box has two GPUs.
"""

from __future__ import annotations

import math
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import quant as oquant
from tests.helpers import ATOL_QUANT, TAG, assert_close_f32, assert_parity_16bit, from_np, paged_case, to_np

pytestmark = pytest.mark.gpu

DEV = "cuda"
LN2 = math.log(2.0)


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _cache(q, k, v, table, lens, ps):
    from flashattntile_b200.paging import PagedKVCache

    return q.to(DEV), PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps)


def _split_and_merge(q, cache, world, out_dtype, scales=None, lse_out=None):
    from flashattntile_b200 import sequence_parallel as sp

    parts = torch.stack([sp.decode_partial(q, sp.shard_view(cache, r, world), scales=scales)
                         for r in range(world)])
    out = sp.merge_partials(parts, q.shape[0], q.shape[1], q.shape[2], out_dtype, lse_out=lse_out)
    torch.cuda.synchronize()
    return out, parts


def _oracle_lse2(q, k, v, table, lens, ps, dtype):
    _, m, l = oatt.decode_split_partials(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), ps, 1,
                                         dtype=TAG[dtype])
    return (m[:, :, 0] + np.log(l[:, :, 0])) / LN2


CASES = [
    # lens, heads, kv_heads, dim, page_size
    ([1, 63, 64, 65, 300, 1000], 8, 2, 128, 16),
    ([5, 2048, 777], 16, 2, 64, 64),
    ([4096, 4095, 129], 64, 8, 128, 64),
    ([33, 1], 4, 4, 128, 8),
]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_split_merge_matches_oracle(world, case, dtype):
    lens, heads, kvh, dim, ps = CASES[case]
    q, k, v, table, lens_t = paged_case(40 + case, lens, heads, kvh, dim, ps, dtype)
    qd, cache = _cache(q, k, v, table, lens_t, ps)
    got, _ = _split_and_merge(qd, cache, world, dtype)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), ps, dtype=TAG[dtype])
    assert_parity_16bit(got, want, dtype)


@pytest.mark.parametrize("world", [1, 2, 5])
def test_lse_and_f32_merge(world):
    lens, heads, kvh, dim, ps = CASES[0]
    q, k, v, table, lens_t = paged_case(7, lens, heads, kvh, dim, ps, torch.float16)
    qd, cache = _cache(q, k, v, table, lens_t, ps)
    lse_out = torch.empty(len(lens), heads, dtype=torch.float32, device=DEV)
    got, parts = _split_and_merge(qd, cache, world, torch.float32, lse_out=lse_out)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), ps, dtype="f16",
                                out_f32=True)
    assert_close_f32(got, want)
    want_lse = _oracle_lse2(q, k, v, table, lens_t, ps, torch.float16)
    np.testing.assert_allclose(lse_out.cpu().numpy(), want_lse, atol=1e-3, rtol=0)
    if world == 1:  # the decode kernel's own lse
        from flashattntile_b200 import sequence_parallel as sp

        _, lse1 = sp.unpack(parts[0], len(lens), heads, dim)
        np.testing.assert_allclose(lse1.cpu().numpy(), want_lse, atol=1e-3, rtol=0)


def test_partial_of_rank_without_tokens_is_neutral():
    """Short sequences leave later ranks empty: o = 0, lse = -inf, and the merge ignores them."""
    from flashattntile_b200 import sequence_parallel as sp

    lens, heads, kvh, dim, ps = [3, 20, 200], 8, 2, 128, 16
    q, k, v, table, lens_t = paged_case(11, lens, heads, kvh, dim, ps, torch.float16)
    qd, cache = _cache(q, k, v, table, lens_t, ps)
    world = 4  # 13 pages -> 4 per rank; sequence 0 lives on rank 0 only
    parts = torch.stack([sp.decode_partial(qd, sp.shard_view(cache, r, world)) for r in range(world)])
    torch.cuda.synchronize()
    o, lse = sp.unpack(parts[3], len(lens), heads, dim)
    assert torch.isneginf(lse[0]).all() and torch.isneginf(lse[1]).all()
    assert (o[0] == 0).all() and (o[1] == 0).all()
    assert torch.isfinite(lse[2]).all()
    got = sp.merge_partials(parts, len(lens), heads, dim, torch.float16)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), ps, dtype="f16")
    assert_parity_16bit(got, want, torch.float16)
    import flashattntile_b200

    assert flashattntile_b200.device_error() == 0


def test_merge_of_all_empty_rows_is_zero():
    from flashattntile_b200 import sequence_parallel as sp

    b, h, d = 2, 4, 64
    parts = torch.zeros(3, sp.packed_size(b, h, d), device=DEV)
    parts[:, b * h * d:] = -math.inf
    lse_out = torch.empty(b * h, device=DEV)
    out = sp.merge_partials(parts, b, h, d, torch.bfloat16, lse_out=lse_out)
    torch.cuda.synchronize()
    assert (out == 0).all() and torch.isneginf(lse_out).all()


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
@pytest.mark.parametrize("world", [2, 3])
def test_quantised_split_merge(mode, world):
    lens, heads, kvh, dim, ps = [17, 255, 1000], 8, 2, 128, 32
    q, k, v, table, lens_t = paged_case(13, lens, heads, kvh, dim, ps, torch.float32)
    qk, qv, sk, sv = oquant.quantize_kv_pages(k.numpy(), v.numpy(), mode)
    tdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
    q16 = q.to(torch.float16)
    qd, cache = _cache(q16, from_np(qk, tdt), from_np(qv, tdt), table, lens_t, ps)
    scales = {"k": torch.from_numpy(sk).to(DEV), "v": torch.from_numpy(sv).to(DEV)}
    got, _ = _split_and_merge(qd, cache, world, torch.float32, scales=scales)
    dk, dv = oquant.dequantize_kv_pages(qk, qv, sk, sv, mode)
    dk_t, dv_t = torch.from_numpy(dk).to(torch.float16), torch.from_numpy(dv).to(torch.float16)
    want = oatt.attention_paged(to_np(q16), to_np(dk_t), to_np(dv_t), to_np(table), to_np(lens_t), ps,
                                dtype="f16", out_f32=True)
    assert_close_f32(got, want, atol=ATOL_QUANT)


def test_split_merge_equals_unsplit_kernel():
    """Against the unsplit decode kernel on a cfg5-shaped (shortened) problem."""
    from flashattntile_b200.kernels.decode import launch_decode

    lens, heads, kvh, dim, ps = [8192] * 4, 64, 8, 128, 64
    q, k, v, table, lens_t = paged_case(5, lens, heads, kvh, dim, ps, torch.float16)
    qd, cache = _cache(q, k, v, table, lens_t, ps)
    full = launch_decode(qd, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, ps, dim ** -0.5,
                         out_dtype=torch.float32)
    for world in (2, 8):
        got, _ = _split_and_merge(qd, cache, world, torch.float32)
        assert float((got - full).abs().max()) <= 1e-4


def test_merge_rejects_bad_shapes():
    from flashattntile_b200 import sequence_parallel as sp

    with pytest.raises(ValueError):
        sp.merge_partials(torch.zeros(2, 10, device=DEV), 2, 4, 64)
    with pytest.raises(ValueError):
        sp.merge_partials(torch.zeros(2, sp.packed_size(2, 4, 64), device=DEV, dtype=torch.float16), 2, 4, 64)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_nccl_two_ranks():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, PYTHONPATH=str(root), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(root / "tests" / "sp_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "sp_worker ok" in res.stdout
