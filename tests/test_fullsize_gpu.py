"""BASELINE cfg4 and cfg5 at full size on the GPU, checked against the oracle.

The pattern is the reference's correctness test (``tests/test_kernel_correctness.py:183-195``):
quantised decode is held to the dequantise-then-oracle target within 2e-2,
16-bit decode to 2e-3.  The kernels run on the whole batch; the oracle, which
needs seconds per long sequence, checks a sample of sequences (the shortest,
the longest, the first and the last).

* cfg4: B128, H32/8, D128, ps32, ctx ~ U[1024, 16384] (seed 3, the benchmark's
  draw), K/V N(0,1) quantised to INT8 and to e4m3 with one fp32 scale per
  (page, KV head), fp16 queries.
* cfg5: B8, H64/8 (GQA 8), D128, ps64, ctx 131072, fp16 N(0,1); also split the
  way the multi-GPU paths split it (by KV head over 8 ranks, and by page range
  over 4 ranks with the owner exchange and log-sum-exp merge), emulated on one
  GPU, against the unsplit decode.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from helpers import ATOL_QUANT, assert_close_f32, to_np

from oracle import attention as oatt
from oracle import quant as oquant

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _pool(lens, ps, seed):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    pages = [math.ceil(n / ps) for n in lens]
    pool = sum(pages)
    perm = torch.randperm(pool, generator=gen, device=DEV).to(torch.int32)
    table = torch.zeros((len(lens), max(pages)), dtype=torch.int32, device=DEV)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    return gen, pool, table, torch.tensor(lens, dtype=torch.int32, device=DEV)


def _sample(lens):
    lens = list(lens)
    return sorted({0, len(lens) - 1, int(np.argmin(lens)), int(np.argmax(lens))})


def _seq_pages(table, lens, b, ps):
    return table[b, :math.ceil(int(lens[b]) / ps)].long()


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
def test_cfg4_full_size_quantised_decode(mode):
    from flashattntile_b200 import quant
    from flashattntile_b200.kernels.decode import launch_decode

    batch, heads, kvh, dim, ps = 128, 32, 8, 128, 32
    ctx = torch.randint(1024, 16385, (batch,), generator=torch.Generator().manual_seed(3)).tolist()
    gen, pool, table, lens = _pool(ctx, ps, 3)
    cdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
    kq = torch.empty((pool, ps, kvh, dim), dtype=cdt, device=DEV)
    vq = torch.empty_like(kq)
    ks = torch.empty((pool, kvh), dtype=torch.float32, device=DEV)
    vs = torch.empty_like(ks)
    for p0 in range(0, pool, 4096):
        p1 = min(pool, p0 + 4096)
        kf = torch.randn((p1 - p0, ps, kvh, dim), generator=gen, device=DEV)
        vf = torch.randn((p1 - p0, ps, kvh, dim), generator=gen, device=DEV)
        kq[p0:p1], vq[p0:p1], ks[p0:p1], vs[p0:p1], _ = quant.quantize_kv_pages(kf, vf, mode=mode)
    q = torch.randn((batch, heads, dim), generator=gen, device=DEV).half()
    out = launch_decode(q, kq, vq, table, lens, ps, dim ** -0.5, 1, k_scale=ks, v_scale=vs)
    out32 = launch_decode(q, kq, vq, table, lens, ps, dim ** -0.5, 1, k_scale=ks, v_scale=vs,
                          out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.isfinite(out32).all()
    worst_target = worst_exact = 0.0
    for b in _sample(ctx):
        pg = _seq_pages(table, ctx, b, ps)
        codes_k, codes_v = kq[pg].cpu(), vq[pg].cpu()
        if mode != "int8":
            codes_k, codes_v = codes_k.view(torch.uint8), codes_v.view(torch.uint8)
        dk, dv = oquant.dequantize_kv_pages(codes_k.numpy(), codes_v.numpy(), ks[pg].cpu().numpy(),
                                            vs[pg].cpu().numpy(), mode)
        t1 = np.arange(len(pg), dtype=np.int32)[None]
        l1 = np.array([ctx[b]], dtype=np.int32)
        qb = to_np(q[b:b + 1])
        # The reference's target: the cache dequantised to fp16, then the fp32 oracle.
        target = oatt.attention_paged(qb, dk.astype(np.float16), dv.astype(np.float16), t1, l1, ps, dtype="f16",
                                      out_f32=True)
        exact = oatt.attention_paged(qb.astype(np.float32), dk, dv, t1, l1, ps, dtype="f32", out_f32=True)
        worst_target = max(worst_target, assert_close_f32(out32[b:b + 1], target, atol=ATOL_QUANT))
        worst_exact = max(worst_exact, assert_close_f32(out32[b:b + 1], exact, atol=2e-3))
        assert float((out[b].float() - out32[b]).abs().max()) <= 1e-3  # fp16 output = the fp32 one rounded
    assert worst_target <= 4e-3 and worst_exact <= 2e-3, (worst_target, worst_exact)


@pytest.fixture(scope="module")
def cfg5():
    batch, heads, kvh, dim, ps, ctx = 8, 64, 8, 128, 64, 131072
    gen, pool, table, lens = _pool([ctx] * batch, ps, 5)
    k = torch.empty((pool, ps, kvh, dim), dtype=torch.float16, device=DEV)
    v = torch.empty_like(k)
    for p0 in range(0, pool, 2048):
        p1 = min(pool, p0 + 2048)
        k[p0:p1] = torch.randn((p1 - p0, ps, kvh, dim), generator=gen, device=DEV).half()
        v[p0:p1] = torch.randn((p1 - p0, ps, kvh, dim), generator=gen, device=DEV).half()
    q = torch.randn((batch, heads, dim), generator=gen, device=DEV).half()
    yield {"q": q, "k": k, "v": v, "table": table, "lens": lens, "ps": ps}
    del k, v
    torch.cuda.empty_cache()


def test_cfg5_full_size_decode(cfg5):
    from flashattntile_b200.kernels.decode import launch_decode

    c = cfg5
    ps, dim = c["ps"], c["q"].shape[-1]
    out = launch_decode(c["q"], c["k"], c["v"], c["table"], c["lens"], ps, dim ** -0.5, 1)
    out32 = launch_decode(c["q"], c["k"], c["v"], c["table"], c["lens"], ps, dim ** -0.5, 1,
                          out_dtype=torch.float32)
    torch.cuda.synchronize()
    for b in (0, 7):
        pg = c["table"][b].long()
        kb, vb = to_np(c["k"][pg]), to_np(c["v"][pg])
        t1 = np.arange(len(pg), dtype=np.int32)[None]
        want = oatt.attention_paged(to_np(c["q"][b:b + 1]), kb, vb, t1, np.array([131072], np.int32), ps,
                                    dtype="f16", out_f32=True)
        assert_close_f32(out32[b:b + 1], want, atol=1e-4)
        assert float(np.abs(out[b:b + 1].float().cpu().numpy() - want).max()) <= 2e-3


def test_cfg5_head_first_and_page_split_match_unsplit(cfg5):
    from flashattntile_b200 import sharding
    from flashattntile_b200 import sequence_parallel as sp
    from flashattntile_b200.kernels.decode import launch_decode
    from flashattntile_b200.paging import PagedKVCache

    c = cfg5
    ps, dim = c["ps"], c["q"].shape[-1]
    cache = PagedKVCache(c["k"], c["v"], c["table"], c["lens"], ps)
    whole = launch_decode(c["q"], c["k"], c["v"], c["table"], c["lens"], ps, dim ** -0.5, 1,
                          out_dtype=torch.float32)
    # By KV head over 8 ranks: each rank reads a strided view of its one KV head.
    plan = sharding.plan_shards(8, 8, "page")
    assert (plan.head_groups, plan.splits) == (8, 1)
    got = torch.empty_like(whole)
    for r in range(8):
        sh = plan.shard(r)
        local = sharding.shard_cache(cache, plan, r)
        h0, h1 = sh.query_heads(64, 8)
        got[:, h0:h1] = sharding.sharded_decode(sharding.shard_query(c["q"], plan, r).contiguous(), local, plan, r,
                                                out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float((got - whole).abs().max()) <= 1e-5
    # By page range over 4 ranks: partials, rows to their owners, LSE merge.
    pplan = sharding.plan_shards(8, 4, "page", head_groups=1)
    packs = [sp.decode_partial(c["q"], sharding.shard_cache(cache, pplan, r)) for r in range(4)]
    rows = 8 * 64
    merged = torch.empty((rows, dim), dtype=torch.float32, device=DEV)
    for i, (r0, r1) in enumerate(sharding.owner_rows(rows, 4)):
        o = [sp.unpack(p, 8, 64, dim)[0].reshape(rows, dim)[r0:r1] for p in packs]
        lse = [sp.unpack(p, 8, 64, dim)[1].reshape(rows)[r0:r1] for p in packs]
        parts = torch.cat([torch.stack(o).view(4, -1), torch.stack(lse)], dim=1)
        merged[r0:r1] = sharding.merge_owned(parts, r1 - r0, dim, torch.float32)
    torch.cuda.synchronize()
    assert float((merged.view(8, 64, dim) - whole).abs().max()) <= 1e-4
