"""CUDA-graph decode loop: replays equal the eager (append, decode) sequence bit for bit."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _clone(cache):
    from flashattntile_b200.paging import PagedKVCache

    return PagedKVCache(cache.k_cache.clone(), cache.v_cache.clone(), cache.page_table.clone(),
                        cache.seq_lens.clone(), cache.page_size)


@pytest.mark.parametrize("kind", ["f16", "bf16", "int8", "e4m3"])
def test_graph_replays_match_eager_steps(kind):
    import flashattntile_b200
    from flashattntile_b200.decode_loop import DecodeLoop
    from flashattntile_b200.kernels.append import launch_append
    from flashattntile_b200.kernels.decode import launch_decode
    from flashattntile_b200.paging import PagedKVCache

    gen = torch.Generator(device=DEV).manual_seed(11)
    batch, heads, kvh, dim, ps, pages = 6, 16, 4, 128, 16, 9
    cdt = {"f16": torch.float16, "bf16": torch.bfloat16, "int8": torch.int8, "e4m3": torch.float8_e4m3fn}[kind]
    qdt = torch.bfloat16 if kind == "bf16" else torch.float16
    pool = batch * pages
    table = torch.randperm(pool, generator=gen, device=DEV).view(batch, pages).to(torch.int32)
    base = torch.randn(pool, ps, kvh, dim, generator=gen, device=DEV)
    k = base.to(cdt) if kind in ("f16", "bf16") else (base * 20).clamp(-100, 100).to(cdt)
    v = (base * 0.5).to(cdt) if kind in ("f16", "bf16") else (base * 10).clamp(-100, 100).to(cdt)
    lens = torch.tensor([0, 5, 16, 31, 70, 100], dtype=torch.int32, device=DEV)
    scales = None
    if kind in ("int8", "e4m3"):
        scales = {"k": torch.rand(pool, kvh, generator=gen, device=DEV) * 0.1 + 0.01,
                  "v": torch.rand(pool, kvh, generator=gen, device=DEV) * 0.1 + 0.01}
    cache = PagedKVCache(k, v, table, lens, ps)
    ref = _clone(cache)
    ref_scales = None if scales is None else {"k": scales["k"].clone(), "v": scales["v"].clone()}
    loop = DecodeLoop(cache, heads, scales=scales, q_dtype=qdt)
    for step in range(20):
        q = torch.randn(batch, heads, dim, generator=gen, device=DEV).to(qdt)
        nk = torch.randn(batch, kvh, dim, generator=gen, device=DEV).to(loop.in_dtype)
        nv = torch.randn(batch, kvh, dim, generator=gen, device=DEV).to(loop.in_dtype)
        got = loop.step(q, nk, nv).clone()
        launch_append(ref.k_cache, ref.v_cache, ref.page_table, ref.seq_lens, nk, nv, ps,
                      k_scale=None if ref_scales is None else ref_scales["k"],
                      v_scale=None if ref_scales is None else ref_scales["v"])
        want = launch_decode(q, ref.k_cache, ref.v_cache, ref.page_table, ref.seq_lens, ps, dim ** -0.5,
                             k_scale=None if ref_scales is None else ref_scales["k"],
                             v_scale=None if ref_scales is None else ref_scales["v"])
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"step {step}"
    assert torch.equal(cache.seq_lens, ref.seq_lens)
    assert cache.seq_lens.tolist() == [20, 25, 36, 51, 90, 120]
    assert torch.equal(cache.k_cache.view(torch.uint8), ref.k_cache.view(torch.uint8))
    assert flashattntile_b200.device_error() == 0


@pytest.mark.parametrize("kind", ["f16", "bf16", "int8", "e4m3"])
def test_graph_replays_match_oracle_every_step(kind):
    """The reference's decode loop checks each step against ``ref_attention_paged``
    on the cache as appended so far (``scripts/demo_decode_loop.py:138-145``); so
    does this one, through the CUDA-graph replays: the oracle attends over the
    appended cache (dequantised with the scales the append left, for 8-bit)."""
    import numpy as np
    from helpers import ATOL_QUANT, TAG, assert_close_f32, assert_parity_16bit, to_np

    from flashattntile_b200.decode_loop import DecodeLoop
    from flashattntile_b200.paging import PagedKVCache
    from oracle import attention as oatt
    from oracle import quant as oquant

    gen = torch.Generator(device=DEV).manual_seed(12)
    batch, heads, kvh, dim, ps, pages = 4, 16, 4, 128, 16, 8
    cdt = {"f16": torch.float16, "bf16": torch.bfloat16, "int8": torch.int8, "e4m3": torch.float8_e4m3fn}[kind]
    qdt = torch.bfloat16 if kind == "bf16" else torch.float16
    pool = batch * pages
    table = torch.randperm(pool, generator=gen, device=DEV).view(batch, pages).to(torch.int32)
    lens = torch.tensor([1, 15, 40, 90], dtype=torch.int32, device=DEV)
    scales = None
    if kind in ("f16", "bf16"):
        k = torch.randn(pool, ps, kvh, dim, generator=gen, device=DEV).to(cdt)
        v = torch.randn(pool, ps, kvh, dim, generator=gen, device=DEV).to(cdt)
    else:
        from flashattntile_b200 import quant

        mode = "int8" if kind == "int8" else "float8_e4m3fn"
        k, v, sk, sv, _ = quant.quantize_kv_pages(torch.randn(pool, ps, kvh, dim, generator=gen, device=DEV),
                                                  torch.randn(pool, ps, kvh, dim, generator=gen, device=DEV), mode)
        scales = {"k": sk, "v": sv}
    cache = PagedKVCache(k, v, table, lens, ps)
    loop = DecodeLoop(cache, heads, scales=scales, q_dtype=qdt)
    for step in range(12):
        q = torch.randn(batch, heads, dim, generator=gen, device=DEV).to(qdt)
        nk = torch.randn(batch, kvh, dim, generator=gen, device=DEV).to(loop.in_dtype)
        nv = torch.randn(batch, kvh, dim, generator=gen, device=DEV).to(loop.in_dtype)
        got = loop.step(q, nk, nv)
        torch.cuda.synchronize()
        lens_np, table_np = to_np(cache.seq_lens), to_np(cache.page_table)
        if scales is None:
            want = oatt.attention_paged(to_np(q), to_np(cache.k_cache), to_np(cache.v_cache), table_np, lens_np, ps,
                                        dtype=TAG[qdt])
            assert_parity_16bit(got, want, qdt)
        else:
            mode = "int8" if kind == "int8" else "float8_e4m3fn"
            dk, dv = oquant.dequantize_kv_pages(to_np(cache.k_cache), to_np(cache.v_cache),
                                                to_np(scales["k"]), to_np(scales["v"]), mode)
            # The reference's target: the cache dequantised to the query dtype, then the fp32 oracle.
            want = oatt.attention_paged(to_np(q), dk.astype(np.float16), dv.astype(np.float16), table_np, lens_np,
                                        ps, dtype="f16", out_f32=True)
            assert_close_f32(got, want, atol=ATOL_QUANT)
        assert lens_np.tolist() == [n + step + 1 for n in (1, 15, 40, 90)]
