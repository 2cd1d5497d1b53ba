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
