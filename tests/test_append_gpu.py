"""Device-side KV append (``fat_append_tokens``) against the reference and the oracle.

16-bit caches: bit-exact against the reference's own ``append_tokens`` output
(golden) and the oracle restatement.  INT8 / FP8 caches: codes, scales and
lengths bit-exact against ``oracle.quant.append_tokens_quantized`` over many
steps with ragged starting lengths (so pages fill, start fresh and get their
scales raised mid-way).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paging as opaging
from oracle import quant as oquant
from tests.conftest import load_golden
from tests.helpers import from_np, to_np

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _no_device_error():
    import flashattntile_b200

    assert flashattntile_b200.device_error() == 0


def test_append_matches_reference_golden():
    from flashattntile_b200.paging import PagedKVCache, append_tokens

    c = load_golden("append_f16")
    ps = c["meta"]["page_size"]
    steps_k, steps_v = c["steps_k"], c["steps_v"]
    pool = c["k_cache"].shape[0]
    shape = (pool, ps) + steps_k.shape[2:]
    cache = PagedKVCache(torch.zeros(shape, dtype=torch.float16, device=DEV),
                         torch.zeros(shape, dtype=torch.float16, device=DEV),
                         torch.from_numpy(c["page_table"]).to(DEV),
                         torch.zeros(steps_k.shape[1], dtype=torch.int32, device=DEV), ps)
    for t in range(steps_k.shape[0]):
        append_tokens(cache, torch.from_numpy(steps_k[t]).to(DEV), torch.from_numpy(steps_v[t]).to(DEV))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.k_cache.cpu().numpy(), c["k_cache"])
    np.testing.assert_array_equal(cache.v_cache.cpu().numpy(), c["v_cache"])
    np.testing.assert_array_equal(cache.seq_lens.cpu().numpy(), c["seq_lens"])
    _no_device_error()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim,ps", [(64, 16), (128, 8), (256, 32), (80, 16)])
def test_append_16bit_matches_oracle(dtype, dim, ps):
    from flashattntile_b200 import value_checks
    from flashattntile_b200.paging import PagedKVCache, append_tokens

    gen = torch.Generator().manual_seed(dim + ps)
    batch, kvh, steps = 5, 3, 9
    start = [0, 3, ps - 1, 2 * ps, 17]
    pages = (max(start) + steps) // ps + 1
    pool = batch * pages + 2
    table = torch.randperm(pool, generator=gen)[: batch * pages].view(batch, pages).to(torch.int32)
    k = torch.randn(pool, ps, kvh, dim, generator=gen).to(dtype)
    v = torch.randn(pool, ps, kvh, dim, generator=gen).to(dtype)
    lens = torch.tensor(start, dtype=torch.int32)
    kn, vn, ln = to_np(k).copy(), to_np(v).copy(), to_np(lens).copy()
    cache = PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps)
    for t in range(steps):
        nk = torch.randn(batch, kvh, dim, generator=gen).to(dtype)
        nv = torch.randn(batch, kvh, dim, generator=gen).to(dtype)
        with value_checks(t % 2 == 0):  # both the checked and the sync-free path
            append_tokens(cache, nk.to(DEV), nv.to(DEV))
        opaging.append_tokens(kn, vn, to_np(table), ln, ps, to_np(nk), to_np(nv))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(cache.k_cache), kn)
    np.testing.assert_array_equal(to_np(cache.v_cache), vn)
    np.testing.assert_array_equal(to_np(cache.seq_lens), ln)
    _no_device_error()


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("dim,ps", [(128, 16), (64, 32), (96, 8)])
def test_quantised_append_matches_oracle(mode, in_dtype, dim, ps):
    from flashattntile_b200 import value_checks
    from flashattntile_b200.paging import PagedKVCache
    from flashattntile_b200.quant import QuantScales, append_tokens_quantized

    gen = torch.Generator().manual_seed(7 * dim + ps)
    batch, kvh, steps = 4, 2, 2 * ps + 3
    start = [0, 1, ps - 1, ps + 5]
    pages = (max(start) + steps) // ps + 1
    pool = batch * pages + 3
    table = torch.randperm(pool, generator=gen)[: batch * pages].view(batch, pages).to(torch.int32)
    # Pre-existing content: quantise a random float cache offline (reference format).
    base = torch.randn(pool, ps, kvh, dim, generator=gen)
    qk, qv, sk, sv = oquant.quantize_kv_pages(base.numpy(), (base * 0.5).numpy(), mode)
    tdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
    lens = np.array(start, np.int32)
    cache = PagedKVCache(from_np(qk, tdt).to(DEV), from_np(qv, tdt).to(DEV), table.to(DEV),
                         torch.from_numpy(lens.copy()).to(DEV), ps)
    scales = QuantScales(torch.from_numpy(sk.copy()).to(DEV), torch.from_numpy(sv.copy()).to(DEV), mode)
    for t in range(steps):
        amp = float(1 + (t % 4))  # some steps raise the page scale, others do not
        nk = (torch.randn(batch, kvh, dim, generator=gen) * amp).to(in_dtype)
        nv = (torch.randn(batch, kvh, dim, generator=gen) * 0.25).to(in_dtype)
        with value_checks(t % 2 == 1):
            append_tokens_quantized(cache, scales, nk.to(DEV), nv.to(DEV))
        oquant.append_tokens_quantized(qk, qv, sk, sv, to_np(table), lens, nk.float().numpy(), nv.float().numpy(),
                                       ps, mode)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(cache.k_cache), qk)
    np.testing.assert_array_equal(to_np(cache.v_cache), qv)
    np.testing.assert_array_equal(scales.k.cpu().numpy(), sk)
    np.testing.assert_array_equal(scales.v.cpu().numpy(), sv)
    np.testing.assert_array_equal(to_np(cache.seq_lens), lens)
    _no_device_error()


def test_bad_page_is_skipped_and_reported():
    """With value checks off, a sequence at capacity or mapped to a page outside
    the pool is left untouched and FAT_DEVERR_BAD_PAGE is recorded; the others
    are appended."""
    import flashattntile_b200
    from flashattntile_b200 import value_checks
    from flashattntile_b200.paging import PagedKVCache, append_tokens

    ps, kvh, dim = 8, 2, 64
    table = torch.tensor([[0, 1], [2, 3], [4, 99]], dtype=torch.int32)
    lens = torch.tensor([3, 16, 8], dtype=torch.int32)  # seq 1 at capacity, seq 2 lands on page 99
    k = torch.zeros(6, ps, kvh, dim, dtype=torch.float16)
    cache = PagedKVCache(k.to(DEV), k.clone().to(DEV), table.to(DEV), lens.to(DEV), ps)
    nk = torch.ones(3, kvh, dim, dtype=torch.float16, device=DEV)
    with value_checks(False):
        append_tokens(cache, nk, nk * 2)
    torch.cuda.synchronize()
    assert cache.seq_lens.cpu().tolist() == [4, 16, 8]
    assert float(cache.k_cache[0, 3].float().mean()) == 1.0 and float(cache.v_cache[0, 3].float().mean()) == 2.0
    assert float(cache.k_cache.float().abs().sum()) == float(kvh * dim)  # nothing else written
    assert flashattntile_b200.device_error() & 2
    with pytest.raises(AssertionError, match="capacity"):
        append_tokens(cache, nk, nk)


def test_appended_quantised_cache_decodes_like_its_dequantised_copy():
    """Decode after on-device appends equals decode over the dequantised cache."""
    from flashattntile_b200.kernels.decode import launch_decode
    from flashattntile_b200.paging import PagedKVCache
    from flashattntile_b200.quant import QuantScales, append_tokens_quantized, dequantize_kv_pages

    gen = torch.Generator().manual_seed(3)
    batch, heads, kvh, dim, ps = 3, 8, 2, 128, 16
    pages = 6
    table = torch.randperm(batch * pages, generator=gen).view(batch, pages).to(torch.int32).to(DEV)
    q = torch.randn(batch, heads, dim, generator=gen).half().to(DEV)
    cache = PagedKVCache(torch.zeros(batch * pages, ps, kvh, dim, dtype=torch.int8, device=DEV),
                         torch.zeros(batch * pages, ps, kvh, dim, dtype=torch.int8, device=DEV), table,
                         torch.zeros(batch, dtype=torch.int32, device=DEV), ps)
    scales = QuantScales(torch.ones(batch * pages, kvh, device=DEV), torch.ones(batch * pages, kvh, device=DEV), "int8")
    for _ in range(70):
        append_tokens_quantized(cache, scales, torch.randn(batch, kvh, dim, generator=gen).half().to(DEV),
                                torch.randn(batch, kvh, dim, generator=gen).half().to(DEV))
    out = launch_decode(q, cache.k_cache, cache.v_cache, table, cache.seq_lens, ps, dim ** -0.5,
                        k_scale=scales.k, v_scale=scales.v, out_dtype=torch.float32)
    dk, dv = dequantize_kv_pages(cache.k_cache, cache.v_cache, scales.k, scales.v, out_dtype=torch.float32)
    want = launch_decode(q.float().half(), dk.half(), dv.half(), table, cache.seq_lens, ps, dim ** -0.5,
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float((out - want).abs().max()) < 2e-2
