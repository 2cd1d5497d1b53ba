"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every pipeline wait in the decode and prefill kernels gives up after a time
limit, records FAT_DEVERR_TIMEOUT in the caller's error word, raises the
CTA's abort flag, drains its own TMA copies and tensor-core work, frees its
tensor memory and returns.  These tests shorten the limit
(``fat_set_wait_limit_ns``) and ask the next launch to wait once on a barrier
phase that nothing completes (``fat_expire_next_waits``), then check that

* the launch returns with the TIMEOUT bit set and the context stays usable;
* the next call on the same stream, with the default limit back, is correct
  (against the oracle) and reports no error.

Nothing here faults, traps or hangs the GPU: the only wait that cannot end by
itself is bounded by the limit set below.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import TAG, assert_close_f32, paged_case, to_np, varlen_case

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = "cuda"
LIMIT_NS = 20_000_000  # 20 ms: far above any wait of these small launches, short for the test


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture()
def lib():
    from flashattntile_b200 import _lib

    lib = _lib.load()
    yield lib
    lib.fat_expire_next_waits(0)
    lib.fat_set_wait_limit_ns(0)


def _expire_one(lib, fn):
    """Run fn() with one expiring wait and a short limit; returns the error word."""
    from flashattntile_b200 import _lib

    dev = torch.device(DEV, torch.cuda.current_device())
    assert _lib.read_device_error(dev) == 0
    lib.fat_set_wait_limit_ns(LIMIT_NS)
    lib.fat_expire_next_waits(1)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        lib.fat_expire_next_waits(0)
        lib.fat_set_wait_limit_ns(0)
    return _lib.read_device_error(dev)  # also resets this stream's scratch


def test_set_wait_limit_returns_previous(lib):
    assert lib.fat_set_wait_limit_ns(123) == 2_000_000_000
    assert lib.fat_set_wait_limit_ns(0) == 123
    assert lib.fat_set_wait_limit_ns(0) == 2_000_000_000


@pytest.mark.parametrize("dtype", [torch.float16, torch.int8])
def test_decode_wait_runs_out_and_next_call_is_clean(lib, dtype):
    from flashattntile_b200 import _lib, quant
    from flashattntile_b200.kernels.decode import launch_decode

    lens = [3000, 17, 900, 5000]
    q, k, v, table, sl = paged_case(71, lens, 16, 4, 128, 16)
    ks = vs = None
    kf, vf = k.float(), v.float()
    if dtype == torch.int8:
        k, v, ks, vs, _ = quant.quantize_kv_pages(kf, vf, mode="int8")
        kf, vf = quant.dequantize_kv_pages(k, v, ks, vs, out_dtype=torch.float32)
    args = [t.to(DEV) for t in (q, k, v, table, sl)]
    extra = {} if ks is None else {"k_scale": ks.to(DEV), "v_scale": vs.to(DEV)}

    word = _expire_one(lib, lambda: launch_decode(*args, 16, 128 ** -0.5, 1, **extra))
    assert word & _lib.FAT_DEVERR_TIMEOUT, word

    out = launch_decode(*args, 16, 128 ** -0.5, 1, out_dtype=torch.float32, **extra)
    torch.cuda.synchronize()
    dev = torch.device(DEV, torch.cuda.current_device())
    assert _lib.read_device_error(dev) == 0
    want = oatt.attention_paged(to_np(q).astype(np.float32), kf.numpy(), vf.numpy(), to_np(table), to_np(sl), 16,
                                dtype="f32", out_f32=True)
    assert_close_f32(out, want, atol=1e-3)


@pytest.mark.parametrize("paged", [False, True])
def test_prefill_wait_runs_out_and_next_call_is_clean(lib, paged):
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.prefill import launch_prefill, prefill_paged_attention
    from flashattntile_b200.paging import PagedKVCache

    lens = [300, 1000]
    q, k, v, cu_q, cu_k = varlen_case(72, lens, lens, 8, 2, 128)
    d = [t.to(DEV) for t in (q, k, v, cu_q, cu_k)]
    if paged:
        ps = 16
        pages = [(n + ps - 1) // ps for n in lens]
        kc = torch.zeros(sum(pages), ps, 2, 128, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        table = torch.zeros(len(lens), max(pages), dtype=torch.int32)
        p0, t0 = 0, 0
        for b, n in enumerate(lens):
            for t in range(n):
                kc[p0 + t // ps, t % ps] = k[t0 + t]
                vc[p0 + t // ps, t % ps] = v[t0 + t]
            table[b, :pages[b]] = torch.arange(p0, p0 + pages[b], dtype=torch.int32)
            p0, t0 = p0 + pages[b], t0 + n
        cache = PagedKVCache(kc.to(DEV), vc.to(DEV), table.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
                             ps)

        def call(out_dtype=None):
            from flashattntile_b200 import value_checks

            with value_checks(False):
                return prefill_paged_attention(d[0], cache, d[3], max(lens), causal=True, out_dtype=out_dtype)
    else:
        def call(out_dtype=None):
            return launch_prefill(*d, max(lens), max(lens), True, 128 ** -0.5, out_dtype=out_dtype)

    word = _expire_one(lib, call)
    assert word & _lib.FAT_DEVERR_TIMEOUT, word

    out = call(out_dtype=torch.float32)
    torch.cuda.synchronize()
    dev = torch.device(DEV, torch.cuda.current_device())
    assert _lib.read_device_error(dev) == 0
    want = oatt.attention_varlen(to_np(q), to_np(k), to_np(v), to_np(cu_q), to_np(cu_k), True, dtype=TAG[q.dtype],
                                 out_f32=True)
    assert_close_f32(out, want, atol=2e-3)
