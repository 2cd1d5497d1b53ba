"""fat_paged_decode_noalloc: paged decode for callers that cannot allocate.

Engines that plan all device memory up front, plugins that receive no
allocator or scratch pointer, and latency-critical loops that must not risk
an allocation cannot hand fat_paged_decode a workspace.  The no-alloc entry
point runs the same kernel on a fixed 4 MiB scratch array inside the library.
This test calls it through the C ABI, twice in a row (the second call reuses
the scratch the first left behind), and compares each result with the
workspace-taking entry point's within the decode tolerance; then runs fp16,
bf16 and INT8 caches with different batch / head geometries back to back (each
call places its per-unit tickets at different offsets of the shared array),
each against the workspace entry point and the numpy oracle.  It also checks
that an oversized problem is refused on the host with a clear error.

The file name makes pytest collect it last; it passes alone in a fresh
process as well as after the other tests.
"""

from __future__ import annotations

import ctypes

import pytest
import torch
from helpers import paged_case

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _noalloc(lib, q, k, v, table, lens, ps, out, err, k_scale=None, v_scale=None):
    from flashattntile_b200 import _lib

    stream = torch.cuda.current_stream().cuda_stream
    kv_code = _lib.DTYPE_CODE[k.dtype]
    return lib.fat_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        k.shape[0], table.data_ptr(), table.stride(0), table.shape[1], lens.data_ptr(),
        None if k_scale is None else k_scale.data_ptr(), None if v_scale is None else v_scale.data_ptr(),
        0 if k_scale is None else k_scale.stride(0), out.data_ptr(), out.stride(0), out.stride(1), q.shape[0],
        q.shape[1], k.shape[2], q.shape[2], ps, _lib.DTYPE_CODE[q.dtype], kv_code, _lib.DTYPE_CODE[out.dtype],
        q.shape[-1] ** -0.5, 1, err.data_ptr(), stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.decode import launch_decode

    lib = _lib.load()
    # Long and ragged sequences: units split across many CTAs, so the merge
    # scratch is really used.
    lens = [3000, 17, 900, 20000, 1]
    q, k, v, table, lens_t = paged_case(41, lens, 16, 4, 128, 16)
    q, k, v, table, lens_t = (t.to(DEV) for t in (q, k, v, table, lens_t))
    want = launch_decode(q, k, v, table, lens_t, 16, 128 ** -0.5, 1)
    torch.cuda.synchronize()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, k, v, table, lens_t, 16, out, err)
        assert rc == _lib.FAT_OK, lib.fat_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out.float(), want.float(), atol=2e-3, rtol=0)


def test_noalloc_geometries_and_cache_types_back_to_back():
    """fp16, bf16 and INT8 caches, different batch / head layouts, one call after another."""
    import numpy as np

    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.decode import launch_decode
    from helpers import TAG, assert_parity_16bit, to_np

    from oracle import attention as oatt
    from oracle import quant as oquant

    lib = _lib.load()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    cases = [  # lens, heads, kv heads, page size, query dtype, cache kind
        ([5000, 33, 700], 32, 8, 16, torch.float16, "f16"),
        ([1, 2049, 64, 300, 4096, 17], 8, 1, 32, torch.bfloat16, "bf16"),
        ([1200, 77, 9000], 16, 4, 16, torch.float16, "int8"),
        ([2500, 128], 16, 16, 64, torch.float16, "f16"),
    ]
    for seed, (lens, h, kvh, ps, qdt, kind) in enumerate(cases):
        cache_dt = torch.float32 if kind == "int8" else qdt
        q, k, v, table, lens_t = paged_case(60 + seed, lens, h, kvh, 128, ps, cache_dt)
        q = q.to(qdt)
        ks = vs = None
        if kind == "int8":
            qk, qv, sk, sv = oquant.quantize_kv_pages(k.numpy(), v.numpy(), "int8")
            dk, dv = oquant.dequantize_kv_pages(qk, qv, sk, sv, "int8")
            k, v = torch.from_numpy(qk), torch.from_numpy(qv)
            ks, vs = torch.from_numpy(sk).to(DEV), torch.from_numpy(sv).to(DEV)
            want_np = oatt.attention_paged(to_np(q), dk.astype(np.float16), dv.astype(np.float16), to_np(table),
                                           to_np(lens_t), ps, dtype="f16", out_f32=True)
        else:
            want_np = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), ps,
                                           dtype=TAG[qdt])
        dq, dk_, dv_, dt, dl = (t.to(DEV) for t in (q, k, v, table, lens_t))
        ref = launch_decode(dq, dk_, dv_, dt, dl, ps, 128 ** -0.5, 1, k_scale=ks, v_scale=vs)
        out = torch.full_like(dq, float("nan"))
        rc = _noalloc(lib, dq, dk_, dv_, dt, dl, ps, out, err, ks, vs)
        assert rc == _lib.FAT_OK, lib.fat_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, ref), kind  # same kernel, same inputs
        if kind == "int8":
            assert np.abs(out.float().cpu().numpy() - want_np).max() <= 2e-2
        else:
            assert_parity_16bit(out, want_np, qdt)


def test_noalloc_refuses_problems_beyond_its_scratch():
    from flashattntile_b200 import _lib

    lib = _lib.load()
    need = lib.fat_paged_decode_workspace_size(torch.cuda.current_device(), 400000, 8, 8, 128)
    assert need > (4 << 20)
    dummy = ctypes.c_void_p(0)
    rc = lib.fat_paged_decode_noalloc(dummy, 0, 0, dummy, dummy, 0, 0, 0, 1, dummy, 0, 1, dummy, None, None, 0, dummy,
                                      0, 0, 400000, 8, 8, 128, 16, 0, 0, 0, 0.1, 1, None, None)
    assert rc == _lib.FAT_ERR_WORKSPACE
    assert b"4194304" in lib.fat_last_error()
