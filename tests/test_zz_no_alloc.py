"""fat_paged_decode_noalloc: paged decode for callers that cannot allocate.

Engines that plan all device memory up front, plugins that receive no
allocator or scratch pointer, and latency-critical loops that must not risk
an allocation cannot hand fat_paged_decode a workspace.  The no-alloc entry
point runs the same kernel on a fixed 4 MiB scratch array inside the library.
This test calls it through the C ABI, twice in a row (the second call reuses
the scratch the first left behind), and compares each result with the
workspace-taking entry point's within the decode tolerance.  It also checks
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


def _noalloc(lib, q, k, v, table, lens, ps, out, err):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.fat_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        k.shape[0], table.data_ptr(), table.stride(0), table.shape[1], lens.data_ptr(), None, None, 0,
        out.data_ptr(), out.stride(0), out.stride(1), q.shape[0], q.shape[1], k.shape[2], q.shape[2], ps, 0, 0, 0,
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
