"""The decode op's fast path: repeated calls with the same tensors.

After a call has passed every structural check, the op keeps its argument
struct keyed by the tensors' storage, shapes, strides, dtypes and the stream;
later calls with an equal key skip the checks and the argument packing but
still run the value checks on every call (the reference checks ``seq_lens`` and
``page_table`` values each time).  These tests check that

* fast calls give bit-identical results to the first (checked) call and
  follow new values written in place into q, the page table and the lengths;
* a bad value written in place is still caught, with the reference's message;
* anything that changes the key (a different q tensor, another stream) takes
  the full path, and a reallocated scratch buffer is never used stale.
"""

from __future__ import annotations

import pytest
import torch
from helpers import assert_parity_16bit, paged_case, to_np

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _case(seed=61):
    q, k, v, table, lens = paged_case(seed, [700, 33, 2000], 16, 4, 128, 16)
    return [t.to(DEV) for t in (q, k, v, table, lens)], (q, k, v, table, lens)


def test_fast_calls_match_checked_call_and_follow_in_place_updates():
    from flashattntile_b200.kernels import decode as kd

    (q, k, v, table, lens), host = _case()
    op = torch.ops.flashattn_tile.paged_decode
    kd._FAST.clear()
    first = op(q, k, v, table, lens, 16, 0.09, 1)
    assert len(kd._FAST) == 1
    for _ in range(3):
        again = op(q, k, v, table, lens, 16, 0.09, 1)
        assert torch.equal(again, first)
    # New values in place (same storage): the fast path reads them.
    q.mul_(0.5)
    lens[1] = 17
    out = op(q, k, v, table, lens, 16, 0.09, 1)
    torch.cuda.synchronize()
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), 16, scale=0.09, dtype="f16")
    assert_parity_16bit(out, want, torch.float16)
    assert len(kd._FAST) == 1


def test_fast_path_still_runs_the_value_checks():
    from flashattntile_b200.kernels import decode as kd

    (q, k, v, table, lens), _ = _case(62)
    op = torch.ops.flashattn_tile.paged_decode
    op(q, k, v, table, lens, 16, 0.09, 1)
    assert len(kd._FAST) >= 1
    capacity = table.shape[1] * 16
    lens[0] = capacity + 1
    with pytest.raises(AssertionError, match="exceeds page-table capacity"):
        op(q, k, v, table, lens, 16, 0.09, 1)
    lens[0] = 700
    table[2, 0] = k.shape[0] + 5
    with pytest.raises(AssertionError, match="references page"):
        op(q, k, v, table, lens, 16, 0.09, 1)
    table[2, 0] = 0
    lens[1] = 0
    with pytest.raises(ValueError, match="at least one cached token"):
        op(q, k, v, table, lens, 16, 0.09, 1)
    import flashattntile_b200

    flashattntile_b200.device_error()  # clear what the bad calls recorded


def test_key_changes_take_the_full_path():
    from flashattntile_b200.kernels import decode as kd

    (q, k, v, table, lens), _ = _case(63)
    op = torch.ops.flashattn_tile.paged_decode
    kd._FAST.clear()
    a = op(q, k, v, table, lens, 16, 0.09, 1)
    q2 = q.clone()
    b = op(q2, k, v, table, lens, 16, 0.09, 1)  # another q tensor: a second entry
    assert torch.equal(a, b) and len(kd._FAST) == 2
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        c = op(q, k, v, table, lens, 16, 0.09, 1)  # another stream: its own scratch and entry
    side.synchronize()
    assert torch.equal(a, c) and len(kd._FAST) == 3
    # A bigger problem on the same stream grows (reallocates) the scratch buffer;
    # the earlier entry must notice and fall back instead of using the old buffer.
    (q3, k3, v3, t3, l3), _ = _case(64)
    big_q = torch.randn(512, 16, 128, device=DEV).half()
    big_t = torch.zeros(512, t3.shape[1], dtype=torch.int32, device=DEV)
    big_l = torch.full((512,), 16, dtype=torch.int32, device=DEV)
    op(big_q, k3, v3, big_t, big_l, 16, 0.09, 1)
    d = op(q, k, v, table, lens, 16, 0.09, 1)
    assert torch.equal(a, d)


def test_quant_op_fast_path():
    from flashattntile_b200 import quant
    from flashattntile_b200.kernels import decode as kd

    (q, k, v, table, lens), _ = _case(65)
    kq, vq, ks, vs, _ = quant.quantize_kv_pages(k.float(), v.float(), mode="int8")
    op = torch.ops.flashattn_tile.paged_decode_quant
    kd._FAST.clear()
    first = op(q, kq, vq, ks, vs, table, lens, 16, 0.09, 1)
    assert len(kd._FAST) == 1
    assert torch.equal(op(q, kq, vq, ks, vs, table, lens, 16, 0.09, 1), first)
    ks.mul_(2.0)  # new scale values in place: followed
    changed = op(q, kq, vq, ks, vs, table, lens, 16, 0.09, 1)
    assert not torch.equal(changed, first)
