"""Prefill's two grids give bitwise-identical outputs, and the persistent one matches the oracle.

The persistent grid (one CTA per SM claiming (head, sequence, query-pair)
items from a per-stream counter, with ring positions and barrier phases carried
across items) and the per-item grid run the same per-item arithmetic, so every
output element must agree bit for bit.  The cases cover many items per CTA,
many sequences (the claim cursor's sequence scan crosses several 32-lane
chunks), ragged and one-token sequences, q_len != kv_len, GQA / MQA, head_dim
64 / 128 / 256, every precision of P, the paged-K/V kernel, and launches
alternating between two streams (each with its own counters).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import TAG, assert_close_f32, to_np, varlen_case

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _both(fn):
    """fn() under each grid; every launch must also leave the device error word clear."""
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.prefill import schedule

    dev = torch.device(DEV, torch.cuda.current_device())
    assert _lib.read_device_error(dev) == 0
    outs = {}
    for mode in ("persistent", "per_item"):
        with schedule(mode):
            outs[mode] = fn()
            torch.cuda.synchronize()
        assert _lib.read_device_error(dev) == 0, mode
    return outs["persistent"], outs["per_item"]


def _packed(q, k, v, cu_q, cu_k, causal, out_dtype=None):
    from flashattntile_b200.kernels.prefill import launch_prefill

    dq, dk, dv, dcq, dck = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    mq = int((cu_q[1:] - cu_q[:-1]).max())
    mk = int((cu_k[1:] - cu_k[:-1]).max())
    return lambda: launch_prefill(dq, dk, dv, dcq, dck, mq, mk, causal, q.shape[-1] ** -0.5, out_dtype=out_dtype)


CASES = [
    # q_lens, kv_lens, heads, kv_heads, dim
    ([512, 1024, 2048, 4096], None, 32, 8, 128),                 # the benchmark's cfg3 shape
    (list(range(1, 700, 7)), None, 8, 2, 128),                   # 100 ragged sequences, 1..694 tokens
    ([1, 300, 1, 257, 4000, 129], [5, 900, 1, 257, 4100, 200], 16, 1, 128),  # kv > q, MQA
    ([300, 777, 64], None, 8, 8, 64),                            # MHA, head_dim 64
    ([300, 129, 600], [300, 400, 600], 4, 2, 256),               # head_dim 256: one tile per CTA
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [True, False])
def test_schedules_bitwise_equal(case, dtype, causal):
    q_lens, kv_lens, h, kvh, d = CASES[case]
    kv_lens = kv_lens or q_lens
    q, k, v, cu_q, cu_k = varlen_case(300 + case, q_lens, kv_lens, h, kvh, d, dtype)
    a, b = _both(_packed(q, k, v, cu_q, cu_k, causal))
    assert torch.equal(a, b)
    a32, b32 = _both(_packed(q, k, v, cu_q, cu_k, causal, out_dtype=torch.float32))
    assert torch.equal(a32, b32)


@pytest.mark.parametrize("mode", ["rounded", "adaptive", "all_tiles", "fp16_pv"])
def test_schedules_bitwise_equal_for_every_p_precision(mode):
    from flashattntile_b200.kernels.prefill import p_precision

    q, k, v, cu_q, cu_k = varlen_case(310, [700, 33, 2000, 1], [700, 33, 2000, 1], 16, 4, 128, torch.bfloat16)
    with p_precision(mode):
        a, b = _both(_packed(q, k, v, cu_q, cu_k, True, out_dtype=torch.float32))
    assert torch.equal(a, b)


def test_persistent_many_items_per_cta_matches_oracle():
    """Thirty-odd items per CTA on 148 SMs, against the fp32 oracle on sampled sequences."""
    from flashattntile_b200.kernels.prefill import schedule

    lens = [int(x) for x in np.random.default_rng(5).integers(1, 1500, size=150)]
    q, k, v, cu_q, cu_k = varlen_case(311, lens, lens, 32, 8, 128, torch.float16)
    with schedule("persistent"):
        out = _packed(q, k, v, cu_q, cu_k, True, out_dtype=torch.float32)()
        torch.cuda.synchronize()
    cq = cu_q.tolist()
    for b in (0, 1, 77, 149):
        s0, s1 = cq[b], cq[b + 1]
        want = oatt.attention_varlen(to_np(q[s0:s1]), to_np(k[s0:s1]), to_np(v[s0:s1]),
                                     np.array([0, s1 - s0], np.int32), np.array([0, s1 - s0], np.int32), True,
                                     dtype=TAG[torch.float16], out_f32=True)
        assert_close_f32(out[s0:s1], want)


@pytest.mark.parametrize("ps", [16, 128])
def test_paged_schedules_bitwise_equal(ps):
    from flashattntile_b200.kernels.prefill import prefill_paged_attention
    from flashattntile_b200.paging import PagedKVCache
    from tests.test_prefill_paged_gpu import _case

    kv_lens, q_lens = [1000, 257, 64, 3000], [50, 257, 1, 3000]
    q, k, v, table, lens, cu_q = _case(320, kv_lens, q_lens, 8, 2, 128, ps, torch.bfloat16, nan_pool=True)
    cache = PagedKVCache(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps)
    dq, dcq = q.to(DEV), cu_q.to(DEV)
    a, b = _both(lambda: prefill_paged_attention(dq, cache, dcq, max(q_lens), causal=True))
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)


def test_persistent_launches_on_two_streams():
    """Each stream's counters are zeroed again by its launch's last CTA."""
    q, k, v, cu_q, cu_k = varlen_case(312, [900, 2000, 17], [900, 2000, 17], 16, 4, 128, torch.float16)
    run = _packed(q, k, v, cu_q, cu_k, True)
    want = run()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    outs = []
    for i in range(6):
        if i % 2:
            with torch.cuda.stream(side):
                outs.append(run())
            torch.cuda.current_stream().wait_stream(side)
        else:
            outs.append(run())
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)


def test_schedule_switch_rejects_unknown_modes():
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.prefill import set_schedule

    with pytest.raises(ValueError):
        set_schedule("dynamic")
    lib = _lib.load()
    assert lib.fat_set_prefill_schedule(7) == -2
    assert lib.fat_set_prefill_schedule(0) in (0, 1)
