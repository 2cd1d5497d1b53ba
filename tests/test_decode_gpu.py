"""Paged decode on the GPU against the oracle and the reference's golden outputs.

Covers the reference's decode test matrix (``tests/test_decode.py``,
``tests/test_kernel_correctness.py:128-195`` of FlashAttnTile): page sizes,
batches, GQA / MQA / MHA, fp16 / bf16, head dims 64 / 128 / 256, split-K
hints, INT8 / FP8 caches, tails that end inside a page, plus what the B200
kernel adds: sequences long enough to be split over every SM, NaN garbage past
the sequence end, bad page ids reported on the device, fp32-output mode.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_names, load_golden
from helpers import (ATOL_F32_MODE, ATOL_QUANT, TAG, assert_close_f32, assert_parity_16bit, from_np, paged_case,
                     to_np)

from oracle import attention as oatt
from oracle import quant as oquant

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _run(q, k, v, table, lens, ps, out_dtype=None, scale=None, k_scale=None, v_scale=None, split_k=1):
    from flashattntile_b200.kernels.decode import launch_decode

    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = launch_decode(q.to(DEV), k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), ps, scale, split_k,
                        k_scale=None if k_scale is None else k_scale.to(DEV),
                        v_scale=None if v_scale is None else v_scale.to(DEV), out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out


def _no_device_error():
    import flashattntile_b200

    assert flashattntile_b200.device_error() == 0


def _oracle(q, k, v, table, lens, ps, dtype, out_f32=False):
    return oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), ps, dtype=TAG[dtype],
                                out_f32=out_f32)


# --------------------------------------------------------------------------- golden
@pytest.mark.parametrize("name", golden_names("decode_"))
def test_decode_matches_reference_golden(name):
    c = load_golden(name)
    dtype = {"f16": torch.float16, "bf16": torch.bfloat16}[c["meta"]["dtype"]]
    ps = c["meta"]["page_size"]
    args = [from_np(c[k], dtype) for k in ("q", "k_cache", "v_cache")]
    table, lens = torch.from_numpy(c["page_table"]), torch.from_numpy(c["seq_lens"])
    out = _run(*args, table, lens, ps)
    assert out.dtype == dtype and out.shape == tuple(c["q"].shape)
    assert_parity_16bit(out, c["out"], dtype)
    out32 = _run(*args, table, lens, ps, out_dtype=torch.float32)
    assert_close_f32(out32, c["out_f32"], atol=1e-4)
    _no_device_error()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cfg1_shape_matches_reference_golden(dtype):
    """BASELINE cfg1 (fp32 in the reference) run in 16-bit against the fp32 golden output."""
    c = load_golden("cfg1_decode_f32")
    q, k, v = (torch.from_numpy(c[n]).to(dtype) for n in ("q", "k_cache", "v_cache"))
    table, lens = torch.from_numpy(c["page_table"]), torch.from_numpy(c["seq_lens"])
    out32 = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    # Same math on the 16-bit-rounded inputs in the oracle: tight.
    assert_close_f32(out32, _oracle(q, k, v, table, lens, 16, dtype, out_f32=True), atol=1e-4)
    # Against the reference's fp32 output the only difference is input rounding.
    assert_close_f32(out32, c["out"], atol=5e-2 if dtype == torch.bfloat16 else 1e-2)


# --------------------------------------------------------------------------- matrix
def _lens_for_batch(batch, page_size):
    base = [1, page_size - 1, page_size + 1, 2 * page_size + 3, 4 * page_size + 1]
    return [base[i % len(base)] for i in range(batch)]


@pytest.mark.parametrize("page_size", [16, 32])
@pytest.mark.parametrize("batch", [1, 8, 64])
@pytest.mark.parametrize("split_k", [1, 4])
def test_decode_matrix_fp16(page_size, batch, split_k):
    q, k, v, table, lens = paged_case(21, _lens_for_batch(batch, page_size), 32, 8, 128, page_size, scale=0.2)
    out = _run(q, k, v, table, lens, page_size, split_k=split_k)
    assert_parity_16bit(out, _oracle(q, k, v, table, lens, page_size, torch.float16), torch.float16)


@pytest.mark.parametrize("head_dim", [32, 64, 128, 256])
@pytest.mark.parametrize("heads,kv_heads", [(8, 8), (8, 2), (8, 1), (32, 1), (64, 8), (12, 4)])
@pytest.mark.parametrize("page_size", [8, 16, 64])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_gqa_dims_pages(head_dim, heads, kv_heads, page_size, dtype):
    lens = [1, 17, 255, 1000]
    q, k, v, table, lens = paged_case(10 + head_dim + heads, lens, heads, kv_heads, head_dim, page_size, dtype)
    out = _run(q, k, v, table, lens, page_size)
    assert_parity_16bit(out, _oracle(q, k, v, table, lens, page_size, dtype), dtype)
    out32 = _run(q, k, v, table, lens, page_size, out_dtype=torch.float32)
    assert_close_f32(out32, _oracle(q, k, v, table, lens, page_size, dtype, out_f32=True), atol=1e-4)


def test_split_hint_does_not_change_the_result():
    q, k, v, table, lens = paged_case(22, _lens_for_batch(8, 32), 32, 8, 128, 32)
    outs = [_run(q, k, v, table, lens, 32, split_k=s) for s in (1, 2, 4, 8, 64)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_more_splits_than_pages():
    q, k, v, table, lens = paged_case(24, [8, 20], 4, 2, 64, 16)
    out = _run(q, k, v, table, lens, 16, split_k=16)
    assert_parity_16bit(out, _oracle(q, k, v, table, lens, 16, torch.float16), torch.float16)


@pytest.mark.parametrize("length,kv_heads", [(131072, 1), (40000, 2), (5000, 8)])
def test_long_sequence_split_over_all_sms(length, kv_heads):
    """One unit spread over many CTAs: exercises the cross-CTA log-sum-exp merge."""
    q, k, v, table, lens = paged_case(25, [length], 8, kv_heads, 128, 64, pool_extra=0)
    out32 = _run(q, k, v, table, lens, 64, out_dtype=torch.float32)
    assert_close_f32(out32, _oracle(q, k, v, table, lens, 64, torch.float16, out_f32=True), atol=1e-4)
    _no_device_error()


def test_ragged_batch_many_units():
    gen = np.random.default_rng(3)
    lens = gen.integers(1, 3000, size=96).tolist()
    q, k, v, table, lens = paged_case(26, lens, 16, 4, 128, 16)
    out32 = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    assert_close_f32(out32, _oracle(q, k, v, table, lens, 16, torch.float16, out_f32=True), atol=1e-4)


def test_repeated_calls_reuse_the_workspace():
    q, k, v, table, lens = paged_case(27, [3000, 17, 900], 8, 2, 128, 16)
    first = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    for _ in range(5):
        assert torch.equal(_run(q, k, v, table, lens, 16, out_dtype=torch.float32), first)
    _no_device_error()


def test_workspace_is_left_zero_across_shapes():
    """Split merges across shapes share one scratch buffer; it must come back zero-filled."""
    from flashattntile_b200 import _lib

    cases = [([3000, 17, 900], 8, 2, 128, 16), ([1, 17, 255, 1000], 64, 8, 64, 8), ([20000], 8, 1, 256, 64),
             ([400] * 40, 16, 4, 64, 16)]
    for lens, h, hkv, d, ps in cases * 2:
        q, k, v, table, lens_t = paged_case(33 + d, lens, h, hkv, d, ps)
        out32 = _run(q, k, v, table, lens_t, ps, out_dtype=torch.float32)
        assert_close_f32(out32, _oracle(q, k, v, table, lens_t, ps, torch.float16, out_f32=True), atol=1e-4)
        for buf in _lib._WS.values():
            assert int(torch.count_nonzero(buf)) == 0
    _no_device_error()


def test_garbage_past_sequence_end_is_ignored():
    q, k, v, table, lens = paged_case(28, [5, 17, 33], 8, 2, 64, 16)
    clean = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    kd, vd = k.clone(), v.clone()
    for b, n in enumerate(lens.tolist()):
        last = table[b, (n - 1) // 16]
        kd[last, n % 16 or 16:] = float("nan")
        vd[last, n % 16 or 16:] = float("inf")
    dirty = _run(q, kd, vd, table, lens, 16, out_dtype=torch.float32)
    assert torch.equal(clean, dirty)


def test_zero_length_sequence_gives_zeros_without_validation():
    import flashattntile_b200 as fat

    q, k, v, table, lens = paged_case(29, [0, 9], 4, 2, 64, 16)
    with fat.value_checks(False):
        out = _run(q, k, v, table, lens, 16)
    assert torch.all(out[0] == 0)
    assert_parity_16bit(out[1:], _oracle(q[1:], k, v, table[1:], lens[1:], 16, torch.float16), torch.float16)


def test_bad_page_id_is_reported_on_device_not_faulted():
    import flashattntile_b200 as fat

    q, k, v, table, lens = paged_case(30, [20, 20], 4, 2, 64, 16)
    table[1, 0] = k.shape[0] + 5  # outside the pool: the kernel skips it
    with fat.value_checks(False):
        _run(q, k, v, table, lens, 16)
    assert fat.device_error() & 2
    assert fat.device_error() == 0  # reading clears it


# --------------------------------------------------------------------------- quantised
@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim,page_size", [(32, 8), (64, 16), (128, 32), (128, 16), (256, 64)])
def test_quantised_decode_matches_dequantised_oracle(mode, dtype, head_dim, page_size):
    lens = [1, 17, 255, 1000]
    q, k, v, table, lens = paged_case(13, lens, 8, 2, head_dim, page_size, torch.float32)
    qk, qv, sk, sv = oquant.quantize_kv_pages(k.numpy(), v.numpy(), mode)
    tdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
    qk_t, qv_t = from_np(qk, tdt), from_np(qv, tdt)
    q16 = q.to(dtype)
    out32 = _run(q16, qk_t, qv_t, table, lens, page_size, out_dtype=torch.float32,
                 k_scale=torch.from_numpy(sk), v_scale=torch.from_numpy(sv))
    dk, dv = oquant.dequantize_kv_pages(qk, qv, sk, sv, mode)
    # dequantised values rounded to the query dtype are the reference's target
    dk_t, dv_t = torch.from_numpy(dk).to(dtype), torch.from_numpy(dv).to(dtype)
    want = _oracle(q16, dk_t, dv_t, table, lens, page_size, dtype, out_f32=True)
    worst = assert_close_f32(out32, want, atol=ATOL_QUANT)
    # The kernel dequantises exactly in fp32; the only gap is the oracle's
    # rounding of the dequantised cache to 16 bits.
    assert worst <= (1.2e-2 if dtype == torch.bfloat16 else 2e-3)


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_quantised_decode_bf16_query_rows_of_extreme_magnitude(mode, head_dim):
    """8-bit caches compute in fp16 for bf16 queries too: each query row is
    scaled by a power of two into fp16's range. Rows far outside fp16's range
    (1e30, 1e-30), mixed-magnitude rows and zero rows must come out as the
    fp32 oracle on the same bf16 queries and dequantised cache does."""
    ps = 16
    lens = [33, 300, 1000]
    q, k, v, table, lens = paged_case(29, lens, 8, 2, head_dim, ps, torch.float32)
    q = q * 0.05  # keep the 1e4 row's softmax from collapsing onto one token
    gains = [1e4, 1e-6, 1e30, 1e-30, 1.0, 0.0, 3e-3, 1e2]
    for h, gain in enumerate(gains):
        q[:, h] *= gain
    q[:, 4, ::2] *= 1e3  # mixed magnitudes within one row
    qb = q.to(torch.bfloat16)
    qk, qv, sk, sv = oquant.quantize_kv_pages(k.numpy(), v.numpy(), mode)
    tdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
    out32 = _run(qb, from_np(qk, tdt), from_np(qv, tdt), table, lens, ps, out_dtype=torch.float32,
                 k_scale=torch.from_numpy(sk), v_scale=torch.from_numpy(sv))
    dk, dv = oquant.dequantize_kv_pages(qk, qv, sk, sv, mode)
    want = oatt.attention_paged(qb.float().numpy(), dk.astype(np.float32), dv.astype(np.float32), to_np(table),
                                to_np(lens), ps, dtype="f32", out_f32=True)
    assert np.isfinite(to_np(out32)).all()
    worst = assert_close_f32(out32, want, atol=ATOL_QUANT)
    assert worst <= 2e-3
    _no_device_error()


def test_quantised_op_and_golden():
    import flashattntile_b200  # noqa: F401

    for mode in ("int8", "float8_e4m3fn"):
        c = load_golden(f"quant_{mode}")
        tdt = torch.int8 if mode == "int8" else torch.float8_e4m3fn
        out = torch.ops.flashattn_tile.paged_decode_quant(
            torch.from_numpy(c["q"]).to(DEV), from_np(c["qk"], tdt).to(DEV), from_np(c["qv"], tdt).to(DEV),
            torch.from_numpy(c["scale_k"]).to(DEV), torch.from_numpy(c["scale_v"]).to(DEV),
            torch.from_numpy(c["page_table"]).to(DEV), torch.from_numpy(c["seq_lens"]).to(DEV),
            c["meta"]["page_size"], c["q"].shape[-1] ** -0.5, 1)
        assert_parity_16bit(out, c["out"], torch.float16)


# --------------------------------------------------------------------------- ops / full size
def test_custom_op_matches_oracle_and_rejects_cpu():
    import flashattntile_b200  # noqa: F401

    q, k, v, table, lens = paged_case(31, [1, 40, 77], 8, 2, 64, 16)
    out = torch.ops.flashattn_tile.paged_decode(q.to(DEV), k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), 16,
                                                0.35, 1)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), 16, scale=0.35, dtype="f16")
    assert_parity_16bit(out, want, torch.float16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.flashattn_tile.paged_decode(q, k, v, table, lens, 16, 0.35, 1)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cfg2_full_size_parity(dtype):
    """BASELINE cfg2 at full size (B32, ctx 4096, H32/8, D128, ps16) against the oracle."""
    q, k, v, table, lens = paged_case(1, [4096] * 32, 32, 8, 128, 16, dtype, pool_extra=0)
    out = _run(q, k, v, table, lens, 16)
    want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens), 16, dtype=TAG[dtype],
                                out_f32=True, threads=8)
    g = out.float().cpu().numpy()
    assert np.abs(g - want).max() <= 2e-3
    out32 = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    assert_close_f32(out32, want, atol=1e-4)
    _no_device_error()


# --------------------------------------------------------------------------- gather
def test_gather_bit_exact_golden():
    from flashattntile_b200.paging import gather_paged

    c = load_golden("gather_f16")
    args = [torch.from_numpy(c[n]).to(DEV) for n in ("k_cache", "v_cache", "page_table", "seq_lens")]
    gk, gv = gather_paged(*args, c["meta"]["page_size"])
    assert np.array_equal(to_np(gk).view(np.uint16), c["gather_k"].view(np.uint16))
    assert np.array_equal(to_np(gv).view(np.uint16), c["gather_v"].view(np.uint16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.int8, torch.float32])
def test_gather_bit_exact_random(dtype):
    from flashattntile_b200.paging import gather_paged

    from oracle import paging as opaging

    gen = torch.Generator().manual_seed(5)
    raw = torch.randint(-100, 100, (40, 8, 3, 24), generator=gen)
    k = raw.to(dtype)
    v = (raw * 2 + 1).to(dtype)
    table = torch.randperm(40, generator=gen)[:36].view(4, 9).to(torch.int32)
    lens = torch.tensor([0, 71, 8, 33], dtype=torch.int32)
    gk, gv = gather_paged(k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV), 8)
    ek, ev = opaging.gather_paged(to_np(k), to_np(v), to_np(table), to_np(lens), 8)
    assert np.array_equal(to_np(gk), ek) and np.array_equal(to_np(gv), ev)


def test_gather_rejects_out_of_pool_page():
    from flashattntile_b200.paging import gather_paged

    k = torch.zeros(4, 4, 1, 8, dtype=torch.float16, device=DEV)
    table = torch.tensor([[0, 1], [4, 2]], dtype=torch.int32, device=DEV)
    lens = torch.tensor([8, 8], dtype=torch.int32, device=DEV)
    with pytest.raises(AssertionError, match="page id outside"):
        gather_paged(k, k, table, lens, 4)


def test_f32_mode_precision_on_unit_scale_inputs():
    q, k, v, table, lens = paged_case(32, [4096, 1, 2, 3000], 32, 8, 128, 16)
    out32 = _run(q, k, v, table, lens, 16, out_dtype=torch.float32)
    assert_close_f32(out32, _oracle(q, k, v, table, lens, 16, torch.float16, out_f32=True), atol=ATOL_F32_MODE / 20)


def _torch_value_stats(lens, table, ps):
    """The torch reductions the kernel replaces (same definition of "used")."""
    big = torch.iinfo(torch.int32).max
    hi = int(lens.max())
    need = max(0, -(-hi // ps)) if hi > 0 else 0
    need = min(need, table.shape[1])
    used = table[:, :need]
    if used.numel() == 0:
        return [int(lens.min()), hi, 0, -1]
    return [int(lens.min()), hi, int(used.min()), int(used.max())]


_STATS_CASES = ["ragged", "zeros", "negative", "clamped", "strided", "wide"]


@pytest.mark.parametrize("case", _STATS_CASES)
def test_cache_value_stats_kernel_matches_torch(case):
    """fat_cache_value_stats (one kernel + 16-byte read-back) gives the statistics
    the validation checks, exactly as the torch reductions would."""
    from flashattntile_b200 import _lib

    gen = torch.Generator().manual_seed(_STATS_CASES.index(case))
    ps = 16
    if case == "wide":
        batch, max_pages = 300, 1100
    else:
        batch, max_pages = 37, 20
    table = torch.randint(-3, 5000, (batch, max_pages), generator=gen, dtype=torch.int32)
    lens = torch.randint(0, max_pages * ps, (batch,), generator=gen, dtype=torch.int32)
    if case == "zeros":
        lens.zero_()
    elif case == "negative":
        lens[5] = -7
    elif case == "clamped":
        lens[3] = max_pages * ps + 100  # past the capacity: the scan stops at the table's width
    table_d = table.to(DEV)
    if case == "strided":
        table_d = torch.randint(0, 9, (batch, 2 * max_pages), dtype=torch.int32, device=DEV)[:, ::2]
        table = table_d.cpu()
    got = _lib.cache_value_stats(lens.to(DEV), table_d, ps)
    assert got == _torch_value_stats(lens, table, ps)


@pytest.mark.parametrize("host_kind", ["pinned", "pageable"])
@pytest.mark.parametrize("scratch_offset", [0, 4])
def test_cache_value_stats_host_buffers(host_kind, scratch_offset):
    """The C ABI writes pinned (device-mapped) host memory from the kernel and
    copies into pageable memory; a device scratch that is only 4-byte aligned
    is written element by element.  Both give the torch reductions' numbers."""
    import ctypes

    from flashattntile_b200 import _lib

    gen = torch.Generator().manual_seed(77)
    batch, max_pages, ps = 41, 70, 16
    table = torch.randint(0, 9000, (batch, max_pages), generator=gen, dtype=torch.int32)
    lens = torch.randint(1, max_pages * ps, (batch,), generator=gen, dtype=torch.int32)
    want = _torch_value_stats(lens, table, ps)
    lens_d, table_d = lens.to(DEV), table.to(DEV)
    scratch = torch.zeros(8, dtype=torch.int32, device=DEV)
    if host_kind == "pinned":
        host = torch.full((4,), -99, dtype=torch.int32).pin_memory()
        host_ptr = host.data_ptr()
    else:
        host_np = np.full(4, -99, dtype=np.int32)
        host_ptr = host_np.ctypes.data
    stream = torch.cuda.current_stream()
    status = _lib.load().fat_cache_value_stats(lens_d.data_ptr(), table_d.data_ptr(), table_d.stride(0), batch,
                                               max_pages, ps, scratch.data_ptr() + scratch_offset,
                                               ctypes.c_void_p(host_ptr), stream.cuda_stream)
    assert status == 0
    stream.synchronize()
    got = host.tolist() if host_kind == "pinned" else host_np.tolist()
    assert got == want
    if host_kind == "pageable":  # the copy path went through the scratch words
        assert scratch.cpu()[scratch_offset // 4:scratch_offset // 4 + 4].tolist() == want


def test_validation_errors_raised_through_the_stats_kernel():
    """The op's value checks (reference messages) still fire with the kernel path."""
    from flashattntile_b200.paging import validate_cache

    from flashattntile_b200.paging import PagedKVCache

    _, k, v, table, lens = paged_case(41, [40, 70], 8, 2, 64, 16)
    k, v, table, lens = k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV)

    cache = PagedKVCache(k, v, table.clone(), lens.clone(), 16)
    assert validate_cache(cache) == (40, 70)
    bad = table.clone()
    bad[1, 0] = k.shape[0]
    with pytest.raises(AssertionError, match="references page"):
        validate_cache(PagedKVCache(k, v, bad, lens.clone(), 16))
    bad[1, 0] = -1
    with pytest.raises(AssertionError, match="negative page id"):
        validate_cache(PagedKVCache(k, v, bad, lens.clone(), 16))
    neg = lens.clone()
    neg[0] = -1
    with pytest.raises(AssertionError, match="non-negative"):
        validate_cache(PagedKVCache(k, v, table.clone(), neg, 16))
    over = lens.clone()
    over[0] = table.shape[1] * 16 + 1
    with pytest.raises(AssertionError, match="capacity"):
        validate_cache(PagedKVCache(k, v, table.clone(), over, 16))


@pytest.mark.parametrize("quant", [False, True])
def test_op_raises_reference_errors_with_overlapped_checks(quant):
    """The op queues the value statistics, launches, then raises the reference's
    error before returning; the kernel itself never faults on the bad metadata."""
    import flashattntile_b200
    from flashattntile_b200.kernels.decode import paged_decode_attention, paged_decode_attention_fp8
    from flashattntile_b200.paging import PagedKVCache

    q, k, v, table, lens = paged_case(43, [40, 70, 9], 8, 2, 64, 16)
    q, k, v, table, lens = q.to(DEV), k.to(DEV), v.to(DEV), table.to(DEV), lens.to(DEV)
    scales = None
    if quant:
        k, v = k.to(torch.int8), v.to(torch.int8)
        ones = torch.ones(k.shape[0], k.shape[2], device=DEV)
        scales = {"k": ones, "v": ones}

    def run(table_, lens_, q_=q):
        cache = PagedKVCache(k, v, table_, lens_, 16)
        if quant:
            return paged_decode_attention_fp8(q_, cache, scales)
        return paged_decode_attention(q_, cache)

    good = run(table, lens)
    torch.cuda.synchronize()
    bad = table.clone()
    bad[1, 2] = k.shape[0] + 5
    with pytest.raises(AssertionError, match="references page"):
        run(bad, lens)
    bad[1, 2] = -4
    with pytest.raises(AssertionError, match="negative page id"):
        run(bad, lens)
    over = lens.clone()
    over[0] = table.shape[1] * 16 + 3
    with pytest.raises(AssertionError, match="capacity"):
        run(table, over)
    zero = lens.clone()
    zero[2] = 0
    with pytest.raises(ValueError, match="at least one cached token"):
        run(table, zero)
    # A q error as well: the cache values are reported first, as in the reference.
    with pytest.raises(AssertionError, match="negative page id"):
        run(bad, lens, q[:, :, :32])
    with pytest.raises(ValueError, match="head_dim"):
        run(table, lens, q[:, :, :32])
    torch.cuda.synchronize()
    flashattntile_b200.device_error()  # the invalid launches recorded bad pages: clear the word
    again = run(table, lens)
    torch.cuda.synchronize()
    assert torch.equal(again, good)
    assert flashattntile_b200.device_error() == 0
