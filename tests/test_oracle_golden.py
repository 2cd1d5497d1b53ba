"""Pin the numpy oracle to the reference's own outputs (tests/golden/*.npz).

These vectors were produced by running FlashAttnTile's CPU implementation
(``reference.py``, ``paging.py``, ``quant.py``) on seeded inputs; see
``tests/golden/make_golden.py``.  fp32 results agree to float rounding
(different summation order); results stored in a 16-bit dtype agree to one
unit in the last place (two independently rounded copies of nearly equal
fp32 values); integer, code and copy results agree bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden_names, load_golden

from oracle import attention, numerics, paging, quant

F32_ATOL, F32_RTOL = 2e-6, 2e-5


def _assert_within_one_ulp(got, want, dtype):
    g = numerics.to_f32(got, dtype).astype(np.float64)
    w = numerics.to_f32(want, dtype).astype(np.float64)
    bound = numerics.ulp(w, dtype) * 1.0001
    diff = np.abs(g - w)
    assert np.all(diff <= bound), f"max diff {diff.max()} vs 1-ulp bound"
    assert np.mean(diff == 0) > 0.98, "oracle and reference disagree on too many roundings"


def test_cfg1_decode_matches_reference():
    c = load_golden("cfg1_decode_f32")
    out = attention.attention_paged(c["q"], c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"],
                                    c["meta"]["page_size"], dtype="f32")
    np.testing.assert_allclose(out, c["out"], atol=F32_ATOL, rtol=F32_RTOL)
    assert out.shape == (2, 8, 64)


@pytest.mark.parametrize("name", golden_names("decode_"))
def test_decode_cases_match_reference(name):
    c = load_golden(name)
    dt, ps = c["meta"]["dtype"], c["meta"]["page_size"]
    args = (c["q"], c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"], ps)
    out = attention.attention_paged(*args, dtype=dt)
    _assert_within_one_ulp(out, c["out"], dt)
    out32 = attention.attention_paged(*args, dtype=dt, out_f32=True)
    np.testing.assert_allclose(out32, c["out_f32"], atol=F32_ATOL, rtol=F32_RTOL)


@pytest.mark.parametrize("name", golden_names("prefill_"))
def test_prefill_cases_match_reference(name):
    c = load_golden(name)
    dt, causal = c["meta"]["dtype"], c["meta"]["causal"]
    args = (c["q"], c["k"], c["v"], c["cu_q"], c["cu_k"], causal)
    out = attention.attention_varlen(*args, dtype=dt)
    _assert_within_one_ulp(out, c["out"], dt)
    out32 = attention.attention_varlen(*args, dtype=dt, out_f32=True)
    np.testing.assert_allclose(out32, c["out_f32"], atol=F32_ATOL, rtol=F32_RTOL)
    # The thread-pool mode (the timed CPU baseline) is the same arithmetic.
    np.testing.assert_array_equal(attention.attention_varlen(*args, dtype=dt, out_f32=True, threads=3), out32)


@pytest.mark.parametrize("name", golden_names("decode_"))
def test_threaded_paged_oracle_is_bitwise_serial(name):
    c = load_golden(name)
    args = (c["q"], c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"], c["meta"]["page_size"])
    serial = attention.attention_paged(*args, dtype=c["meta"]["dtype"], out_f32=True)
    np.testing.assert_array_equal(attention.attention_paged(*args, dtype=c["meta"]["dtype"], out_f32=True,
                                                            threads=3), serial)


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
def test_quantisation_matches_reference_bit_for_bit(mode):
    c = load_golden(f"quant_{mode}")
    qk, qv, sk, sv = quant.quantize_kv_pages(c["k_f32"], c["v_f32"], mode)
    np.testing.assert_array_equal(sk, c["scale_k"])
    np.testing.assert_array_equal(sv, c["scale_v"])
    np.testing.assert_array_equal(qk.view(np.uint8), c["qk"].view(np.uint8))
    np.testing.assert_array_equal(qv.view(np.uint8), c["qv"].view(np.uint8))
    dk, dv = quant.dequantize_kv_pages(qk, qv, sk, sv, mode)
    np.testing.assert_array_equal(dk[:3], c["deq_k"])
    np.testing.assert_array_equal(dv[:3], c["deq_v"])
    assert float(sk.min()) == pytest.approx(1e-8)  # the zeroed page hits the floor


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
def test_quantised_decode_target_matches_reference(mode):
    """The quantised-decode parity target: dequantise to fp16, then the oracle."""
    c = load_golden(f"quant_{mode}")
    dk, dv = quant.dequantize_kv_pages(c["qk"], c["qv"], c["scale_k"], c["scale_v"], mode)
    dk16, dv16 = dk.astype(np.float16), dv.astype(np.float16)
    out = attention.attention_paged(c["q"], dk16, dv16, c["page_table"], c["seq_lens"],
                                    c["meta"]["page_size"], dtype="f16")
    _assert_within_one_ulp(out, c["out"], "f16")


def test_gather_bit_exact_with_zero_length_rows():
    c = load_golden("gather_f16")
    gk, gv = paging.gather_paged(c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"],
                                 c["meta"]["page_size"])
    np.testing.assert_array_equal(gk.view(np.uint16), c["gather_k"].view(np.uint16))
    np.testing.assert_array_equal(gv.view(np.uint16), c["gather_v"].view(np.uint16))


def test_append_bit_exact_through_permuted_table():
    c = load_golden("append_f16")
    steps_k, steps_v = c["steps_k"], c["steps_v"]
    batch, kvh, dim = steps_k.shape[1:]
    ps = c["meta"]["page_size"]
    table = c["page_table"].copy()
    pages = table.size
    k = np.zeros((pages, ps, kvh, dim), np.float16)
    v = np.zeros_like(k)
    lens = np.zeros(batch, np.int32)
    for t in range(steps_k.shape[0]):
        paging.append_tokens(k, v, table, lens, ps, steps_k[t], steps_v[t])
    np.testing.assert_array_equal(k.view(np.uint16), c["k_cache"].view(np.uint16))
    np.testing.assert_array_equal(v.view(np.uint16), c["v_cache"].view(np.uint16))
    np.testing.assert_array_equal(lens, c["seq_lens"])
