"""The library's own quantisation helpers (``flashattntile_b200.quant``) against
the reference's golden vectors.

``tests/golden/quant_*.npz`` hold the output of FlashAttnTile's
``quantize_kv_pages`` / ``dequantize_kv_pages`` (``flashattn_tile/quant.py:84-191``)
on seeded fp32 pages, one of them all zeros (its scale hits the 1e-8 floor).
The helpers here are what callers and the benchmark use to build INT8 / FP8
caches, so they must reproduce the reference's codes and scales bit for bit,
on the CPU and on the GPU alike.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import load_golden

from flashattntile_b200 import quant
from flashattntile_b200.paging import PagedKVCache

MODES = ["int8", "float8_e4m3fn"]
CODE_DTYPE = {"int8": torch.int8, "float8_e4m3fn": getattr(torch, "float8_e4m3fn", None)}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.uint8).numpy()


def _check_against_golden(mode: str, device: str) -> None:
    c = load_golden(f"quant_{mode}")
    k = torch.from_numpy(c["k_f32"]).to(device)
    v = torch.from_numpy(c["v_f32"]).to(device)
    qk, qv, sk, sv, info = quant.quantize_kv_pages(k, v, mode=mode)
    assert qk.dtype == CODE_DTYPE[mode] and qv.dtype == CODE_DTYPE[mode]
    assert sk.dtype == torch.float32 and tuple(sk.shape) == c["scale_k"].shape
    np.testing.assert_array_equal(sk.cpu().numpy(), c["scale_k"])
    np.testing.assert_array_equal(sv.cpu().numpy(), c["scale_v"])
    np.testing.assert_array_equal(_bits(qk), c["qk"].view(np.uint8))
    np.testing.assert_array_equal(_bits(qv), c["qv"].view(np.uint8))
    # The info dict of quant.py:131-143 (keys and values callers read).
    assert info["mode"] == mode
    assert info["granularity"] == "per_page_per_head"
    assert info["page_size"] == c["meta"]["page_size"]
    assert info["num_kv_heads"] == k.shape[2] and info["head_dim"] == k.shape[3]
    assert info["max_representable"] == (127.0 if mode == "int8" else 448.0)
    assert info["scale_min"] == pytest.approx(c["meta"]["scale_min"], rel=0, abs=0)
    assert info["rounding"] == ("round-to-nearest" if mode == "int8" else "cast-to-fp8")

    # Dequantisation: fp32 bit for bit, fp16 = the fp32 value rounded to nearest even.
    dk, dv = quant.dequantize_kv_pages(qk, qv, sk, sv, out_dtype=torch.float32)
    np.testing.assert_array_equal(dk[:3].cpu().numpy(), c["deq_k"])
    np.testing.assert_array_equal(dv[:3].cpu().numpy(), c["deq_v"])
    hk, hv = quant.dequantize_kv_pages(qk, qv, sk, sv)
    assert hk.dtype == torch.float16
    np.testing.assert_array_equal(hk[:3].cpu().numpy().view(np.uint16),
                                  c["deq_k"].astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(hv[:3].cpu().numpy().view(np.uint16),
                                  c["deq_v"].astype(np.float16).view(np.uint16))

    # The cache-level wrappers give the same codes and scales.
    table = torch.from_numpy(c["page_table"]).to(device)
    lens = torch.from_numpy(c["seq_lens"]).to(device)
    cache = PagedKVCache(k, v, table, lens, c["meta"]["page_size"])
    qcache, scales = quant.quantize_cache(cache, mode=mode)
    np.testing.assert_array_equal(_bits(qcache.k_cache), c["qk"].view(np.uint8))
    np.testing.assert_array_equal(_bits(qcache.v_cache), c["qv"].view(np.uint8))
    np.testing.assert_array_equal(scales.k.cpu().numpy(), c["scale_k"])
    assert scales.mode == mode and scales.granularity == "per_page_per_head"
    back = quant.dequantize_cache(qcache, scales, out_dtype=torch.float32)
    np.testing.assert_array_equal(back.k_cache[:3].cpu().numpy(), c["deq_k"])
    back2 = quant.dequantize_cache(qcache, scales.as_dict(), out_dtype=torch.float32)
    np.testing.assert_array_equal(back2.v_cache[:3].cpu().numpy(), c["deq_v"])
    assert back.page_table is qcache.page_table and back.page_size == cache.page_size


@pytest.mark.parametrize("mode", MODES)
def test_product_quant_helpers_match_reference_on_cpu(mode):
    if CODE_DTYPE[mode] is None:
        pytest.skip("this torch build has no float8_e4m3fn")
    _check_against_golden(mode, "cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
def test_product_quant_helpers_match_reference_on_gpu(mode, cuda_device):
    _check_against_golden(mode, str(cuda_device))


def test_quant_helper_errors_match_reference():
    k = torch.zeros(2, 16, 2, 64)
    with pytest.raises(ValueError, match="k/v shape mismatch"):
        quant.quantize_kv_pages(k, torch.zeros(2, 16, 2, 32))
    with pytest.raises(ValueError, match=r"\[num_pages, page_size, num_kv_heads, head_dim\]"):
        quant.quantize_kv_pages(k[0], k[0])
    with pytest.raises(ValueError, match="expects a float cache"):
        quant.quantize_kv_pages(k.to(torch.int8), k.to(torch.int8))
    with pytest.raises(ValueError, match="unknown quantisation mode"):
        quant.quantize_kv_pages(k, k, mode="int4")
    qk, qv, sk, sv, _ = quant.quantize_kv_pages(k, k, mode="int8")
    with pytest.raises(ValueError, match="scale_k shape"):
        quant.dequantize_kv_pages(qk, qv, sk[:1], sv)
    with pytest.raises(ValueError, match="quantised k/v shapes must match"):
        quant.dequantize_kv_pages(qk, qv[:1], sk, sv)


def test_bytes_per_token_matches_reference_accounting():
    # quant.py:194-208: K+V payload plus two fp32 scales per page and KV head, per token.
    assert quant.kv_bytes_per_token(8, 128, "fp16", 16) == 2 * 8 * 128 * 2 + 2 * 8 * 4 / 16
    assert quant.kv_bytes_per_token(8, 128, "int8", 32) == 2 * 8 * 128 + 2 * 8 * 4 / 32
