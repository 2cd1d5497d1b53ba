"""Seeded input builders and parity checks shared by the tests.

Inputs are drawn on the CPU with ``torch.Generator`` so the numpy oracle and
the CUDA kernels see identical values; ``to_np`` hands the oracle raw storage
(bf16 as uint16 bit patterns, e4m3 as uint8 codes).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import numerics

TAG = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}
# Parity bar for 16-bit outputs: 2e-3 max-abs, or one unit in the last place of
# the output dtype where |out| is large enough that a single rounding step of
# two independently rounded results exceeds 2e-3 (bf16 above |x| = 0.25).
ATOL_16BIT = 2e-3
ATOL_F32_MODE = 2e-3
ATOL_QUANT = 2e-2


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if hasattr(torch, "float8_e4m3fn") and t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def from_np(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    if hasattr(torch, "float8_e4m3fn") and dtype == torch.float8_e4m3fn:
        return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)


def paged_case(seed, lens, heads, kv_heads, dim, page_size, dtype=torch.float16, pool_extra=3, scale=1.0):
    """q [B,H,D], K/V pool, permuted page table, seq_lens -- all CPU tensors."""
    gen = torch.Generator().manual_seed(seed)
    batch = len(lens)
    max_pages = max(1, math.ceil(max(lens) / page_size))
    pool = batch * max_pages + pool_extra
    k = (torch.randn(pool, page_size, kv_heads, dim, generator=gen) * scale).to(dtype)
    v = (torch.randn(pool, page_size, kv_heads, dim, generator=gen) * scale).to(dtype)
    q = (torch.randn(batch, heads, dim, generator=gen) * scale).to(dtype)
    table = torch.randperm(pool, generator=gen)[: batch * max_pages].view(batch, max_pages).to(torch.int32)
    return q, k, v, table, torch.tensor(lens, dtype=torch.int32)


def varlen_case(seed, q_lens, kv_lens, heads, kv_heads, dim, dtype=torch.float16, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(sum(q_lens), heads, dim, generator=gen) * scale).to(dtype)
    k = (torch.randn(sum(kv_lens), kv_heads, dim, generator=gen) * scale).to(dtype)
    v = (torch.randn(sum(kv_lens), kv_heads, dim, generator=gen) * scale).to(dtype)
    cu_q = torch.tensor([0] + np.cumsum(q_lens).tolist(), dtype=torch.int32)
    cu_k = torch.tensor([0] + np.cumsum(kv_lens).tolist(), dtype=torch.int32)
    return q, k, v, cu_q, cu_k


def assert_parity_16bit(got: torch.Tensor, want_storage: np.ndarray, dtype: torch.dtype, atol=ATOL_16BIT):
    """``got`` (kernel, 16-bit) against the oracle/reference output of the same dtype."""
    tag = TAG[dtype]
    g = got.detach().float().cpu().numpy().astype(np.float64)
    w = numerics.to_f32(want_storage, tag).astype(np.float64)
    assert np.isfinite(g).all(), "kernel produced non-finite values"
    bound = np.maximum(atol, numerics.ulp(w, tag) * 1.0001)
    diff = np.abs(g - w)
    worst = float(diff.max()) if diff.size else 0.0
    assert np.all(diff <= bound), f"max-abs {worst:.3e} exceeds max(2e-3, 1 ulp)"
    return worst


def assert_close_f32(got: torch.Tensor, want: np.ndarray, atol=ATOL_F32_MODE):
    g = got.detach().float().cpu().numpy()
    assert np.isfinite(g).all(), "kernel produced non-finite values"
    worst = float(np.abs(g - want).max()) if g.size else 0.0
    assert worst <= atol, f"max-abs {worst:.3e} > {atol}"
    return worst
