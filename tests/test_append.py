"""Quantise-on-write append: properties of the oracle restatement (CPU only).

``oracle.quant.append_tokens_quantized`` defines the semantics the CUDA kernel
must reproduce bit for bit (``tests/test_append_gpu.py``).  It has no
FlashAttnTile counterpart, so it is pinned here by properties tied to the
reference's offline format (``quant.py:84-142``).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import numerics
from oracle import quant as oquant


def _run_appends(mode, steps, batch=3, heads=2, dim=16, ps=4, seed=0, start=None):
    rng = np.random.default_rng(seed)
    pages_per_seq = (steps + (max(start) if start else 0)) // ps + 2
    pool = batch * pages_per_seq
    table = rng.permutation(pool).astype(np.int32).reshape(batch, pages_per_seq)
    qdt = np.int8 if mode == "int8" else np.uint8
    qk = np.zeros((pool, ps, heads, dim), qdt)
    qv = np.zeros_like(qk)
    sk = np.full((pool, heads), np.float32(1.0), np.float32)  # stale scales must not matter at slot 0
    sv = sk.copy()
    lens = np.array(start if start else [0] * batch, np.int32)
    tokens = []
    for t in range(steps):
        nk = (rng.standard_normal((batch, heads, dim)) * (1 + t % 3)).astype(np.float32)
        nv = (rng.standard_normal((batch, heads, dim)) * 0.5).astype(np.float32)
        tokens.append((lens.copy(), nk, nv))
        oquant.append_tokens_quantized(qk, qv, sk, sv, table, lens, nk, nv, ps, mode)
    return qk, qv, sk, sv, table, lens, tokens


def _decode(codes, mode):
    return codes.astype(np.float32) if mode == "int8" else numerics.e4m3_bits_to_f32(codes)


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
def test_single_token_pages_match_offline_quantisation(mode):
    """With one token per page (page_size 1) every append is a fresh page: the
    codes and scales equal quantize_kv_pages of that token exactly."""
    qk, qv, sk, sv, table, lens, tokens = _run_appends(mode, steps=5, ps=1)
    for pos, nk, nv in tokens:
        for b in range(nk.shape[0]):
            page = table[b, pos[b]]
            rk, rv, rsk, rsv = oquant.quantize_kv_pages(nk[b][None, None], nv[b][None, None], mode)
            np.testing.assert_array_equal(qk[page], rk[0])
            np.testing.assert_array_equal(qv[page], rv[0])
            np.testing.assert_array_equal(sk[page], rsk[0])
            np.testing.assert_array_equal(sv[page], rsv[0])


@pytest.mark.parametrize("mode", ["int8", "float8_e4m3fn"])
def test_scales_track_the_page_absmax(mode):
    max_val = oquant.INT8_MAX if mode == "int8" else oquant.FP8_MAX
    qk, qv, sk, sv, table, lens, tokens = _run_appends(mode, steps=11, ps=4)
    assert lens.tolist() == [11, 11, 11]
    for b in range(3):
        for lp in range(3):  # pages 0..2 of each sequence are complete (12 > 11 tokens: page 2 partly)
            page = table[b, lp]
            n = min(4, 11 - 4 * lp)
            for h in range(2):
                for codes, scales, idx in ((qk, sk, 1), (qv, sv, 2)):
                    x = np.stack([tokens[4 * lp + r][idx][b, h] for r in range(n)])
                    amax = np.abs(x).max()
                    s = scales[page, h]
                    # the scale covers every token of the page, and no more than the
                    # requantisation steps can have added
                    assert s >= np.float32(amax / np.float32(max_val)) * (1 - 1e-6)
                    assert s <= amax / max_val * 1.02
                    deq = _decode(codes[page, :n, h], mode) * s
                    # each requantisation may add half a step (int8) or half an e4m3
                    # ulp (2^-4 relative) of error
                    tol = (0.5 * n + 0.5) * s if mode == "int8" else 0.0625 * (n + 1) * np.abs(x) + 2 * s
                    assert np.all(np.abs(deq - x) <= tol)


def test_slot_zero_ignores_stale_page_contents():
    """A page reused by a new sequence starts from its first token only."""
    mode = "int8"
    qk = np.full((2, 4, 1, 8), 127, np.int8)  # stale codes of a previous owner
    qv = qk.copy()
    sk = np.full((2, 1), np.float32(100.0), np.float32)
    sv = sk.copy()
    table = np.array([[1, 0]], np.int32)
    lens = np.array([0], np.int32)
    nk = np.full((1, 1, 8), 0.5, np.float32)
    oquant.append_tokens_quantized(qk, qv, sk, sv, table, lens, nk, nk, 4, mode)
    assert sk[1, 0] == np.float32(np.float32(0.5) / np.float32(127.0))
    assert np.all(qk[1, 0, 0] == 127) and lens[0] == 1


def test_unchanged_scale_leaves_old_codes_alone():
    mode = "int8"
    qk = np.zeros((1, 4, 1, 4), np.int8)
    qv = qk.copy()
    sk = np.zeros((1, 1), np.float32)
    sv = sk.copy()
    table = np.array([[0]], np.int32)
    lens = np.array([0], np.int32)
    big = np.array([[[4.0, -2.0, 1.0, 0.25]]], np.float32)
    small = np.array([[[1.0, 1.0, -1.0, 0.5]]], np.float32)
    oquant.append_tokens_quantized(qk, qv, sk, sv, table, lens, big, big, 4, mode)
    before = qk[0, 0].copy()
    oquant.append_tokens_quantized(qk, qv, sk, sv, table, lens, small, small, 4, mode)
    np.testing.assert_array_equal(qk[0, 0], before)
    assert qk[0, 0, 0, 0] == 127 and lens[0] == 2
