"""Varlen prefill on the GPU against the oracle and the reference's golden outputs.

Mirrors FlashAttnTile's prefill tests (``tests/test_prefill.py``,
``tests/test_kernel_correctness.py:71-122``): ragged and odd lengths, head dims
64/128, GQA / MQA / MHA, causal and not, fp16 / bf16, a query tile longer than
the sequence, kv_len > q_len bottom-right alignment, and comparison with
torch SDPA; plus the benchmark's cfg3 shape at full size.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_names, load_golden
from helpers import TAG, assert_close_f32, assert_parity_16bit, from_np, to_np, varlen_case

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = "cuda"
ODD_LENS = [1, 17, 255, 1000]
GQA_CASES = [(8, 8), (8, 2), (8, 1)]
# The north-star bar for both 16-bit dtypes: 2e-3 max-abs in fp32-output mode,
# and within max(2e-3, 1 ulp) in the output dtype.  bf16 meets it because P
# enters P.V as a bf16 head plus remainder on every key tile holding a key that
# weighs more than 1/16 of its row so far (the default "adaptive" mode; the
# reference kernel rounds P once, prefill.py:128, which alone costs up to ~4e-3
# where a row has few keys or a few dominant ones).
F32_ATOL = {torch.float16: 2e-3, torch.bfloat16: 2e-3}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _run(q, k, v, cu_q, cu_k, causal, out_dtype=None, scale=None):
    from flashattntile_b200.kernels.prefill import launch_prefill

    scale = q.shape[-1] ** -0.5 if scale is None else scale
    qlens = (cu_q[1:] - cu_q[:-1]).tolist()
    klens = (cu_k[1:] - cu_k[:-1]).tolist()
    out = launch_prefill(q.to(DEV), k.to(DEV), v.to(DEV), cu_q.to(DEV), cu_k.to(DEV), max(qlens), max(klens),
                         causal, scale, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out


def _oracle(q, k, v, cu_q, cu_k, causal, dtype, out_f32=False):
    return oatt.attention_varlen(to_np(q), to_np(k), to_np(v), to_np(cu_q), to_np(cu_k), causal, dtype=TAG[dtype],
                                 out_f32=out_f32)


def _check(q, k, v, cu_q, cu_k, causal, dtype):
    import flashattntile_b200 as fat

    out = _run(q, k, v, cu_q, cu_k, causal)
    assert out.dtype == dtype and out.shape == q.shape
    worst16 = assert_parity_16bit(out, _oracle(q, k, v, cu_q, cu_k, causal, dtype), dtype,
                                  atol=F32_ATOL[dtype])
    out32 = _run(q, k, v, cu_q, cu_k, causal, out_dtype=torch.float32)
    worst32 = assert_close_f32(out32, _oracle(q, k, v, cu_q, cu_k, causal, dtype, out_f32=True),
                               atol=F32_ATOL[dtype])
    assert fat.device_error() == 0
    return worst16, worst32


@pytest.mark.parametrize("name", golden_names("prefill_"))
def test_prefill_matches_reference_golden(name):
    c = load_golden(name)
    dtype = {"f16": torch.float16, "bf16": torch.bfloat16}[c["meta"]["dtype"]]
    q, k, v = (from_np(c[n], dtype) for n in ("q", "k", "v"))
    cu_q, cu_k = torch.from_numpy(c["cu_q"]), torch.from_numpy(c["cu_k"])
    causal = c["meta"]["causal"]
    out = _run(q, k, v, cu_q, cu_k, causal)
    assert_parity_16bit(out, c["out"], dtype, atol=F32_ATOL[dtype])
    out32 = _run(q, k, v, cu_q, cu_k, causal, out_dtype=torch.float32)
    assert_close_f32(out32, c["out_f32"], atol=F32_ATOL[dtype])


@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("heads,kv_heads", GQA_CASES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_matrix(head_dim, heads, kv_heads, causal, dtype):
    q, k, v, cu_q, cu_k = varlen_case(7, ODD_LENS, ODD_LENS, heads, kv_heads, head_dim, dtype, scale=0.2)
    _check(q, k, v, cu_q, cu_k, causal, dtype)


@pytest.mark.parametrize("seqlen", ODD_LENS)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_single_odd_length_unit_scale(seqlen, dtype):
    q, k, v, cu_q, cu_k = varlen_case(8, [seqlen], [seqlen], 8, 2, 128, dtype)
    for causal in (True, False):
        _check(q, k, v, cu_q, cu_k, causal, dtype)


def test_prefill_kv_longer_than_q_bottom_right():
    q, k, v, cu_q, cu_k = varlen_case(9, [3, 130, 1, 40], [300, 130, 77, 400], 8, 2, 64, torch.float16)
    _check(q, k, v, cu_q, cu_k, True, torch.float16)
    _check(q, k, v, cu_q, cu_k, False, torch.float16)


def test_prefill_zero_length_sequences_in_batch():
    q, k, v, cu_q, cu_k = varlen_case(10, [5, 0, 70, 0], [5, 0, 70, 3], 4, 4, 64, torch.float16)
    _check(q, k, v, cu_q, cu_k, True, torch.float16)


@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("heads,kv_heads", GQA_CASES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_matches_sdpa(head_dim, heads, kv_heads, causal, dtype):
    gen = torch.Generator().manual_seed(9)
    batch, seqlen = 2, 255
    q = (torch.randn(batch, heads, seqlen, head_dim, generator=gen) * 0.2).to(dtype).to(DEV)
    k = (torch.randn(batch, kv_heads, seqlen, head_dim, generator=gen) * 0.2).to(dtype).to(DEV)
    v = (torch.randn(batch, kv_heads, seqlen, head_dim, generator=gen) * 0.2).to(dtype).to(DEV)
    qt = q.transpose(1, 2).reshape(batch * seqlen, heads, head_dim)
    kt = k.transpose(1, 2).reshape(batch * seqlen, kv_heads, head_dim)
    vt = v.transpose(1, 2).reshape(batch * seqlen, kv_heads, head_dim)
    cu = torch.tensor([b * seqlen for b in range(batch + 1)], dtype=torch.int32)
    out = _run(qt, kt, vt, cu, cu, causal)
    out = out.reshape(batch, seqlen, heads, head_dim).transpose(1, 2)
    g = heads // kv_heads
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.repeat_interleave(g, 1).float(), v.repeat_interleave(g, 1).float(), is_causal=causal)
    torch.testing.assert_close(out.float(), ref, atol=1e-2, rtol=1e-2)


def test_prefill_op_and_non_contiguous_views():
    import flashattntile_b200  # noqa: F401

    q, k, v, cu_q, cu_k = varlen_case(11, [33, 7], [33, 7], 8, 2, 64, torch.float16)
    qkv = torch.cat([q, k, v], dim=1).to(DEV)  # [T, 8 + 2 + 2, 64] packed projection output
    qv, kv_, vv = qkv[:, :8], qkv[:, 8:10], qkv[:, 10:12]
    out = torch.ops.flashattn_tile.prefill_varlen(qv, kv_, vv, cu_q.to(DEV), cu_k.to(DEV), 33, 33, True, 0.125)
    want = oatt.attention_varlen(to_np(q), to_np(k), to_np(v), to_np(cu_q), to_np(cu_k), True, scale=0.125,
                                 dtype="f16")
    assert_parity_16bit(out, want, torch.float16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cfg3_full_size_parity(dtype):
    """BASELINE cfg3: lens {512, 1024, 2048, 4096}, H32/8, D128, causal."""
    lens = [512, 1024, 2048, 4096]
    q, k, v, cu_q, cu_k = varlen_case(3, lens, lens, 32, 8, 128, dtype)
    out32 = _run(q, k, v, cu_q, cu_k, True, out_dtype=torch.float32)
    want = _oracle(q, k, v, cu_q, cu_k, True, dtype, out_f32=True)
    err = np.abs(out32.cpu().numpy() - want)
    assert err.max() <= F32_ATOL[dtype], f"max-abs {err.max():.3e}"
    assert err.mean() <= 2e-4


def test_prefill_head_dim_256_long_and_chunked():
    """head_dim 256 (one query tile per CTA): long causal rows and kv longer than q."""
    q, k, v, cu_q, cu_k = varlen_case(12, [1000, 129, 3], [1000, 300, 700], 8, 2, 256, torch.bfloat16, scale=0.5)
    _check(q, k, v, cu_q, cu_k, True, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_p_precision_modes(dtype):
    """"all_tiles" keeps P to ~2^-16 everywhere; "rounded" is the reference
    kernel's arithmetic (one rounding of P to the input dtype); "adaptive" splits
    only tiles holding a key that weighs > 1/16 of its row; "fp16_pv" (the bf16
    default) runs P.V in fp16 against a scaled fp16 copy of V (for fp16 inputs
    it is "rounded")."""
    from flashattntile_b200.kernels.prefill import p_precision, set_p_precision

    q, k, v, cu_q, cu_k = varlen_case(13, [700, 130, 9], [700, 130, 9], 16, 4, 128, dtype)
    want = _oracle(q, k, v, cu_q, cu_k, True, dtype, out_f32=True)
    errs, outs = {}, {}
    for mode in ("rounded", "adaptive", "all_tiles", "fp16_pv"):
        with p_precision(mode):
            out32 = _run(q, k, v, cu_q, cu_k, True, out_dtype=torch.float32)
        outs[mode] = out32
        errs[mode] = float(np.abs(out32.cpu().numpy() - want).max())
    assert errs["all_tiles"] <= 1e-4, errs
    assert errs["adaptive"] <= 1e-3, errs
    assert errs["fp16_pv"] <= 1e-3, errs
    assert errs["rounded"] <= (2e-3 if dtype == torch.float16 else 8e-3), errs
    if dtype == torch.float16:
        assert torch.equal(outs["fp16_pv"], outs["rounded"])
    assert set_p_precision("auto") == "auto"
    with pytest.raises(ValueError):
        set_p_precision("fp8")


@pytest.mark.parametrize("vscale", [1e-3, 3e5, 1e12, 1e30])
def test_fp16_pv_scales_any_bf16_range(vscale):
    """bf16 V far outside fp16's range (and tiny V) through the fp16 P.V path: the
    pre-pass scales each (sequence, KV head) by a power of two, so the result is
    the oracle's to the same relative precision as at unit scale."""
    from flashattntile_b200.kernels.prefill import p_precision

    q, k, v, cu_q, cu_k = varlen_case(14, [300, 1, 777], [300, 1, 777], 8, 2, 128, torch.bfloat16)
    v = (v.float() * vscale).to(torch.bfloat16)
    v[300:301, 1] *= 0  # a sequence whose one token has an all-zero V row on one KV head
    want = _oracle(q, k, v, cu_q, cu_k, True, torch.bfloat16, out_f32=True)
    with p_precision("fp16_pv"):
        out32 = _run(q, k, v, cu_q, cu_k, True, out_dtype=torch.float32)
    got = out32.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() <= 1e-3 * vscale * 4



@pytest.mark.parametrize("causal", [True, False])
def test_fp16_pv_keeps_finite_columns_when_v_holds_inf_or_nan(causal):
    """An inf or NaN in bf16 V leaves the other columns of its (sequence, KV head) intact on the fp16
    P.V path, as on the paths that read V directly: the pre-pass's scale comes from the largest finite
    |v| (inf and NaN convert as they are), so no finite value is flushed by a scale set for an inf.
    The non-finite outputs sit where the direct path has them; every finite one matches it."""
    from flashattntile_b200.kernels.prefill import p_precision

    q, k, v, cu_q, cu_k = varlen_case(16, [300, 257, 40], [300, 257, 40], 8, 2, 128, torch.bfloat16)
    v[150, 0, 5] = float("inf")   # sequence 0, KV head 0, column 5
    v[400, 1, 7] = float("nan")   # sequence 1, KV head 1, column 7
    outs = {}
    for mode in ("fp16_pv", "all_tiles"):
        with p_precision(mode):
            outs[mode] = _run(q, k, v, cu_q, cu_k, causal, out_dtype=torch.float32).cpu()
    a, b = outs["fp16_pv"], outs["all_tiles"]
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin)
    assert not fin.all()
    assert (a[fin] - b[fin]).abs().max().item() <= 2e-3
    # Columns other than the poisoned ones stay finite everywhere.
    assert torch.isfinite(a[:, :, [c for c in range(128) if c not in (5, 7)]]).all()


def test_fp16_pv_rejects_misaligned_v_through_the_c_abi():
    """A C caller's bf16 V that is not 16-byte aligned is refused before anything runs: the fp16 P.V
    pre-pass reads V in 16-byte vectors, and its tensor map describes the fp16 copy, not V, so the
    entry point's own alignment check is what guards it."""
    from flashattntile_b200 import _lib

    lib = _lib.load()
    q, k, v, cu_q, cu_k = (t.to(DEV) for t in varlen_case(15, [64, 40], [64, 40], 4, 2, 128, torch.bfloat16))
    vbuf = torch.zeros(v.numel() + 8, dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.fat_prefill_varlen(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), vbuf.data_ptr() + 2,
        v.stride(0), v.stride(1), out.data_ptr(), out.stride(0), out.stride(1), cu_q.data_ptr(), cu_k.data_ptr(), 2,
        q.shape[0], k.shape[0], 4, 2, 128, 64, 64, 1, 128 ** -0.5, _lib.DTYPE_CODE[torch.bfloat16],
        _lib.DTYPE_CODE[torch.bfloat16], err.data_ptr(), stream)
    assert rc == _lib.FAT_ERR_UNSUPPORTED
    assert b"16-byte" in lib.fat_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
