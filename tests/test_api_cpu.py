"""Host-side behaviour of the drop-in surface, on the CPU (no kernels launched).

Mirrors the reference's own host-side tests (``tests/test_ops.py``,
``tests/test_paging.py``, ``tests/test_decode.py``, ``tests/test_prefill.py``,
``tests/test_autotune.py``): op registration and schemas, fake-tensor shapes,
``torch.compile(fullgraph=True)`` without graph breaks, backend geometry and
validation, and the validation errors (types and messages) callers match on.
Results are checked on the GPU (``*_gpu.py``); here nothing reaches a kernel.
"""

from __future__ import annotations

import pytest
import torch

import flashattntile_b200  # noqa: F401  (registers the ops)
from flashattntile_b200 import autotune as at
from flashattntile_b200.backend import AttentionMetadata, FlashAttnTileBackend
from flashattntile_b200.kernels.decode import HAS_TRITON as DECODE_HAS_TRITON
from flashattntile_b200.kernels.decode import paged_decode_attention
from flashattntile_b200.kernels.prefill import HAS_TRITON as PREFILL_HAS_TRITON
from flashattntile_b200.kernels.prefill import prefill_attention
from flashattntile_b200.ops import PAGED_DECODE_OP, PREFILL_OP, ops_available
from flashattntile_b200.paging import PagedKVCache, allocate, append_tokens, validate_cache


def _cpu_cache(batch=2, lens=(5, 9), ps=16, kvh=2, dim=16, dtype=torch.float16):
    pages = max(1, -(-max(lens) // ps))
    k = torch.randn(batch * pages, ps, kvh, dim).to(dtype)
    table = torch.arange(batch * pages, dtype=torch.int32).view(batch, pages)
    return PagedKVCache(k, k.clone(), table, torch.tensor(lens, dtype=torch.int32), ps)


# --------------------------------------------------------------------------- ops
def test_custom_ops_registered_with_reference_schemas():
    assert ops_available()
    assert PAGED_DECODE_OP in str(torch.ops.flashattn_tile.paged_decode._schemas)
    assert PREFILL_OP in str(torch.ops.flashattn_tile.prefill_varlen._schemas)
    assert hasattr(torch.ops.flashattn_tile, "paged_decode_quant")


def test_fake_shapes():
    with torch._subclasses.fake_tensor.FakeTensorMode():
        q = torch.empty(3, 4, 8, device="meta")
        k = torch.empty(12, 16, 2, 8, device="meta")
        pt = torch.empty(3, 3, dtype=torch.int32, device="meta")
        sl = torch.full((3,), 5, dtype=torch.int32, device="meta")
        out = torch.ops.flashattn_tile.paged_decode(q, k, k, pt, sl, 16, 0.35, 1)
        assert out.shape == (3, 4, 8) and out.dtype == torch.float32
        qp = torch.empty(11, 4, 8, device="meta")
        kp = torch.empty(11, 2, 8, device="meta")
        cu = torch.zeros(3, dtype=torch.int32, device="meta")
        outp = torch.ops.flashattn_tile.prefill_varlen(qp, kp, kp, cu, cu, 7, 7, True, 0.35)
        assert outp.shape == (11, 4, 8)


def test_compile_fullgraph_has_zero_graph_breaks():
    k = torch.empty(12, 16, 2, 8, dtype=torch.float16, device="meta")
    pt = torch.empty(2, 6, dtype=torch.int32, device="meta")
    sl = torch.empty(2, dtype=torch.int32, device="meta")
    kp = torch.empty(9, 2, 8, dtype=torch.float16, device="meta")
    cu = torch.empty(3, dtype=torch.int32, device="meta")

    def decode(x):
        return torch.ops.flashattn_tile.paged_decode(x, k, k, pt, sl, 16, 0.35, 1) * 2

    def prefill(x):
        return torch.ops.flashattn_tile.prefill_varlen(x, kp, kp, cu, cu, 6, 6, True, 0.35) + 1

    for fn, x in ((decode, torch.empty(2, 4, 8, dtype=torch.float16, device="meta")),
                  (prefill, torch.empty(9, 4, 8, dtype=torch.float16, device="meta"))):
        explanation = torch._dynamo.explain(fn)(x)
        assert explanation.graph_break_count == 0, explanation.break_reasons
        out = torch.compile(fn, fullgraph=True, backend="eager")(x)
        assert out.shape == x.shape


def test_triton_flags_are_boolean_and_off():
    assert DECODE_HAS_TRITON is False and PREFILL_HAS_TRITON is False


# --------------------------------------------------------------------------- backend
def test_backend_kv_cache_shape_matches_allocate():
    backend = FlashAttnTileBackend(num_heads=8, num_kv_heads=2, head_dim=16, page_size=16)
    cache = backend.allocate_kv_cache(batch=2, max_seq_len=160, dtype=torch.float16, device="cpu")
    shape = backend.get_kv_cache_shape(num_blocks=cache.num_pages, block_size=16, num_kv_heads=2, head_dim=16)
    assert shape == (2, cache.num_pages, 16, 2, 16)
    assert shape[1:] == cache.k_cache.shape
    assert backend.get_kv_cache_shape_per_tensor(cache.num_pages, 16, 2, 16) == cache.k_cache.shape
    assert backend.get_name() == "flashattn_tile"


def test_backend_validation():
    backend = FlashAttnTileBackend(num_heads=4, num_kv_heads=2, head_dim=16, page_size=16)
    cache = _cpu_cache()
    with pytest.raises(ValueError, match="cu_seqlens"):
        backend.forward(torch.randn(2, 4, 16), cache, AttentionMetadata(is_prefill=True))
    with pytest.raises(ValueError, match="heads"):
        backend.forward(torch.randn(2, 3, 16), cache, AttentionMetadata())
    with pytest.raises(ValueError, match="3-D"):
        backend.forward(torch.randn(2, 4), cache, AttentionMetadata())
    with pytest.raises(TypeError):
        backend.forward(torch.randn(2, 4, 16), object(), AttentionMetadata())
    with pytest.raises(ValueError, match="divisible"):
        FlashAttnTileBackend(num_heads=5, num_kv_heads=2, head_dim=8, page_size=16)
    with pytest.raises(ValueError, match="page_size"):
        FlashAttnTileBackend(num_heads=4, num_kv_heads=2, head_dim=8, page_size=0)
    with pytest.raises(ValueError, match="2, blocks"):
        backend.forward(torch.randn(2, 4, 16), torch.zeros(3, 4, 16, 2, 16), AttentionMetadata())


def test_backend_routes_cpu_tensors_to_no_cpu_path():
    backend = FlashAttnTileBackend(num_heads=4, num_kv_heads=2, head_dim=16, page_size=16)
    with pytest.raises(RuntimeError, match="CUDA"):
        backend.forward(torch.randn(2, 4, 16, dtype=torch.float16), _cpu_cache(), AttentionMetadata())


# --------------------------------------------------------------------------- paging
def test_append_validates_dtype_and_shape():
    cache = allocate(2, 32, 2, 16, 16, dtype=torch.float16, device="cpu")
    with pytest.raises(AssertionError, match="new_k must be"):
        append_tokens(cache, torch.zeros(2, 3, 16, dtype=torch.float16), torch.zeros(2, 3, 16, dtype=torch.float16))
    with pytest.raises(AssertionError, match="dtype"):
        append_tokens(cache, torch.zeros(2, 2, 16), torch.zeros(2, 2, 16))


def test_append_respects_page_capacity():
    cache = allocate(1, 16, 1, 8, 16, dtype=torch.float16, device="cpu")
    cache.seq_lens[0] = cache.capacity
    with pytest.raises(AssertionError, match="capacity"):
        append_tokens(cache, torch.zeros(1, 1, 8, dtype=torch.float16), torch.zeros(1, 1, 8, dtype=torch.float16))


@pytest.mark.parametrize("bad_dtype", [torch.int64, torch.float32])
def test_page_table_dtype_is_strict(bad_dtype):
    cache = _cpu_cache()
    cache.page_table = cache.page_table.to(bad_dtype)
    with pytest.raises(AssertionError, match="page_table must be int32"):
        validate_cache(cache)


def test_out_of_bounds_page_table_is_rejected():
    cache = _cpu_cache()
    cache.page_table[1, 0] = cache.num_pages
    with pytest.raises(AssertionError, match="references page"):
        validate_cache(cache)
    cache.page_table[1, 0] = -1
    with pytest.raises(AssertionError, match="negative page id"):
        validate_cache(cache)


# --------------------------------------------------------------------------- decode / prefill
def test_decode_validation_errors():
    cache = _cpu_cache()
    with pytest.raises(ValueError, match="q batch"):
        paged_decode_attention(torch.randn(3, 4, 16, dtype=torch.float16), cache)
    with pytest.raises(ValueError, match="divisible"):
        paged_decode_attention(torch.randn(2, 3, 16, dtype=torch.float16), cache)
    with pytest.raises(ValueError, match="head_dim"):
        paged_decode_attention(torch.randn(2, 4, 8, dtype=torch.float16), cache)
    with pytest.raises(ValueError, match="split_k"):
        paged_decode_attention(torch.randn(2, 4, 16, dtype=torch.float16), cache, config={"split_k": 0})



DECODE_BAD_CONFIGS = [
    # (config, message of decode.py:474-500)
    ({"bogus": 1}, "unknown decode config keys: ['bogus']"),
    ({"split_k": 0}, "split_k must be a positive integer, got 0"),
    ({"split_k": 2.0}, "split_k must be a positive integer, got 2.0"),
    ({"split_k": 65}, "split_k must be <= 64, got 65"),
    ({"num_warps": 3}, "num_warps must be a power of two <= 32, got 3"),
    ({"num_warps": 64}, "num_warps must be a power of two <= 32, got 64"),
    ({"num_stages": 0}, "num_stages must be >= 1, got 0"),
]


@pytest.mark.parametrize("config,message", DECODE_BAD_CONFIGS)
def test_decode_config_is_refused_with_the_reference_messages(config, message):
    with pytest.raises(ValueError) as exc:
        paged_decode_attention(torch.randn(2, 4, 16, dtype=torch.float16), _cpu_cache(), config=config)
    assert message in str(exc.value)


def test_decode_inputs_are_refused_with_the_reference_messages():
    """decode.py:503-522: exception type and message per malformed input (checks that need no GPU)."""
    cache = _cpu_cache()
    with pytest.raises(TypeError, match="cache must be a PagedKVCache"):
        paged_decode_attention(torch.randn(2, 4, 16, dtype=torch.float16), object())
    with pytest.raises(ValueError, match=r"q must be \[batch, heads, head_dim\], got \(2, 64\)"):
        paged_decode_attention(torch.randn(2, 64, dtype=torch.float16), cache)
    with pytest.raises(ValueError, match="q must be floating point, got torch.int16"):
        paged_decode_attention(torch.zeros(2, 4, 16, dtype=torch.int16), cache)
    with pytest.raises(ValueError, match="q head_dim 8 != cache head_dim 16"):
        paged_decode_attention(torch.randn(2, 4, 8, dtype=torch.float16), cache)
    with pytest.raises(ValueError, match="num_heads 3 must be divisible by num_kv_heads 2"):
        paged_decode_attention(torch.randn(2, 3, 16, dtype=torch.float16), cache)


def test_zero_length_sequence_is_rejected_for_decode():
    cache = _cpu_cache(lens=(4, 4))
    cache.seq_lens[1] = 0
    with pytest.raises(ValueError, match="at least one cached token"):
        paged_decode_attention(torch.randn(2, 4, 16, dtype=torch.float16), cache)


def test_prefill_config_and_offsets_are_validated():
    q = torch.randn(3, 2, 16, dtype=torch.float16)
    cu = torch.tensor([0, 3], dtype=torch.int32)
    with pytest.raises(ValueError, match="power of two"):
        prefill_attention(q, q, q, cu, cu, 3, 3, config={"BLOCK_M": 48})
    with pytest.raises(ValueError, match="unknown prefill config keys"):
        prefill_attention(q, q, q, cu, cu, 3, 3, config={"BLOCK_K": 32})
    bad = torch.tensor([0, 5], dtype=torch.int32)
    with pytest.raises(ValueError, match="must equal q.shape"):
        prefill_attention(torch.randn(4, 2, 16, dtype=torch.float16), q, q, bad, bad, 4, 4)



def _prefill_case(**over):
    """Valid CPU inputs for prefill_attention (2 sequences of 3 and 2 tokens, 4 / 2 heads), with overrides."""
    f16 = torch.float16
    args = dict(q=torch.randn(5, 4, 16, dtype=f16), k=torch.randn(6, 2, 16, dtype=f16),
                v=torch.randn(6, 2, 16, dtype=f16), cu_q=torch.tensor([0, 3, 5], dtype=torch.int32),
                cu_k=torch.tensor([0, 3, 6], dtype=torch.int32), causal=True)
    args.update(over)
    return args


PREFILL_BAD_INPUTS = [
    # (overrides, message of prefill.py:194-233, in the order the checks run)
    (dict(q=torch.randn(5, 64, dtype=torch.float16)), "must be 3-D"),
    (dict(v=torch.randn(6, 2, 8, dtype=torch.float16)), "k shape (6, 2, 16) != v shape (6, 2, 8)"),
    (dict(q=torch.randn(5, 4, 8, dtype=torch.float16)), "q head_dim 8 != k head_dim 16"),
    (dict(q=torch.randn(5, 4, 16, dtype=torch.bfloat16)), "dtype mismatch"),
    (dict(q=torch.zeros(5, 4, 16, dtype=torch.int16), k=torch.zeros(6, 2, 16, dtype=torch.int16),
          v=torch.zeros(6, 2, 16, dtype=torch.int16)), "expected floating point inputs"),
    (dict(cu_q=torch.tensor([[0, 3, 5]], dtype=torch.int32)), "must be 1-D"),
    (dict(cu_k=torch.tensor([0, 6], dtype=torch.int32)), "same batch dimension"),
    (dict(cu_q=torch.tensor([5], dtype=torch.int32), cu_k=torch.tensor([6], dtype=torch.int32)),
     "at least batch + 1 entries"),
    (dict(cu_q=torch.tensor([0, 3, 5], dtype=torch.int64)), "must be int32"),
    (dict(cu_q=torch.tensor([1, 3, 5], dtype=torch.int32)), "must start at 0"),
    (dict(cu_q=torch.tensor([0, 3, 4], dtype=torch.int32)), "cu_seqlens_q[-1] must equal q.shape[0]"),
    (dict(cu_k=torch.tensor([0, 3, 7], dtype=torch.int32)), "cu_seqlens_k[-1] must equal k.shape[0]"),
    (dict(cu_q=torch.tensor([0, 0, 3, 2, 5], dtype=torch.int32), cu_k=torch.tensor([0, 1, 3, 4, 6], dtype=torch.int32)),
     "cu_seqlens_q must be non-decreasing"),
    (dict(cu_q=torch.tensor([0, 1, 3, 4, 5], dtype=torch.int32), cu_k=torch.tensor([0, 3, 2, 4, 6], dtype=torch.int32)),
     "cu_seqlens_k must be non-decreasing"),
    (dict(cu_k=torch.tensor([0, 2, 6], dtype=torch.int32)), "requires kv_len >= q_len per sequence"),
    (dict(k=torch.randn(6, 3, 16, dtype=torch.float16), v=torch.randn(6, 3, 16, dtype=torch.float16)),
     "num_heads (4) must be divisible by num_kv_heads (3)"),
]


@pytest.mark.parametrize("over,message", PREFILL_BAD_INPUTS)
def test_prefill_inputs_are_refused_with_the_reference_messages(over, message):
    """Every check of prefill.py:194-233 that needs no GPU, hit by its own input, with its message."""
    a = _prefill_case(**over)
    with pytest.raises(ValueError) as exc:
        prefill_attention(a["q"], a["k"], a["v"], a["cu_q"], a["cu_k"], 3, 3, causal=a["causal"])
    assert message in str(exc.value)


def test_prefill_kv_shorter_than_q_is_allowed_without_the_causal_mask():
    """The kv_len >= q_len rule is the causal alignment's; the checks pass without it (the launch then
    refuses CPU tensors: there is no CPU path)."""
    a = _prefill_case(cu_k=torch.tensor([0, 2, 6], dtype=torch.int32), causal=False)
    with pytest.raises(RuntimeError, match="CUDA"):
        prefill_attention(a["q"], a["k"], a["v"], a["cu_q"], a["cu_k"], 3, 4, causal=False)


# --------------------------------------------------------------------------- work accounting
def test_flops_causal_and_noncausal():
    assert at.flops_attention(1, 4, 2, 3, causal=False) == 4 * 1 * 4 * 6
    assert at.flops_attention(1, 4, 2, 3, causal=True) == 4 * 1 * 4 * 5  # pairs 2*(3-2) + 2*3//2
    assert at.flops_attention(8, 128, 1, 4096, causal=True, batch=4) == 4 * 4 * 8 * 128 * 4096


def test_flops_varlen_sums_sequences():
    total = at.flops_attention_varlen(2, 8, [1, 4], [10, 4], causal=True)
    assert total == at.flops_attention(2, 8, 1, 10, causal=True) + at.flops_attention(2, 8, 4, 4, causal=True)
    with pytest.raises(ValueError):
        at.flops_attention_varlen(2, 8, [1], [1, 2])


def test_bytes_attention_modes():
    nbytes = at.bytes_attention("decode", 8, 1, 4096, 32, 8, 128, elem_bytes=2)
    assert nbytes == 8 * 4096 * 8 * 128 * 2 * 2 + 2 * 8 * 32 * 128 * 2
    assert 3.0 < at.arithmetic_intensity(at.flops_attention(32, 128, 1, 4096, causal=True, batch=8), nbytes) < 5.0
    assert at.bytes_attention("prefill", 1, 1024, 1024, 32, 8, 128, 2) == \
        2 * (1024 * 32 * 128 * 2) + 1024 * 8 * 128 * 2 * 2
    with pytest.raises(ValueError):
        at.bytes_attention("backward", 1, 1, 1, 1, 1, 1)
    with pytest.raises(ValueError):
        at.bytes_attention("decode", 1, 2, 4, 1, 1, 1)


def test_cfg2_algorithmic_bytes():
    """The headline roofline numerator: Q + O + K/V rows of every cached token."""
    assert at.bytes_decode_paged([4096] * 32, 32, 8, 128, 16, q_bytes=2, kv_bytes=2) == 537_395_200


def test_oracle_and_library_accounting_agree():
    """bench.py's reference arm counts bytes with the oracle copy (it must not load the library)."""
    from oracle import work

    assert work.bytes_decode_paged([4096] * 32, 32, 8, 128, 16) == 537_395_200
    for lens, ps, kvb, sb in (([1, 17, 4095], 16, 2, 0), ([1024, 16384, 7], 32, 1, 4), ([131072] * 8, 64, 2, 0)):
        assert work.bytes_decode_paged(lens, 64, 8, 128, ps, 2, kvb, sb) == \
            at.bytes_decode_paged(lens, 64, 8, 128, ps, q_bytes=2, kv_bytes=kvb, scale_bytes=sb)
    assert work.flops_attention_varlen(32, 128, [512, 1024, 2048, 4096], [512, 1024, 2048, 4096], causal=True) \
        == at.flops_attention_varlen(32, 128, [512, 1024, 2048, 4096], [512, 1024, 2048, 4096], causal=True) \
        == 182_599_024_640
