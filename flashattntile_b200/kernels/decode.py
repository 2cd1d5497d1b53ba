"""Paged decode attention on B200: launcher of the sm_100a decode kernel.

Python API of FlashAttnTile's ``flashattn_tile/kernels/decode.py``:

* ``paged_decode_attention(q, cache, softmax_scale=None, config=None, grouped=False)``
  (``decode.py:533-642``)
* ``paged_decode_attention_fp8(q, cache, scales, softmax_scale=None, config=None)``
  (``decode.py:645-704``)
* ``DEFAULT_CONFIG`` (``decode.py:458``)

Both run the same CUDA kernel (``fat_paged_decode``): one persistent CTA per
SM, pages split evenly over all SMs from ``seq_lens`` on the device, K/V
pages staged by TMA once per GQA group, scores and P.V on the tensor cores
with fp32 accumulation, INT8/e4m3 dequantised in registers.  ``split_k``,
``num_warps``, ``num_stages`` and ``grouped`` are validated as in the
reference and otherwise ignored: the split is chosen on the device and the
result does not depend on them.

There is no CPU or fp32 path: CPU tensors raise ``RuntimeError``; fp32
queries raise ``NotImplementedError``.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from .. import _config, _lib
from ..paging import (PagedKVCache, check_value_numbers, check_value_stats, validate_cache_values,
                      validate_metadata)

DEFAULT_CONFIG = {"split_k": 1, "num_warps": 4, "num_stages": 2}
# Import compatibility with code written against the reference: this build has
# no Triton kernels; HAS_CUDA_KERNELS says whether the sm_100a library loads.
HAS_TRITON = False
HAS_CUDA_KERNELS = _lib.available()

_QUANT_DTYPES = (torch.int8,) + ((torch.float8_e4m3fn,) if hasattr(torch, "float8_e4m3fn") else ())


def _resolve_config(config: dict | None) -> dict:
    """Key and range checks of ``decode.py:474-500`` (messages kept)."""
    resolved = dict(DEFAULT_CONFIG)
    if config is not None:
        unknown = set(config) - set(DEFAULT_CONFIG)
        if unknown:
            raise ValueError(f"unknown decode config keys: {sorted(unknown)}")
        resolved.update(config)
    split_k = resolved["split_k"]
    if not isinstance(split_k, int) or split_k < 1:
        raise ValueError(f"split_k must be a positive integer, got {split_k}")
    if split_k > 64:
        raise ValueError(f"split_k must be <= 64, got {split_k}")
    if resolved["num_warps"] not in (1, 2, 4, 8, 16, 32):
        raise ValueError(f"num_warps must be a power of two <= 32, got {resolved['num_warps']}")
    if resolved["num_stages"] < 1:
        raise ValueError(f"num_stages must be >= 1, got {resolved['num_stages']}")
    return resolved


def _q_error(q: torch.Tensor, cache: PagedKVCache) -> Exception | None:
    if q.dim() != 3:
        return ValueError(f"q must be [batch, heads, head_dim], got {tuple(q.shape)}")
    if q.shape[0] != cache.batch_size:
        return ValueError(f"q batch {q.shape[0]} != cache batch {cache.batch_size}")
    if q.shape[2] != cache.head_dim:
        return ValueError(f"q head_dim {q.shape[2]} != cache head_dim {cache.head_dim}")
    if q.shape[1] % cache.num_kv_heads != 0:
        return ValueError(f"num_heads {q.shape[1]} must be divisible by num_kv_heads {cache.num_kv_heads}")
    if q.device != cache.k_cache.device:
        return ValueError("q and cache must live on the same device")
    if not q.is_floating_point():
        return ValueError(f"q must be floating point, got {q.dtype}")
    return None


def _value_checks(cache: PagedKVCache) -> None:
    """The value checks of ``decode.py:503-522`` (one device->host read-back)."""
    if not _config.validate_values():
        return
    _check_lengths(validate_cache_values(cache))


def _check_lengths(stats) -> None:
    if stats is not None and stats[0] <= 0:
        raise ValueError("decode requires every sequence to hold at least one cached token")


def _run_checked(cache: PagedKVCache, fire):
    """Launch ``fire`` and apply the value checks, raising the reference's error
    (type and message) before returning.  On CUDA the statistics are queued
    first and the kernel right behind them, so the GPU does not idle while the
    host waits for the 16-byte read-back; the kernel is memory-safe on any
    metadata (page ids outside the pool are skipped and reported on the device,
    lengths are bounded by the page table), so an invalid call only costs an
    unused output before it raises."""
    lens, table = cache.seq_lens, cache.page_table
    if not _config.validate_values() or lens.numel() == 0:
        return fire()
    if not (lens.is_cuda and table.is_cuda and lens.device == table.device):
        _value_checks(cache)
        return fire()
    host, event = _lib.cache_value_stats_async(lens, table, cache.page_size)
    out = fire()
    event.synchronize()
    _check_lengths(check_value_stats(cache, host.tolist()))
    return out


def _check_decode_structure(q: torch.Tensor, cache: PagedKVCache) -> None:
    """``decode.py:503-522`` minus the value checks: every check that reads no
    device memory, same exception types and messages.  A q error is raised after
    the value checks, as the reference checks the cache values first; on success
    the caller applies the value checks around the launch (``_run_checked``)."""
    if not isinstance(cache, PagedKVCache):
        raise TypeError("cache must be a PagedKVCache")
    validate_metadata(cache)
    err = _q_error(q, cache)
    if err is not None:
        if _config.validate_values():
            validate_cache_values(cache)
        raise err


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "flashattntile_b200 runs on CUDA tensors only; it has no CPU path "
                f"(got a tensor on {t.device})")


def _aligned_q(q: torch.Tensor) -> torch.Tensor:
    eb = q.element_size()
    ok = (q.stride(2) == 1 and q.data_ptr() % 16 == 0 and (q.stride(0) * eb) % 16 == 0
          and (q.stride(1) * eb) % 16 == 0)
    return q if ok else q.contiguous()


def prepare_decode(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k=1,
                   k_scale=None, v_scale=None, out=None, out_dtype=None, lse=None, remember=False):
    """All of :func:`launch_decode`'s host work (checks, output, scratch, the
    argument struct) without the launch: returns a callable that launches on the
    stream current now and returns the output.  Callers that must synchronise
    before launching (value checks) prepare first, so the GPU waits for no host
    work after the synchronisation.

    ``remember``: keep the argument struct for the op fast path when nothing was
    copied on the way (see ``_fast_decode``).
    """
    _require_cuda(q, k_cache, v_cache, page_table, seq_lens)
    lib = _lib.load()
    dev = q.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    q_in, table_in, lens_in, ks_in, vs_in = q, page_table, seq_lens, k_scale, v_scale
    q = _aligned_q(q)
    if k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache must have identical strides")
    if k_cache.stride(3) != 1:
        raise ValueError("k_cache/v_cache must be contiguous along head_dim")
    if page_table.stride(1) != 1:
        page_table = page_table.contiguous()
    if not seq_lens.is_contiguous():
        seq_lens = seq_lens.contiguous()
    batch, heads, dim = q.shape
    kvh = k_cache.shape[2]
    if out is not None:
        # A given output fixes the dtype the kernel writes.
        if out_dtype is not None and out_dtype != out.dtype:
            raise ValueError(f"out_dtype {out_dtype} does not match out's dtype {out.dtype}")
        if tuple(out.shape) != (batch, heads, dim) or not out.is_cuda:
            raise ValueError(f"out must be a CUDA tensor of shape {(batch, heads, dim)}, got {tuple(out.shape)}")
        out_dtype = out.dtype
    out_dtype = out_dtype or q.dtype
    own_out = out is None
    if out is None:
        out = torch.empty((batch, heads, dim), dtype=out_dtype, device=dev)
    scale_stride = 0
    if k_scale is not None:
        if k_scale.stride(1) != 1 or v_scale.stride() != k_scale.stride():
            k_scale, v_scale = k_scale.contiguous(), v_scale.contiguous()
        scale_stride = k_scale.stride(0)
    stream_obj = torch.cuda.current_stream(dev)
    stream = stream_obj.cuda_stream
    ws = _lib.workspace_for(idx, stream, dev, lib.fat_paged_decode_workspace_size(idx, batch, heads, kvh, dim))
    err = _lib.error_word_for(idx, stream, dev)
    if lse is not None:
        if lse.dtype != torch.float32 or lse.device != dev or lse.dim() != 2 or lse.stride(1) != 1 \
                or tuple(lse.shape) != (batch, heads):
            raise ValueError(f"lse must be a float32 [{batch}, {heads}] tensor on {dev} with unit stride along heads")
    call = _lib.DecodeCall(
        q=q.data_ptr(), q_stride_b=q.stride(0), q_stride_h=q.stride(1), k_cache=k_cache.data_ptr(),
        v_cache=v_cache.data_ptr(), kv_stride_page=k_cache.stride(0), kv_stride_slot=k_cache.stride(1),
        kv_stride_head=k_cache.stride(2), num_pages=k_cache.shape[0], page_table=page_table.data_ptr(),
        page_table_stride=page_table.stride(0), max_pages=page_table.shape[1], seq_lens=seq_lens.data_ptr(),
        k_scale=_lib.ptr(k_scale), v_scale=_lib.ptr(v_scale), scale_stride_page=scale_stride, out=out.data_ptr(),
        out_stride_b=out.stride(0), out_stride_h=out.stride(1), lse=_lib.ptr(lse),
        lse_stride_b=0 if lse is None else lse.stride(0), batch=batch, num_heads=heads, num_kv_heads=kvh,
        head_dim=dim, page_size=int(page_size), q_dtype=_lib.DTYPE_CODE[q.dtype],
        kv_dtype=_lib.DTYPE_CODE[k_cache.dtype], out_dtype=_lib.DTYPE_CODE[out_dtype],
        softmax_scale=float(softmax_scale), split_k_hint=int(split_k), workspace=ws.data_ptr(),
        workspace_bytes=ws.numel(), error_word=err.data_ptr(), stream=stream, stats_out=None, stats_scratch=None)
    fn = lib.fat_paged_decode_call

    def fire() -> torch.Tensor:
        # `call` itself (not just its address) lives in this closure: the struct
        # must outlive prepare_decode until the library has read it.
        if idx == torch.cuda.current_device():
            status = fn(ctypes.addressof(call))
        else:
            with torch.cuda.device(idx):
                status = fn(ctypes.addressof(call))
        _lib.check(status, "paged_decode")
        return out

    if (remember and own_out and lse is None and q is q_in and page_table is table_in and seq_lens is lens_in
            and k_scale is ks_in and v_scale is vs_in and idx == torch.cuda.current_device()):
        _remember(_fast_key(q_in, k_cache, v_cache, table_in, lens_in, page_size, softmax_scale, split_k, ks_in,
                            vs_in), call, out, ws, idx, stream, stream_obj, k_cache.shape[0],
                  table_in.shape[1] * int(page_size))
    return fire


# --------------------------------------------------------------------------- fast path
# A serving loop calls the op with the same tensors (same storage, shapes,
# strides, dtypes, stream) step after step.  After one call has passed every
# structural check, its argument struct is kept under a key made of exactly
# those properties; the next call with an equal key skips the checks and the
# argument packing, allocates its output, runs the value checks (the
# statistics kernel is queued in the same library call) and launches.  Entries
# hold pointers and sizes only, never tensors, so they keep no memory alive;
# the scratch buffer is re-checked on every hit.
_FAST: dict = {}
_FAST_MAX = 256


class _Plan:
    __slots__ = ("call", "addr", "out_shape", "out_dtype", "device", "ws_key", "ws_ptr", "stream_obj", "stats_host",
                 "stats_host_ptr", "stats_dev_ptr", "stats_event", "num_pages", "capacity")


def _fast_key(q, k, v, table, lens, page_size, scale, split_k, k_scale=None, v_scale=None):
    dev = q.get_device()
    if dev < 0:
        return None
    key = (threading.get_ident(), dev, torch._C._cuda_getCurrentRawStream(dev), q.data_ptr(), q.shape, q.stride(),
           q.dtype, k.data_ptr(), k.shape, k.stride(), k.dtype, v.data_ptr(), v.shape, v.stride(), v.dtype,
           table.data_ptr(), table.shape, table.stride(), table.dtype, table.get_device(), lens.data_ptr(),
           lens.shape, lens.stride(), lens.dtype, lens.get_device(), int(page_size), float(scale), int(split_k))
    if k_scale is not None:
        key += (k_scale.data_ptr(), k_scale.shape, k_scale.stride(), k_scale.dtype, v_scale.data_ptr(),
                v_scale.shape, v_scale.stride(), v_scale.dtype)
    return key


def _remember(key, call, out, ws, idx, stream, stream_obj, num_pages, capacity) -> None:
    if key is None:
        return
    plan = _Plan()
    plan.call, plan.addr = call, ctypes.addressof(call)
    plan.out_shape, plan.out_dtype, plan.device = tuple(out.shape), out.dtype, out.device
    plan.ws_key, plan.ws_ptr = (idx, stream), ws.data_ptr()
    plan.stream_obj = stream_obj
    scratch, host, event = _lib.stats_buffers(idx, stream, out.device)
    if event.cuda_event == 0:
        event.record(stream_obj)  # creates the CUDA event, whose handle the library records
    plan.stats_host, plan.stats_host_ptr, plan.stats_dev_ptr, plan.stats_event = host, host.data_ptr(), \
        scratch.data_ptr(), event
    plan.num_pages, plan.capacity = int(num_pages), int(capacity)
    if len(_FAST) >= _FAST_MAX:
        _FAST.clear()
    _FAST[key] = plan


def _fast_decode(key) -> torch.Tensor | None:
    """Launch a remembered decode (value checks included); None when there is no usable entry."""
    plan = _FAST.get(key) if key is not None else None
    if plan is None:
        return None
    ws = _lib._WS.get(plan.ws_key)
    if ws is None or ws.data_ptr() != plan.ws_ptr or plan.device.index != torch.cuda.current_device():
        return None
    out = torch.empty(plan.out_shape, dtype=plan.out_dtype, device=plan.device)
    call = plan.call
    call.out = out.data_ptr()
    checks = _config.validate_values()
    if checks:
        # The library queues the statistics, records the event, then the decode:
        # the host waits for the 16-byte statistics only, never for the decode.
        call.stats_out, call.stats_scratch = plan.stats_host_ptr, plan.stats_dev_ptr
        call.stats_event = plan.stats_event.cuda_event
    else:
        call.stats_out = call.stats_scratch = call.stats_event = None
    status = _lib.load().fat_paged_decode_call(plan.addr)
    _lib.check(status, "paged_decode")
    if checks:
        plan.stats_event.synchronize()
        lo, _ = check_value_numbers(plan.stats_host.tolist(), plan.capacity, plan.num_pages)
        _check_lengths((lo, None))
    return out


def launch_decode(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k=1,
                  k_scale=None, v_scale=None, out=None, out_dtype=None, lse=None):
    """Run ``fat_paged_decode`` on the current stream of q's device.

    With ``lse`` (fp32 ``[B, H]``, unit stride along H) the kernel also writes
    the base-2 log-sum-exp of each row's scaled scores (``fat_paged_decode_lse``),
    -inf for a sequence with no cached tokens.

    No host<->device synchronisation happens here; device-side problems are
    recorded in the stream's error word (``flashattntile_b200.device_error``).
    """
    return prepare_decode(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale, split_k,
                          k_scale=k_scale, v_scale=v_scale, out=out, out_dtype=out_dtype, lse=lse)()


def _fast_args(q, cache, softmax_scale, config):
    """(scale, split_k) when this call may take the fast path, else None."""
    if type(cache) is not PagedKVCache or not isinstance(q, torch.Tensor) or q.dim() != 3:
        return None
    if config is None:
        split_k = 1
    elif type(config) is dict and len(config) == 1 and type(config.get("split_k")) is int:
        split_k = config["split_k"]
    else:
        return None
    if softmax_scale is None:
        scale = q.shape[-1] ** -0.5
    elif isinstance(softmax_scale, (int, float)):
        scale = float(softmax_scale)
    else:
        return None
    return scale, split_k


def paged_decode_attention(q: torch.Tensor, cache: PagedKVCache, softmax_scale: float | None = None,
                           config: dict | None = None, grouped: bool = False) -> torch.Tensor:
    """One query per sequence against a paged fp16/bf16 cache -> ``[B, H, D]`` in q's dtype."""
    fast = _fast_args(q, cache, softmax_scale, config)
    if fast is not None:
        out = _fast_decode(_fast_key(q, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens,
                                     cache.page_size, *fast))
        if out is not None:
            return out
    _check_decode_structure(q, cache)
    del grouped  # every launch shares each K/V page across its GQA group
    try:
        scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
        cfg = _resolve_config(config)
        _require_cuda(q)
        if q.dtype not in (torch.float16, torch.bfloat16):
            raise NotImplementedError(f"paged decode has fp16/bf16 kernels only, got {q.dtype}")
        if cache.k_cache.dtype != q.dtype:
            raise ValueError(f"q dtype {q.dtype} must match cache dtype {cache.k_cache.dtype}")
        fire = prepare_decode(q, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens,
                              cache.page_size, scale, cfg["split_k"], remember=True)
    except Exception:
        _value_checks(cache)  # the reference reports bad cache values first
        raise
    return _run_checked(cache, fire)


def paged_decode_attention_fp8(q: torch.Tensor, cache: PagedKVCache, scales, softmax_scale: float | None = None,
                               config: dict | None = None) -> torch.Tensor:
    """Decode against an INT8 / float8_e4m3fn cache with per-(page, KV-head) fp32 scales."""
    fast = _fast_args(q, cache, softmax_scale, config)
    if fast is not None and isinstance(scales, dict) and isinstance(scales.get("k"), torch.Tensor) \
            and isinstance(scales.get("v"), torch.Tensor):
        out = _fast_decode(_fast_key(q, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens,
                                     cache.page_size, *fast, scales["k"], scales["v"]))
        if out is not None:
            return out
    _check_decode_structure(q, cache)
    try:
        fire = _prepare_decode_fp8(q, cache, scales, softmax_scale, config)
    except Exception:
        _value_checks(cache)  # the reference reports bad cache values first
        raise
    return _run_checked(cache, fire)


def _prepare_decode_fp8(q, cache, scales, softmax_scale, config):
    k_scale = scales["k"] if isinstance(scales, dict) else scales.k
    v_scale = scales["v"] if isinstance(scales, dict) else scales.v
    if cache.k_cache.dtype not in _QUANT_DTYPES:
        raise ValueError(f"expected int8/float8 cache, got {cache.k_cache.dtype}")
    expected = (cache.num_pages, cache.num_kv_heads)
    if tuple(k_scale.shape) != expected or tuple(v_scale.shape) != expected:
        raise ValueError(f"scales must have shape {expected}, got {tuple(k_scale.shape)}")
    scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
    cfg = _resolve_config(config)
    _require_cuda(q, k_scale, v_scale)
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"quantised decode requires fp16/bf16 queries, got {q.dtype}")
    return prepare_decode(q, cache.k_cache, cache.v_cache, cache.page_table, cache.seq_lens, cache.page_size,
                          scale, cfg["split_k"], k_scale=k_scale.float(), v_scale=v_scale.float(), remember=True)
