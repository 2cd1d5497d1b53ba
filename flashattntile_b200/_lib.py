"""ctypes binding of ``libflashattn_sm100.so`` (the C ABI in include/flashattn_tile_b200.h).

The library is built in-tree by ``flashattntile_b200.csrc.build`` and loaded
lazily on first use.  There is no fallback: if the library is missing or the
tensors are not on a CUDA device, calls raise ``RuntimeError``.

Status codes from the C ABI map to Python exceptions: invalid arguments ->
``ValueError``, unsupported shapes -> ``NotImplementedError``, CUDA failures
and too-small scratch buffers -> ``RuntimeError``; the message is the
library's ``fat_last_error()``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libflashattn_sm100.so"

FAT_OK = 0
FAT_ERR_INVALID_ARGUMENT = 1
FAT_ERR_UNSUPPORTED = 2
FAT_ERR_CUDA = 3
FAT_ERR_WORKSPACE = 4

FAT_DEVERR_TIMEOUT = 1
FAT_DEVERR_BAD_PAGE = 2
FAT_DEVERR_BAD_LENGTH = 4

DTYPE_CODE = {
    torch.float16: 0,
    torch.bfloat16: 1,
    torch.float32: 2,
    torch.int8: 3,
}
if hasattr(torch, "float8_e4m3fn"):
    DTYPE_CODE[torch.float8_e4m3fn] = 4

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_vp = ctypes.c_void_p
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol the public header declares.
SIGNATURES: dict[str, tuple] = {
    "fat_version": (ctypes.c_char_p, []),
    "fat_last_error": (ctypes.c_char_p, []),
    "fat_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "fat_expire_next_waits": (None, [_i32]),
    "fat_set_prefill_p_split": (_i32, [_i32]),
    "fat_set_prefill_schedule": (_i32, [_i32]),
    "fat_paged_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "fat_paged_decode": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _sz, _vp, _vp],
    ),
    "fat_paged_decode_lse": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i64,
         _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _sz, _vp, _vp],
    ),
    "fat_paged_decode_call": (_i32, [_vp]),
    "fat_lse_merge": (_i32, [_vp, _i64, _vp, _i64, _i32, _i64, _i32, _vp, _i32, _vp, _vp]),
    "fat_paged_decode_noalloc": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _vp],
    ),
    "fat_prefill_varlen": (
        _i32,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i32, _i64, _i64, _i32, _i32,
         _i32, _i32, _i32, _i32, _f32, _i32, _i32, _vp, _vp],
    ),
    "fat_prefill_paged": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i32, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _vp, _vp],
    ),
    "fat_append_tokens": (
        _i32,
        [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32,
         _i32, _i32, _i32, _i32, _vp, _vp],
    ),
    "fat_cache_value_stats": (_i32, [_vp, _vp, _i64, _i32, _i64, _i32, _vp, _vp, _vp]),
    "fat_gather_paged": (
        _i32,
        [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _vp, _vp],
    ),
}



class DecodeCall(ctypes.Structure):
    """``fat_decode_call`` (include/flashattn_tile_b200.h): fat_paged_decode_lse's
    arguments in one struct, plus the optional value-statistics outputs."""

    _fields_ = [
        ("q", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64), ("k_cache", _vp), ("v_cache", _vp),
        ("kv_stride_page", _i64), ("kv_stride_slot", _i64), ("kv_stride_head", _i64), ("num_pages", _i64),
        ("page_table", _vp), ("page_table_stride", _i64), ("max_pages", _i64), ("seq_lens", _vp),
        ("k_scale", _vp), ("v_scale", _vp), ("scale_stride_page", _i64), ("out", _vp), ("out_stride_b", _i64),
        ("out_stride_h", _i64), ("lse", _vp), ("lse_stride_b", _i64), ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("page_size", ctypes.c_int32), ("q_dtype", ctypes.c_int32), ("kv_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32), ("softmax_scale", ctypes.c_float), ("split_k_hint", ctypes.c_int32),
        ("workspace", _vp), ("workspace_bytes", _sz), ("error_word", _vp), ("stream", _vp), ("stats_out", _vp),
        ("stats_scratch", _vp), ("stats_event", _vp),
    ]


_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None
_ERROR: str | None = None


def load() -> ctypes.CDLL:
    """Load the library once (thread-safe); raise RuntimeError if it is missing."""
    global _LIB, _ERROR
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                _ERROR = (f"{LIB_PATH.name} is not built; run `python -m flashattntile_b200.csrc.build` "
                          "(or __graft_entry__.build())")
                raise RuntimeError(_ERROR)
            lib = ctypes.CDLL(os.fspath(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                try:
                    fn = getattr(lib, name)
                except AttributeError:
                    _ERROR = f"{LIB_PATH.name} lacks {name}: it is out of date, rebuild it"
                    raise RuntimeError(_ERROR) from None
                fn.restype = res
                fn.argtypes = args
            _LIB = lib
    return _LIB


def available() -> bool:
    try:
        load()
        return True
    except (OSError, RuntimeError):
        return False


def unavailable_reason() -> str:
    if available():
        return ""
    return _ERROR or "library failed to load"


def check(status: int, what: str) -> None:
    if status == FAT_OK:
        return
    msg = load().fat_last_error().decode(errors="replace") or what
    if status == FAT_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == FAT_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"{what} failed (status {status}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# Scratch buffers: one zero-filled buffer per (device, stream), grown on demand.
# The decode kernel leaves its tickets zeroed on success, so calls ordered on
# one stream can share the buffer; a call that reported a device error resets it.
# ---------------------------------------------------------------------------
_WS: dict[tuple[int, int], torch.Tensor] = {}
_ERR: dict[tuple[int, int], torch.Tensor] = {}
_STATS: dict[tuple[int, int], tuple[torch.Tensor, torch.Tensor, torch.cuda.Event]] = {}


def workspace_for(index: int, stream: int, device: torch.device, nbytes: int) -> torch.Tensor:
    buf = _WS.get((index, stream))
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WS[(index, stream)] = buf
    return buf


def error_word_for(index: int, stream: int, device: torch.device) -> torch.Tensor:
    buf = _ERR.get((index, stream))
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[(index, stream)] = buf
    return buf


def _key(device: torch.device) -> tuple[int, int]:
    index = device.index if device.index is not None else torch.cuda.current_device()
    return index, torch.cuda.current_stream(torch.device("cuda", index)).cuda_stream


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    index, stream = _key(device)
    return workspace_for(index, stream, device, nbytes)


def error_word(device: torch.device) -> torch.Tensor:
    index, stream = _key(device)
    return error_word_for(index, stream, device)


def reset_workspace(device: torch.device) -> None:
    key = _key(device)
    if key in _WS:
        _WS[key].zero_()
    if key in _ERR:
        _ERR[key].zero_()


def stats_buffers(index: int, stream: int, device: torch.device):
    """This stream's (device scratch, pinned host int32[4], event) for the value statistics."""
    bufs = _STATS.get((index, stream))
    if bufs is None:
        bufs = (torch.zeros(4, dtype=torch.int32, device=device), torch.zeros(4, dtype=torch.int32).pin_memory(),
                torch.cuda.Event())
        _STATS[(index, stream)] = bufs
    return bufs


def cache_value_stats_async(seq_lens: torch.Tensor, page_table: torch.Tensor,
                            page_size: int) -> tuple[torch.Tensor, torch.cuda.Event]:
    """Queue ``fat_cache_value_stats`` on the current stream: returns the pinned
    host buffer that will hold [min len, max len, min used page id, max used page
    id] and an event recorded after the copy (synchronise it before reading).
    The buffer is per stream: read it before the next call on the same stream."""
    lib = load()
    dev = seq_lens.device
    index, stream = _key(dev)
    bufs = stats_buffers(index, stream, dev)
    if page_table.stride(1) != 1:
        page_table = page_table.contiguous()
    if not seq_lens.is_contiguous():
        seq_lens = seq_lens.contiguous()
    status = lib.fat_cache_value_stats(seq_lens.data_ptr(), page_table.data_ptr(), page_table.stride(0),
                                       seq_lens.numel(), page_table.shape[1], int(page_size), bufs[0].data_ptr(),
                                       bufs[1].data_ptr(), stream)
    check(status, "cache_value_stats")
    bufs[2].record(torch.cuda.current_stream(dev))
    return bufs[1], bufs[2]


def cache_value_stats(seq_lens: torch.Tensor, page_table: torch.Tensor, page_size: int) -> list[int]:
    """:func:`cache_value_stats_async`, waited for."""
    host, event = cache_value_stats_async(seq_lens, page_table, page_size)
    event.synchronize()
    return host.tolist()


def read_device_error(device: torch.device) -> int:
    """Synchronously read (and clear) the device error word of this stream."""
    word = error_word(device)
    value = int(word.item())
    if value:
        reset_workspace(device)
    return value
