"""Native-extension entry points (FlashAttnTile's ``flashattn_tile/native.py:54-84``).

In the reference this lazily JIT-builds a CUDA C++ decode baseline.  Here the
native library *is* the implementation: ``is_available`` reports whether
``libflashattn_sm100.so`` loads and a CUDA device is present, and
``paged_decode_attention`` calls the same sm_100a decode kernel as the ops.
"""

from __future__ import annotations

import torch

from . import _lib
from .kernels.decode import launch_decode


def is_available() -> bool:
    return torch.cuda.is_available() and _lib.available()


def unavailable_reason() -> str:
    if not torch.cuda.is_available():
        return "no CUDA device detected"
    return _lib.unavailable_reason()


def paged_decode_attention(q, k_cache, v_cache, page_table, seq_lens, page_size, softmax_scale=None):
    """Decode through the sm_100a kernel; RuntimeError when it is unavailable."""
    if not is_available():
        raise RuntimeError(f"native CUDA path unavailable: {unavailable_reason()}")
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    return launch_decode(q, k_cache, v_cache, page_table, seq_lens, int(page_size), float(softmax_scale))
