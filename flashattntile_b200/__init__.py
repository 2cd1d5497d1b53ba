"""flashattntile_b200: B200-native (sm_100a) paged attention, drop-in for FlashAttnTile's ops.

Importing the package registers the ``torch.ops.flashattn_tile`` custom ops
(``paged_decode``, ``prefill_varlen``, ``paged_decode_quant``) whose CUDA
implementations live in ``libflashattn_sm100.so`` (C ABI in
``include/flashattn_tile_b200.h``).  Module layout follows the reference
package: ``ops``, ``paging``, ``quant``, ``backend``, ``native``,
``kernels.decode``, ``kernels.prefill`` and ``autotune`` (work accounting).

The fp32 reference attention of FlashAttnTile is not part of the library;
its restatement lives in the repository's test oracle.
"""

from __future__ import annotations

__version__ = "0.1.0"

import torch

from . import _lib
from . import ops as _ops  # noqa: F401  (registers the custom ops)
from ._config import set_validate_values, validate_values, value_checks
from .ops import PAGED_DECODE_OP, PAGED_DECODE_QUANT_OP, PREFILL_OP, paged_decode, paged_decode_quant, prefill_varlen
from .paging import PagedKVCache, allocate, append_tokens, gather_contiguous, gather_paged


def device_error(device: torch.device | str | int | None = None) -> int:
    """Read and clear the device error word of the current stream (synchronises).

    Bit 1 (``FAT_DEVERR_TIMEOUT``): a bounded in-kernel wait gave up.
    Bit 2 (``FAT_DEVERR_BAD_PAGE``): a page id outside the cache was skipped.
    Bit 4 (``FAT_DEVERR_BAD_LENGTH``): a sequence length beyond the page table's
    capacity (``max_pages * page_size``) was cut to that capacity.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return _lib.read_device_error(dev)


def library_path() -> str:
    return str(_lib.LIB_PATH)


__all__ = [
    "__version__",
    "PAGED_DECODE_OP",
    "PREFILL_OP",
    "PAGED_DECODE_QUANT_OP",
    "paged_decode",
    "prefill_varlen",
    "paged_decode_quant",
    "PagedKVCache",
    "allocate",
    "append_tokens",
    "gather_contiguous",
    "gather_paged",
    "device_error",
    "library_path",
    "validate_values",
    "set_validate_values",
    "value_checks",
]
