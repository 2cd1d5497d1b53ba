"""Process-wide switches.

``FLASHATTN_TILE_VALIDATE`` (default ``1``) selects how much each op checks on
the host before launching:

* ``1`` -- everything FlashAttnTile checks, including the value checks that
  read ``seq_lens`` / ``page_table`` / ``cu_seqlens`` back to the host
  (``paging.py:114-130``, ``decode.py:521``, ``prefill.py:217-229``), with the
  same exception types and messages.  Each of those reads synchronises the
  stream, as it does in the reference.
* ``0`` -- shape, dtype and device checks only: no device->host reads, so the
  ops can run inside CUDA-graph capture.  Bad page ids are then caught on the
  device (the page is skipped and ``FAT_DEVERR_BAD_PAGE`` is recorded in the
  per-stream error word, see ``flashattntile_b200.device_error``).
"""

from __future__ import annotations

import contextlib
import os

_VALIDATE = os.environ.get("FLASHATTN_TILE_VALIDATE", "1") not in ("0", "false", "False", "")


def validate_values() -> bool:
    return _VALIDATE


def set_validate_values(flag: bool) -> None:
    global _VALIDATE
    _VALIDATE = bool(flag)


@contextlib.contextmanager
def value_checks(flag: bool):
    """Temporarily enable / disable host-side value checks."""
    global _VALIDATE
    old = _VALIDATE
    _VALIDATE = bool(flag)
    try:
        yield
    finally:
        _VALIDATE = old
