"""CPU oracle for the paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithm of FlashAttnTile's fp32
reference path so that the CUDA kernels of ``flashattntile_b200`` can be
checked against it on machines where the reference itself is absent:

* ``oracle.attention``  -- ``flashattn_tile/reference.py:50-219`` (varlen,
  paged and dense fp32 attention, bottom-right causal alignment, GQA
  ``h // G``, output rounded to the input dtype) plus the split-K
  log-sum-exp merge of ``flashattn_tile/kernels/decode.py:12-14,341-352``.
* ``oracle.paging``     -- ``flashattn_tile/paging.py:84-256`` (validation
  messages, one-token append, padded page-table gather).
* ``oracle.quant``      -- ``flashattn_tile/quant.py:84-208`` (per-(page,
  KV-head) INT8 / FP8-e4m3 scales).
* ``oracle.work``       -- ``flashattn_tile/autotune.py:31-112`` (the
  algorithmic FLOP and byte counts every throughput number divides by).
* ``oracle.numerics``   -- fp16 / bf16 / e4m3 encodings used by the above.

Pinning: ``tests/golden/make_golden.py`` runs the reference implementation
itself (imported from a reference checkout) on seeded inputs and stores the
inputs and outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every function here against those vectors.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
baseline leg and its ``--impl reference`` arm) may import this package, and
only as the checker or the timed CPU baseline.  The library
``flashattntile_b200`` never imports it and has no CPU fallback.
"""

from . import attention, numerics, paging, quant, work  # noqa: F401

__all__ = ["attention", "numerics", "paging", "quant", "work"]
