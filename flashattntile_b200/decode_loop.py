"""One decode iteration per CUDA-graph replay: append the step's K/V, then paged decode.

FlashAttnTile's decode loop (``scripts/demo_decode_loop.py:103-140``, through
``backend.forward``, ``backend.py:132-175``) calls a ``torch.compile``d
``flashattn_tile::paged_decode`` each step, with host-side value checks that
read ``seq_lens``/``page_table`` back, and appends the new token with torch
indexing and more host reads (``paging.py:172-210``).  Here the whole
iteration is two kernels -- the device-side append (which also advances
``seq_lens``) and the decode -- captured once into a CUDA graph with value
checks off, then replayed per token:

    loop = DecodeLoop(cache, num_heads=32)           # or scales=... for INT8/FP8
    out = loop.step(q, new_k, new_v)                  # copy in, replay, output view

Nothing on the host depends on the sequence lengths, so every replay sees the
lengths the previous one left on the device.  A sequence that reaches the end
of its page table is skipped by the append kernel and reported in the device
error word (``flashattntile_b200.device_error()``).
"""

from __future__ import annotations

import torch

from . import _config, _lib
from .kernels.append import launch_append
from .kernels.decode import launch_decode
from .paging import PagedKVCache, validate_metadata


class DecodeLoop:
    """A captured (append, decode) step for a fixed batch / head geometry."""

    def __init__(self, cache: PagedKVCache, num_heads: int, softmax_scale: float | None = None, scales=None,
                 q_dtype: torch.dtype | None = None, in_dtype: torch.dtype | None = None):
        validate_metadata(cache)
        if not cache.k_cache.is_cuda:
            raise RuntimeError("DecodeLoop: flashattntile_b200 runs on CUDA tensors only (no CPU path)")
        if num_heads % cache.num_kv_heads != 0:
            raise ValueError(f"num_heads {num_heads} must be divisible by num_kv_heads {cache.num_kv_heads}")
        quant = cache.k_cache.dtype not in (torch.float16, torch.bfloat16)
        if quant and scales is None:
            raise ValueError("DecodeLoop: an int8/fp8 cache needs its scales")
        self.cache = cache
        self.k_scale = None if scales is None else (scales["k"] if isinstance(scales, dict) else scales.k)
        self.v_scale = None if scales is None else (scales["v"] if isinstance(scales, dict) else scales.v)
        self.scale = float(softmax_scale) if softmax_scale is not None else cache.head_dim ** -0.5
        dev = cache.k_cache.device
        self.q_dtype = q_dtype or (torch.float16 if quant else cache.k_cache.dtype)
        self.in_dtype = in_dtype or (self.q_dtype if quant else cache.k_cache.dtype)
        b, hkv, d = cache.batch_size, cache.num_kv_heads, cache.head_dim
        self.q = torch.zeros((b, num_heads, d), dtype=self.q_dtype, device=dev)
        self.new_k = torch.zeros((b, hkv, d), dtype=self.in_dtype, device=dev)
        self.new_v = torch.zeros_like(self.new_k)
        self.out = torch.empty((b, num_heads, d), dtype=self.q_dtype, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = torch.cuda.CUDAGraph()
        # Library, scratch and error word exist before capture (no allocation,
        # no host synchronisation while capturing); the decode kernel is run
        # once eagerly (it does not change the cache).
        _lib.load()
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            self._decode()
        self.stream.synchronize()
        with _config.value_checks(False), torch.cuda.graph(self.graph, stream=self.stream):
            self._append()
            self._decode()
        torch.cuda.current_stream(dev).wait_stream(self.stream)

    def _append(self):
        c = self.cache
        launch_append(c.k_cache, c.v_cache, c.page_table, c.seq_lens, self.new_k, self.new_v, c.page_size,
                      k_scale=self.k_scale, v_scale=self.v_scale)

    def _decode(self):
        c = self.cache
        launch_decode(self.q, c.k_cache, c.v_cache, c.page_table, c.seq_lens, c.page_size, self.scale,
                      k_scale=self.k_scale, v_scale=self.v_scale, out=self.out)

    def step(self, q: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor) -> torch.Tensor:
        """Append (new_k, new_v) at each sequence's end, then attend q over the
        updated cache.  Returns the static output buffer (overwritten by the
        next step)."""
        self.q.copy_(q, non_blocking=True)
        self.new_k.copy_(new_k, non_blocking=True)
        self.new_v.copy_(new_v, non_blocking=True)
        self.graph.replay()
        return self.out

    def replay(self) -> torch.Tensor:
        """Replay with whatever the static buffers ``q``/``new_k``/``new_v`` hold."""
        self.graph.replay()
        return self.out


__all__ = ["DecodeLoop"]
