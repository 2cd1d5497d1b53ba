"""Prefill captured into CUDA graphs.

A stream that ran a prefill before capture already has its per-stream state
(the persistent grid's work counters; for bf16 the fp16 copy of V): its graph
replays the same kernels and must give bitwise the eager result, replay after
replay (the counters are zeroed again by every launch's last CTA).  A stream
first seen while it is being captured cannot get that state (no allocation
during capture), so it runs one CTA per item and, for bf16, feeds P as head +
remainder; its replays must still match the fp32 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import TAG, assert_close_f32, to_np, varlen_case

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashattntile_b200  # noqa: F401


def _inputs(seed, dtype):
    lens = [700, 33, 1500, 1]
    q, k, v, cu_q, cu_k = varlen_case(seed, lens, lens, 16, 4, 128, dtype)
    dev = [t.to(DEV) for t in (q, k, v, cu_q, cu_k)]
    return (q, k, v, cu_q, cu_k), dev, max(lens)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_graph_on_a_warmed_stream_equals_eager(dtype):
    from flashattntile_b200.kernels.prefill import launch_prefill

    _, (q, k, v, cu_q, cu_k), m = _inputs(400, dtype)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    out = torch.empty(q.shape, dtype=torch.float32, device=DEV)
    with torch.cuda.stream(s):
        launch_prefill(q, k, v, cu_q, cu_k, m, m, True, 128 ** -0.5, out=out)
        s.synchronize()
        want = out.clone()
        out.zero_()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            launch_prefill(q, k, v, cu_q, cu_k, m, m, True, 128 ** -0.5, out=out)
        for _ in range(3):
            out.zero_()
            g.replay()
            s.synchronize()
            assert torch.equal(out, want)
    del g


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_graph_on_a_stream_first_seen_in_capture_matches_oracle(dtype):
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.prefill import launch_prefill, p_precision, schedule

    (hq, hk, hv, hcq, hck), (q, k, v, cu_q, cu_k), m = _inputs(401, dtype)
    want = oatt.attention_varlen(to_np(hq), to_np(hk), to_np(hv), to_np(hcq), to_np(hck), True, dtype=TAG[dtype],
                                 out_f32=True)
    # The kernels the capture falls back to, run once on another stream first: a
    # kernel's first launch on a device sets its shared-memory limit, which is
    # not a call to make inside a capture.
    with schedule("per_item"), p_precision("adaptive" if dtype == torch.bfloat16 else "rounded"):
        launch_prefill(q, k, v, cu_q, cu_k, m, m, True, 128 ** -0.5)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()  # never used before the capture below
    s.wait_stream(torch.cuda.current_stream())
    out = torch.empty(q.shape, dtype=torch.float32, device=DEV)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            launch_prefill(q, k, v, cu_q, cu_k, m, m, True, 128 ** -0.5, out=out)
        for _ in range(2):
            out.fill_(float("nan"))
            g.replay()
            s.synchronize()
            assert_close_f32(out, want)
        assert _lib.read_device_error(torch.device(DEV, torch.cuda.current_device())) == 0
    assert np.isfinite(out.cpu().numpy()).all()
    del g
