"""Runs FlashAttnTile's own GPU kernels (its Triton ops) -- test and benchmark infrastructure.

The reference package registers ``torch.ops.flashattn_tile`` just as this
library does, so it runs in a process of its own with the installed reference
(``baseline/_ref``, made by ``pip install --target baseline/_ref`` from the
reference checkout) first on ``sys.path``.  Its kernels fall back to a CPU path
with a warning when Triton or CUDA is missing; here that is an error.

    python tests/ref_triton_runner.py <ref dir> run <inputs.npz> <outputs.npz>
        every case of the inputs file through the reference's kernels
    python tests/ref_triton_runner.py <ref dir> time <steps> <warmup>
        one JSON line: the reference's Triton decode on cfg2 and prefill on cfg3,
        timed like bench.py times this library (CUDA events, back to back)
"""

from __future__ import annotations

import json
import statistics
import sys
import warnings
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]


def _load_reference(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import flashattn_tile  # noqa: F401
    from flashattn_tile.kernels import decode as rdec
    from flashattn_tile.kernels import prefill as rpre

    if not (rdec.HAS_TRITON and rpre.HAS_TRITON):
        raise SystemExit("the reference's Triton kernels are not available (it would fall back to its CPU path)")
    return rdec, rpre


def _tensor(a: np.ndarray, dtype: str) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype == "bf16":
        t = t.view(torch.int16).view(torch.bfloat16)
    elif dtype == "e4m3":
        t = t.view(torch.float8_e4m3fn)
    return t.cuda()


def _storage(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def run_cases(ref_dir: str, inputs: str, outputs: str) -> None:
    rdec, rpre = _load_reference(ref_dir)
    from flashattn_tile.paging import PagedKVCache

    data = np.load(inputs)
    cases = json.loads(str(data["cases"]))
    out = {}
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        for c in cases:
            name, kind, dt = c["name"], c["kind"], c["dtype"]
            a = {k[len(name) + 1:]: data[k] for k in data.files if k.startswith(name + ".")}
            if kind in ("decode", "decode_quant"):
                q = _tensor(a["q"], dt)
                kvdt = c.get("kv_dtype", dt)
                cache = PagedKVCache(k_cache=_tensor(a["k"], kvdt), v_cache=_tensor(a["v"], kvdt),
                                     page_table=_tensor(a["table"], "i32"), seq_lens=_tensor(a["lens"], "i32"),
                                     page_size=int(c["page_size"]))
                cfg = {"split_k": int(c.get("split_k", 1))}
                if kind == "decode":
                    o = rdec.paged_decode_attention(q, cache, softmax_scale=c["scale"], config=cfg)
                else:
                    scales = {"k": _tensor(a["k_scale"], "f32"), "v": _tensor(a["v_scale"], "f32")}
                    o = rdec.paged_decode_attention_fp8(q, cache, scales, softmax_scale=c["scale"], config=cfg)
            else:
                q, k, v = (_tensor(a[n], dt) for n in ("q", "k", "v"))
                cu_q, cu_k = _tensor(a["cu_q"], "i32"), _tensor(a["cu_k"], "i32")
                o = rpre.prefill_attention(q, k, v, cu_q, cu_k, int(c["max_q"]), int(c["max_k"]),
                                           causal=bool(c["causal"]), softmax_scale=c["scale"])
            torch.cuda.synchronize()
            out[name] = _storage(o)
    fallbacks = [str(w.message) for w in caught if "fall" in str(w.message).lower()]
    if fallbacks:
        raise SystemExit(f"the reference fell back to its CPU path: {fallbacks[0]}")
    np.savez(outputs, **out)
    print(json.dumps({"ran": sorted(out)}))


def _time(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    for i in range(steps):
        ev[i].record()
        fn()
    ev[steps].record()
    torch.cuda.synchronize()
    return statistics.mean(ev[i].elapsed_time(ev[i + 1]) for i in range(steps))


def time_cases(ref_dir: str, steps: int, warmup: int) -> None:
    rdec, rpre = _load_reference(ref_dir)
    from flashattn_tile.paging import PagedKVCache

    dev = torch.device("cuda", 0)
    res = {}
    # cfg2: B32, H32/8, D128, ps16, ctx 4096, fp16 (algorithmic bytes as bench.py counts them).
    g = torch.Generator(device=dev).manual_seed(1)
    pool = 32 * 256
    k = torch.randn((pool, 16, 8, 128), generator=g, device=dev).half()
    v = torch.randn((pool, 16, 8, 128), generator=g, device=dev).half()
    q = torch.randn((32, 32, 128), generator=g, device=dev).half()
    table = torch.randperm(pool, generator=g, device=dev).view(32, 256).to(torch.int32)
    lens = torch.full((32,), 4096, dtype=torch.int32, device=dev)
    cache = PagedKVCache(k_cache=k, v_cache=v, page_table=table, seq_lens=lens, page_size=16)
    nbytes = 537_395_200
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        for split in (1, 2, 4, 8):
            ms = _time(lambda: rdec.paged_decode_attention(q, cache, config={"split_k": split}), steps, warmup)
            res[f"cfg2_decode_reference_triton_split{split}"] = {"value": round(nbytes / (ms * 1e-3) / 1e9, 1),
                                                                  "unit": "GB/s", "ms": round(ms, 4)}
        del k, v, cache
        torch.cuda.empty_cache()
        # cfg3: lens {512, 1024, 2048, 4096}, H32/8, D128, causal; two input sets alternated.
        cu = torch.tensor([0, 512, 1536, 3584, 7680], dtype=torch.int32, device=dev)
        flops = 182_599_024_640
        for dt, tag in ((torch.float16, "f16"), (torch.bfloat16, "bf16")):
            sets = [tuple(torch.randn((7680, h, 128), generator=g, device=dev).to(dt) for h in (32, 8, 8))
                    for _ in range(2)]
            state = {"i": 0}

            def step():
                state["i"] += 1
                q3, k3, v3 = sets[state["i"] & 1]
                return rpre.prefill_attention(q3, k3, v3, cu, cu, 4096, 4096, causal=True)

            ms = _time(step, steps, warmup)
            res[f"cfg3_prefill_{tag}_reference_triton"] = {"value": round(flops / (ms * 1e-3) / 1e12, 1),
                                                           "unit": "TFLOP/s", "ms": round(ms, 4)}
            del sets
    fallbacks = [str(w.message) for w in caught if "fall" in str(w.message).lower()]
    if fallbacks:
        raise SystemExit(f"the reference fell back to its CPU path: {fallbacks[0]}")
    print(json.dumps(res))


if __name__ == "__main__":
    ref, mode = sys.argv[1], sys.argv[2]
    if mode == "run":
        run_cases(ref, sys.argv[3], sys.argv[4])
    else:
        time_cases(ref, int(sys.argv[3]), int(sys.argv[4]))
