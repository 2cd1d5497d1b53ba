#!/usr/bin/env python
"""Benchmark of the paged-attention hot path on B200 (one JSON line on rank 0).

Headline workload (BASELINE cfg2): fp16 paged decode, batch 32, 32 query /
8 KV heads, head_dim 128, page_size 16, every sequence at ctx 4096, seeded
N(0,1) K/V/Q, block table a seeded permutation of a 32x256-page pool.
metric = decode HBM GB/s = algorithmic bytes (Q + K + V + O, FlashAttnTile's
``bytes_attention("decode")``) / device time.

* ``value``: K launches run back to back with inputs resident in HBM (537 MB
  per step, 4x the 126 MB L2, so no step finds its inputs in L2 and no flush
  is needed), CUDA events around each step on the launching stream, max over
  ranks.
* ``e2e``: the same step through the public op ``torch.ops.flashattn_tile.paged_decode``
  as a serving step calls it -- the per-step inputs (q, page table, seq_lens)
  copied from pinned host memory, the default host-side validation, the output
  copied back to pinned host memory -- with the KV cache resident on the GPU.
* ``cpu_baseline``: the numpy restatement of the reference's fp32 path
  (oracle/) on the same cfg2 inputs, timed on this host's cores.
* ``secondary``: the other hot-path kernels measured the same way (quantised
  decode cfg4 and varlen prefill cfg3 at N=1; the cfg5 long-context decode
  split by page range across the N ranks, with its NCCL exchange and LSE
  merge, at every N).

Multi-GPU (torchrun, one rank per GPU): decode shards by (sequence, KV head)
with no communication; every rank owns a cfg2-sized shard (weak scaling) and
``value`` is the bytes of all ranks over the slowest rank's time.

``--impl reference`` times the reference arm instead: the oracle port of the
reference's fp32 CPU path on rank 0 with all host threads, one bounded sample
of cfg2 (8 of the 32 sequences) per step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

CFG2 = dict(batch=32, heads=32, kv_heads=8, head_dim=128, page_size=16, ctx=4096)
# dram__bytes_read.sum + dram__bytes_write.sum of one decode launch at cfg2 from the
# committed ncu capture (profiles/decode_sm100_cfg2.md: 537.72 MB read + 4.23 MB written).
NCU_TRAFFIC_BYTES = {"decode_cfg2": 541011712}  # dram read + write of one launch, profiles/decode_sm100_cfg2.md


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU through NVML."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:  # NVML missing: report no clocks rather than fail the bench
            self._nvml = None
        self.period = period_s

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(int(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)))
                self.reasons |= int(n.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict | None:
        if self._nvml is None or not self.samples:
            return None
        names = [v for k, v in self.REASONS.items() if self.reasons & k and v != "gpu_idle"]
        return {"sm_mhz": int(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# --------------------------------------------------------------------------- workloads
def make_decode_cfg2(device, seed: int, dtype=torch.float16):
    c = CFG2
    gen = torch.Generator(device=device).manual_seed(seed)
    pages_per_seq = c["ctx"] // c["page_size"]
    pool = c["batch"] * pages_per_seq
    shape = (pool, c["page_size"], c["kv_heads"], c["head_dim"])
    k = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)
    v = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)
    q = torch.randn((c["batch"], c["heads"], c["head_dim"]), generator=gen, device=device).to(dtype)
    table = torch.randperm(pool, generator=gen, device=device).view(c["batch"], pages_per_seq).to(torch.int32)
    lens = torch.full((c["batch"],), c["ctx"], dtype=torch.int32, device=device)
    return q, k, v, table, lens


def decode_bytes(lens, heads, kv_heads, head_dim, page_size, elem=2, scale_bytes=0):
    from flashattntile_b200.autotune import bytes_decode_paged

    return bytes_decode_paged(lens, heads, kv_heads, head_dim, page_size, q_bytes=2, kv_bytes=elem,
                              scale_bytes=scale_bytes)


def time_steps(fn, steps: int, warmup: int, flush: torch.Tensor | None) -> list[float]:
    """Per-step device milliseconds of fn() (CUDA events on the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


# --------------------------------------------------------------------------- CPU arms
def cpu_decode_rate(q, k, v, table, lens, seqs: int, iters: int, threads: int) -> tuple[float, float, str]:
    """Oracle (numpy port of the reference fp32 path) on the first `seqs` sequences."""
    import numpy as np

    from oracle import attention as oatt

    qn = q[:seqs].cpu().numpy()
    tn = table[:seqs].cpu().numpy()
    ln = lens[:seqs].cpu().numpy()
    used = np.unique(tn.reshape(-1))
    # Only the pages the sample reads are copied to the host.
    remap = np.full(int(k.shape[0]), -1, dtype=np.int64)
    remap[used] = np.arange(used.size)
    idx = torch.from_numpy(used).to(k.device)
    kn = k.index_select(0, idx).cpu().numpy()
    vn = v.index_select(0, idx).cpu().numpy()
    tn = remap[tn].astype(np.int32)
    nbytes = decode_bytes(ln.tolist(), q.shape[1], k.shape[2], k.shape[3], k.shape[1])
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        oatt.attention_paged(qn, kn, vn, tn, ln, int(k.shape[1]), dtype="f16", threads=threads)
        times.append(time.perf_counter() - t0)
    best = min(times)
    sample = f"cfg2 sequences 0..{seqs - 1} ({seqs} x ctx {int(ln[0])}), fp16 inputs upcast to fp32, min of {iters}"
    return nbytes / best / 1e9, best, sample


# --------------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--only", choices=["decode", "quant", "prefill", "longctx", "loop", "comparators"], default=None,
                    help="run one workload (profiling); decode = the headline line without secondary; "
                         "comparators = library kernels on cfg2/cfg3 beside ours (never in the default run)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import datetime

    import flashattntile_b200  # noqa: F401
    from flashattntile_b200 import _lib
    from flashattntile_b200.kernels.decode import launch_decode

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    peaks = _peaks()
    if args.only in ("quant", "prefill", "longctx", "loop", "comparators"):
        res = run_secondary(device, args, peaks, which=(args.only,), dist=dist)
        if rank == 0:
            print(json.dumps({"only": args.only, "steps": args.steps, "warmup": args.warmup, "results": res}),
                  flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.only == "decode":
        args.no_secondary = True
    c = CFG2
    q, k, v, table, lens = make_decode_cfg2(device, seed=1 + rank)
    lens_list = [c["ctx"]] * c["batch"]
    nbytes = decode_bytes(lens_list, c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])
    scale = c["head_dim"] ** -0.5
    out = torch.empty_like(q)

    def step():
        launch_decode(q, k, v, table, lens, c["page_size"], scale, 1, out=out)

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        times = time_steps(step, args.steps, args.warmup, None)
    torch.cuda.synchronize()
    total_ms = sum(times)
    if dist is not None:
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    ms_per_step = total_ms / args.steps
    value = world * nbytes / (ms_per_step * 1e-3) / 1e9
    kernel_ms = statistics.mean(times)
    achieved = nbytes / (kernel_ms * 1e-3) / 1e9
    dev_err = _lib.read_device_error(device)

    # ---- e2e through the public op with host buffers ----
    q_h = q.cpu().pin_memory()
    t_h = table.cpu().pin_memory()
    l_h = lens.cpu().pin_memory()
    o_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_d, t_d, l_d = torch.empty_like(q), torch.empty_like(table), torch.empty_like(lens)

    def e2e_step():
        q_d.copy_(q_h, non_blocking=True)
        t_d.copy_(t_h, non_blocking=True)
        l_d.copy_(l_h, non_blocking=True)
        o = torch.ops.flashattn_tile.paged_decode(q_d, k, v, t_d, l_d, c["page_size"], scale, 1)
        o_h.copy_(o, non_blocking=True)

    e2e_times = time_steps(e2e_step, max(10, args.steps // 2), args.warmup, None)
    e2e_ms = sum(e2e_times) / len(e2e_times)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = q.numel() * q.element_size() + table.numel() * 4 + lens.numel() * 4
    d2h = q.numel() * q.element_size()
    e2e_ok = torch.allclose(o_h.to(device).float(), out.float(), atol=0, rtol=0)

    secondary = {}
    if not args.no_secondary:
        which = ("quant", "prefill", "longctx", "loop") if world == 1 else ("longctx",)
        secondary = run_secondary(device, args, peaks, which=which, dist=dist)
    if dist is not None:
        dist.barrier()

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            threads = os.cpu_count() or 1
            rate, best, sample = cpu_decode_rate(q, k, v, table, lens, c["batch"], 3, threads)
            cpu = {"value": round(rate, 4), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
                   "seconds_per_call": round(best, 4)}
        traffic = NCU_TRAFFIC_BYTES["decode_cfg2"]
        line = {
            "metric": "decode HBM GB/s (cfg2: fp16 paged decode B32 ctx4096 H32/8 D128 ps16)",
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate)",
            "data": "synthetic N(0,1), seeded per rank",
            "config": {"workload": "cfg2 paged decode", "batch_per_gpu": c["batch"], "global_batch": c["batch"] * world,
                       "ctx": c["ctx"], "heads": c["heads"], "kv_heads": c["kv_heads"], "head_dim": c["head_dim"],
                       "page_size": c["page_size"], "parallelism": f"shard (sequence, kv-head) x{world}, no comm",
                       "l2": "inputs 537 MB per step > 126 MB L2; steps back to back, no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"] + " copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic, "algorithmic_bytes": nbytes, "kernel_ms": round(kernel_ms, 5)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "torch.ops.flashattn_tile.paged_decode, default validation, pinned host q/table/lens/out",
                    "matches_device_path": bool(e2e_ok)},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "device_error_word": dev_err,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_secondary(device, args, peaks, which=("quant", "prefill", "longctx", "loop"), dist=None) -> dict:
    """Quantised decode (cfg4), varlen prefill (cfg3), long-context decode (cfg5), decode loop."""
    res = {}
    if "loop" in which:
        res.update(run_decode_loop(device, args))
    if "quant" in which:
        res.update(run_quant(device, args, peaks))
    if "prefill" in which:
        res.update(run_prefill(device, args, peaks))
    if "longctx" in which:
        res.update(run_longctx(device, args, peaks, dist))
    if "comparators" in which:
        res.update(run_comparators(device, args, peaks))
    return res


def run_comparators(device, args, peaks) -> dict:
    """Same-box library kernels beside ours, reported, not targets: flashinfer's
    trtllm-gen and fa2 (tensor-core) paged decode on cfg2, torch SDPA (one call per
    sequence, GQA) and flash_attn 2 varlen on cfg3.  Timed like our kernels
    (CUDA events, cfg3 alternating two input sets); each also reports its largest
    difference from our output.  A library that fails to run is reported with
    its error.  First calls may JIT-compile, outside the timed region."""
    from flashattntile_b200.autotune import flops_attention_varlen
    from flashattntile_b200.kernels.decode import launch_decode
    from flashattntile_b200.kernels.prefill import launch_prefill

    res = {}
    steps = max(20, args.steps // 2)
    c = CFG2
    q, k, v, table, lens = make_decode_cfg2(device, seed=1)
    nbytes = decode_bytes([c["ctx"]] * c["batch"], c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])
    scale = c["head_dim"] ** -0.5
    ours = launch_decode(q, k, v, table, lens, c["page_size"], scale, 1)
    out = torch.empty_like(q)

    def record(name, fn, ref, work, unit):
        try:
            o = fn()
            torch.cuda.synchronize()
            diff = float((o.float() - ref.float()).abs().max())
            ms = statistics.mean(time_steps(fn, steps, args.warmup, None))
            val = work / (ms * 1e-3) / (1e9 if unit == "GB/s" else 1e12)
            res[name] = {"value": round(val, 1), "unit": unit, "ms": round(ms, 4), "maxdiff_vs_ours": diff}
        except Exception as e:  # a library missing or failing on this box
            res[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}

    record("cfg2_decode_ours", lambda: launch_decode(q, k, v, table, lens, c["page_size"], scale, 1, out=out),
           ours, nbytes, "GB/s")
    try:
        import flashinfer

        ws = torch.zeros(256 << 20, dtype=torch.uint8, device=device)
        record("cfg2_decode_flashinfer_trtllm_gen",
               lambda: flashinfer.decode.trtllm_batch_decode_with_kv_cache(
                   q, (k, v), ws, table, lens, c["ctx"], bmm1_scale=scale, bmm2_scale=1.0, kv_layout="NHD"),
               ours, nbytes, "GB/s")
        B, P = table.shape
        w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD", use_tensor_cores=True)
        w.plan(torch.arange(B + 1, device=device, dtype=torch.int32) * P, table.reshape(-1).contiguous(),
               torch.full((B,), c["page_size"], dtype=torch.int32, device=device), c["heads"], c["kv_heads"],
               c["head_dim"], c["page_size"], q_data_type=q.dtype, kv_data_type=k.dtype, sm_scale=scale)
        record("cfg2_decode_flashinfer_fa2_tc", lambda: w.run(q, (k, v)), ours, nbytes, "GB/s")
    except Exception as e:
        res["cfg2_decode_flashinfer"] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    del q, k, v, table, lens, ours, out

    lens3 = [512, 1024, 2048, 4096]
    flops = flops_attention_varlen(32, 128, lens3, lens3, causal=True)
    offs = [0] + torch.tensor(lens3).cumsum(0).tolist()
    cu = torch.tensor(offs, dtype=torch.int32, device=device)
    g3 = torch.Generator(device=device).manual_seed(2)
    sets = []
    for _ in range(2):
        sets.append(tuple(torch.randn((offs[-1], h, 128), generator=g3, device=device).half() for h in (32, 8, 8)))
    ref3 = launch_prefill(*sets[1], cu, cu, 4096, 4096, True, 128 ** -0.5)
    def alternate(call):
        state = {"i": 0}  # the first call uses sets[1], the set ref3 was computed on

        def fn():
            state["i"] += 1
            return call(*sets[state["i"] & 1])
        return fn

    o3 = torch.empty_like(sets[0][0])
    record("cfg3_prefill_ours", alternate(lambda q3, k3, v3: launch_prefill(q3, k3, v3, cu, cu, 4096, 4096, True,
                                                                            128 ** -0.5, out=o3)),
           ref3, flops, "TFLOP/s")

    def sdpa(q3, k3, v3):
        import torch.nn.functional as F

        outs = []
        for a, b in zip(offs[:-1], offs[1:]):
            o = F.scaled_dot_product_attention(q3[a:b].transpose(0, 1)[None], k3[a:b].transpose(0, 1)[None],
                                               v3[a:b].transpose(0, 1)[None], is_causal=True, scale=128 ** -0.5,
                                               enable_gqa=True)
            outs.append(o[0].transpose(0, 1))
        return torch.cat(outs)

    record("cfg3_prefill_torch_sdpa", alternate(sdpa), ref3, flops, "TFLOP/s")
    try:
        from flash_attn import flash_attn_varlen_func

        record("cfg3_prefill_flash_attn2",
               alternate(lambda q3, k3, v3: flash_attn_varlen_func(q3, k3, v3, cu, cu, 4096, 4096,
                                                                   softmax_scale=128 ** -0.5, causal=True)),
               ref3, flops, "TFLOP/s")
    except Exception as e:
        res["cfg3_prefill_flash_attn2"] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    return res


def run_decode_loop(device, args) -> dict:
    """Per-token latency of a serving decode iteration at cfg2 shapes (B32, H32/8,
    D128, ps16, contexts ~3.8-4k): append the step's K/V, attend, read the output
    back.  Three ways: the reference's flow (custom op + append_tokens with the
    default host-side value checks), the same without value checks, and one
    CUDA-graph replay of both kernels (DecodeLoop).  Host wall time per step,
    synchronised every step as a sampler would be."""
    from flashattntile_b200 import value_checks
    from flashattntile_b200.decode_loop import DecodeLoop
    from flashattntile_b200.paging import PagedKVCache, append_tokens

    c = CFG2
    b, h, hkv, d, ps = c["batch"], c["heads"], c["kv_heads"], c["head_dim"], c["page_size"]
    pages = 4160 // ps
    gen = torch.Generator(device=device).manual_seed(9)
    pool = b * pages
    k = torch.randn((pool, ps, hkv, d), generator=gen, device=device).half()
    v = torch.randn((pool, ps, hkv, d), generator=gen, device=device).half()
    table = torch.randperm(pool, generator=gen, device=device).view(b, pages).to(torch.int32)
    cache = PagedKVCache(k, v, table, torch.full((b,), 3800, dtype=torch.int32, device=device), ps)
    q = torch.randn((b, h, d), generator=gen, device=device).half()
    nk = torch.randn((b, hkv, d), generator=gen, device=device).half()
    nv = torch.randn_like(nk)
    scale = d ** -0.5
    n = 50

    def eager():
        append_tokens(cache, nk, nv)
        return torch.ops.flashattn_tile.paged_decode(q, cache.k_cache, cache.v_cache, cache.page_table,
                                                     cache.seq_lens, ps, scale, 1)

    def wall(fn, steps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            out = fn()
            out.view(-1)[0].item()  # the sampler reads the step's result
            times.append(time.perf_counter() - t0)
        return statistics.median(times) * 1e6

    checked = wall(eager, n)
    with value_checks(False):
        unchecked = wall(eager, n)
    loop = DecodeLoop(cache, h)
    graphed = wall(lambda: loop.step(q, nk, nv), 2 * n)
    del loop
    return {"decode_loop_cfg2": {
        "unit": "us/step (median host wall, synchronised each step)", "batch": b,
        "reference_flow_us": round(checked, 1), "no_value_checks_us": round(unchecked, 1),
        "cuda_graph_us": round(graphed, 1), "cuda_graph_tokens_per_s": round(b / (graphed * 1e-6), 1),
        "step": "append K/V (device kernel) + paged decode; graph = both kernels in one replay"}}


CFG5 = dict(batch=8, heads=64, kv_heads=8, head_dim=128, page_size=64, ctx=131072)


def run_longctx(device, args, peaks, dist=None) -> dict:
    """cfg5: B8, H64/8, D128, ps64, ctx 131072 fp16, pages split by range over the ranks.

    Every rank holds logical pages [p0, p1) of every sequence in its own pool
    (strong scaling: the total cache is fixed, 4.3 GB).  A step is the local
    decode into fp32 partials, the NCCL all-gather of the packed partials and
    the LSE merge; the time is the slowest rank's.  The metric counts the
    whole job's algorithmic bytes (all ranks' K/V plus Q and O once)."""
    from flashattntile_b200 import sequence_parallel as sp
    from flashattntile_b200.paging import PagedKVCache

    c = CFG5
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    pages_per_seq = c["ctx"] // c["page_size"]
    p0, p1 = sp.page_range(pages_per_seq, world, rank)
    local_pages = p1 - p0
    pool = c["batch"] * local_pages
    shape = (pool, c["page_size"], c["kv_heads"], c["head_dim"])
    gen = torch.Generator(device=device).manual_seed(50 + rank)
    k = torch.empty(shape, dtype=torch.float16, device=device)
    v = torch.empty_like(k)
    for i in range(0, pool, 1024):
        k[i:i + 1024].normal_(generator=gen)
        v[i:i + 1024].normal_(generator=gen)
    gq = torch.Generator(device=device).manual_seed(49)  # same q on every rank
    q = torch.randn((c["batch"], c["heads"], c["head_dim"]), generator=gq, device=device).half()
    table = torch.randperm(pool, generator=gen, device=device).view(c["batch"], local_pages).to(torch.int32)
    full_lens = torch.full((c["batch"],), c["ctx"], dtype=torch.int32, device=device)
    cache = PagedKVCache(k, v, table, sp.local_lengths(full_lens, c["page_size"], p0, p1), c["page_size"])
    packed = torch.empty(sp.packed_size(c["batch"], c["heads"], c["head_dim"]), dtype=torch.float32, device=device)
    parts = torch.empty((world, packed.numel()), dtype=torch.float32, device=device)
    out = torch.empty_like(q)
    total_bytes = decode_bytes([c["ctx"]] * c["batch"], c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])

    def step():
        sp.decode_partial(q, cache, packed=packed)
        if dist is not None:
            sp.exchange_partials(packed, out=parts)
        else:
            parts.copy_(packed.view(1, -1))
        sp.merge_partials(parts, c["batch"], c["heads"], c["head_dim"], torch.float16, out=out)

    from flashattntile_b200._config import value_checks

    steps = max(10, args.steps // 2)
    with value_checks(False):  # no host syncs inside the timed loop
        if dist is not None:
            dist.barrier()
        times = time_steps(step, steps, args.warmup, None)
        decode_times = time_steps(lambda: sp.decode_partial(q, cache, packed=packed), steps, args.warmup, None)
    ms, dms = statistics.mean(times), statistics.mean(decode_times)
    if dist is not None:
        t = torch.tensor([ms, dms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, dms = (float(x) for x in t.tolist())
    local_bytes = decode_bytes([c["ctx"] // world] * c["batch"], c["heads"], c["kv_heads"], c["head_dim"],
                               c["page_size"])
    del k, v, cache
    torch.cuda.empty_cache()
    return {"cfg5_longctx_decode": {
        "value": round(total_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms": round(ms, 4), "n_gpus": world,
        "scaling": "strong", "algorithmic_bytes": total_bytes,
        "local_decode_ms": round(dms, 4),
        "local_decode_frac_hbm": round(local_bytes / (dms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        "exchange_bytes_per_rank": packed.numel() * 4,
        "step": "decode partial + NCCL all_gather_into_tensor + LSE merge" if world > 1
                else "decode partial + LSE merge (1 part)"}}


def run_quant(device, args, peaks) -> dict:
    """cfg4: B128, H32/8, D128, ps32, ctx U[1024, 16384], INT8 and e4m3 caches."""
    from flashattntile_b200 import quant
    from flashattntile_b200.kernels.decode import launch_decode

    res = {}
    gen = torch.Generator(device="cpu").manual_seed(3)
    batch, heads, kvh, dim, ps = 128, 32, 8, 128, 32
    ctx = torch.randint(1024, 16385, (batch,), generator=gen)
    pages = [math.ceil(int(n) / ps) for n in ctx]
    pool = sum(pages)
    g2 = torch.Generator(device=device).manual_seed(3)
    perm = torch.randperm(pool, generator=g2, device=device).to(torch.int32)
    table = torch.zeros((batch, max(pages)), dtype=torch.int32, device=device)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    lens = ctx.to(torch.int32).to(device)
    q = torch.randn((batch, heads, dim), generator=g2, device=device).half()
    for mode in ("int8", "float8_e4m3fn"):
        kq = torch.empty((pool, ps, kvh, dim), dtype=torch.int8 if mode == "int8" else torch.float8_e4m3fn,
                         device=device)
        vq = torch.empty_like(kq)
        ks = torch.empty((pool, kvh), dtype=torch.float32, device=device)
        vs = torch.empty_like(ks)
        step_pages = 4096
        for p0 in range(0, pool, step_pages):
            p1 = min(pool, p0 + step_pages)
            kf = torch.randn((p1 - p0, ps, kvh, dim), generator=g2, device=device)
            vf = torch.randn((p1 - p0, ps, kvh, dim), generator=g2, device=device)
            a, b_, sa, sb, _ = quant.quantize_kv_pages(kf, vf, mode=mode)
            kq[p0:p1], vq[p0:p1], ks[p0:p1], vs[p0:p1] = a, b_, sa, sb
        out = torch.empty_like(q)
        nbytes = decode_bytes(ctx.tolist(), heads, kvh, dim, ps, elem=1, scale_bytes=4)

        def step():
            launch_decode(q, kq, vq, table, lens, ps, dim ** -0.5, 1, k_scale=ks, v_scale=vs, out=out)

        times = time_steps(step, max(10, args.steps // 2), args.warmup, None)
        ms = statistics.mean(times)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[f"cfg4_decode_{mode}"] = {"value": round(gbs, 1), "unit": "GB/s", "ms": round(ms, 4),
                                      "algorithmic_bytes": nbytes, "frac_hbm": round(gbs / peaks["hbm_gbs"], 4)}
        del kq, vq, ks, vs
    torch.cuda.empty_cache()
    return res


def run_prefill(device, args, peaks) -> dict:
    """cfg3: varlen causal prefill, lens {512, 1024, 2048, 4096}, H32/8, D128, fp16 and bf16."""
    from flashattntile_b200.autotune import flops_attention_varlen
    from flashattntile_b200.kernels.prefill import launch_prefill

    res = {}
    lens = [512, 1024, 2048, 4096]
    flops = flops_attention_varlen(32, 128, lens, lens, causal=True)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=device)
    g3 = torch.Generator(device=device).manual_seed(2)
    for dt in (torch.float16, torch.bfloat16):
        # Two input sets used alternately: 2 x 157 MB > L2, so no step reuses L2-resident inputs.
        sets = []
        for _ in range(2):
            q3 = torch.randn((sum(lens), 32, 128), generator=g3, device=device).to(dt)
            k3 = torch.randn((sum(lens), 8, 128), generator=g3, device=device).to(dt)
            v3 = torch.randn((sum(lens), 8, 128), generator=g3, device=device).to(dt)
            sets.append((q3, k3, v3, torch.empty_like(q3)))
        state = {"i": 0}

        def pstep():
            q3, k3, v3, o3 = sets[state["i"] & 1]
            state["i"] += 1
            launch_prefill(q3, k3, v3, cu, cu, 4096, 4096, True, 128 ** -0.5, out=o3)

        times = time_steps(pstep, max(10, args.steps // 2), args.warmup, None)
        ms = statistics.mean(times)
        tflops = flops / (ms * 1e-3) / 1e12
        res[f"cfg3_prefill_{'f16' if dt == torch.float16 else 'bf16'}"] = {
            "value": round(tflops, 1), "unit": "TFLOP/s", "ms": round(ms, 4), "algorithmic_flops": flops,
            "frac_tensor": round(tflops / peaks["bf16_tflops"], 4),
            "peak_source": "measured cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops)"}
        del sets
    # The same cfg3 prefill with K/V read through a page table (ps 16, permuted pages).
    from flashattntile_b200.kernels.prefill import prefill_paged_attention
    from flashattntile_b200.paging import PagedKVCache

    ps = 16
    pages = [n // ps for n in lens]
    pool = sum(pages)
    table = torch.zeros((len(lens), max(pages)), dtype=torch.int32, device=device)
    perm = torch.randperm(pool, generator=g3, device=device).to(torch.int32)
    off = 0
    for i, n in enumerate(pages):
        table[i, :n] = perm[off:off + n]
        off += n
    caches = []
    for _ in range(2):
        kc = torch.randn((pool, ps, 8, 128), generator=g3, device=device).half()
        vc = torch.randn((pool, ps, 8, 128), generator=g3, device=device).half()
        q3 = torch.randn((sum(lens), 32, 128), generator=g3, device=device).half()
        caches.append((q3, PagedKVCache(kc, vc, table, torch.tensor(lens, dtype=torch.int32, device=device), ps)))
    state = {"i": 0}

    def ppstep():
        q3, cache = caches[state["i"] & 1]
        state["i"] += 1
        prefill_paged_attention(q3, cache, cu, 4096, causal=True)

    from flashattntile_b200._config import value_checks

    with value_checks(False):
        times = time_steps(ppstep, max(10, args.steps // 2), args.warmup, None)
    ms = statistics.mean(times)
    tflops = flops / (ms * 1e-3) / 1e12
    res["cfg3_prefill_paged_f16_ps16"] = {
        "value": round(tflops, 1), "unit": "TFLOP/s", "ms": round(ms, 4), "algorithmic_flops": flops,
        "frac_tensor": round(tflops / peaks["bf16_tflops"], 4), "page_size": ps}
    del caches
    torch.cuda.empty_cache()
    return res


def run_reference_arm(args, rank: int, world: int) -> None:
    """Reference CPU path (oracle port of reference.py fp32) on rank 0 only."""
    if rank != 0:
        return
    import numpy as np

    from oracle import attention as oatt

    c = CFG2
    seqs = 8
    gen = torch.Generator().manual_seed(1)
    pages_per_seq = c["ctx"] // c["page_size"]
    shape = (seqs * pages_per_seq, c["page_size"], c["kv_heads"], c["head_dim"])
    k = torch.randn(shape, generator=gen).half().numpy()
    v = torch.randn(shape, generator=gen).half().numpy()
    q = torch.randn((seqs, c["heads"], c["head_dim"]), generator=gen).half().numpy()
    table = torch.randperm(shape[0], generator=gen).view(seqs, pages_per_seq).to(torch.int32).numpy()
    lens = np.full(seqs, c["ctx"], dtype=np.int32)
    threads = os.cpu_count() or 1
    nbytes = decode_bytes(lens.tolist(), c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])
    for _ in range(args.warmup):
        oatt.attention_paged(q, k, v, table, lens, c["page_size"], dtype="f16", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oatt.attention_paged(q, k, v, table, lens, c["page_size"], dtype="f16", threads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    value = nbytes / dt / 1e9
    sample = f"cfg2 sequences 0..{seqs - 1} of 32 (ctx 4096), fp16 inputs upcast to fp32 per step"
    print(json.dumps({
        "impl": "reference",
        "metric": "decode HBM GB/s (cfg2: fp16 paged decode B32 ctx4096 H32/8 D128 ps16)",
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": "cfg2 paged decode", "batch": c["batch"], "ctx": c["ctx"], "heads": c["heads"],
                   "kv_heads": c["kv_heads"], "head_dim": c["head_dim"], "page_size": c["page_size"]},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
