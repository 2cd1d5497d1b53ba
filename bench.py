#!/usr/bin/env python
"""Benchmark of the paged-attention hot path on B200 (one JSON line on rank 0).

Headline workload (BASELINE cfg2): fp16 paged decode, batch 32, 32 query /
8 KV heads, head_dim 128, page_size 16, every sequence at ctx 4096, seeded
N(0,1) K/V/Q, block table a seeded permutation of a 32x256-page pool.
metric = decode HBM GB/s = algorithmic bytes (Q + K + V + O, FlashAttnTile's
``bytes_attention("decode")``) / device time.

* ``value``: K launches back to back with inputs resident in HBM (537 MB per
  step per GPU, 4x the 126 MB L2, so no step finds its inputs in L2 and no
  flush is needed), CUDA events around each step on the launching stream, max
  over ranks.
* ``e2e``: the same step through the public op
  ``torch.ops.flashattn_tile.paged_decode`` as a serving loop calls it: every
  step's inputs (q, page table, seq_lens) packed in one pinned host buffer
  and uploaded in one copy on a copy stream (two input sets, so uploads run
  ahead of the kernels), the default host-side validation, and the output
  copied back to pinned host memory on the same copy stream; the KV cache
  stays resident.
  Timed on the device from the first upload to the last download.
* ``cpu_baseline``: the numpy restatement of the reference's fp32 path
  (``oracle/``) on the whole cfg2 batch, timed on this host's cores.
* ``secondary``: the other hot-path kernels measured the same way, each with
  its own ``roofline``, ``e2e`` through its op and (N=1) ``cpu_baseline``:
  quantised decode cfg4, varlen prefill cfg3 (N=1), the cfg5 long-context
  decode, the decode loop (N=1).

Multi-GPU (torchrun, one rank per GPU): decode shards by KV head first
(``flashattntile_b200.sharding``), then by sequence, with no communication.
The global problem at N GPUs is cfg2's geometry with batch 32 N; rank r holds
only its slice of the cache (8 / N KV heads of all 32 N sequences at N <= 8),
so every GPU carries a cfg2-sized share (weak scaling) and ``value`` is the
bytes of all ranks over the slowest rank's time.  cfg5 (fixed 4.3 GB, strong
scaling) shards by KV head as well; a page-split variant, whose partials meet
their owners in one all-to-all and merge by log-sum-exp, is reported beside it.

``--impl reference`` times the reference arm instead: the oracle port of the
reference's fp32 CPU path (``oracle/``) on rank 0 with all host threads, the
whole cfg2 batch per step.  It never loads this library.
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
CFG4 = dict(batch=128, heads=32, kv_heads=8, head_dim=128, page_size=32, ctx_lo=1024, ctx_hi=16384)
CFG5 = dict(batch=8, heads=64, kv_heads=8, head_dim=128, page_size=64, ctx=131072)
CFG3_LENS = [512, 1024, 2048, 4096]
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one cfg2 decode launch,
# copied from an ncu capture of the current kernel (537.279744 MB read + 4.544256 MB
# written); ncu does not run inside this benchmark, so the figure is a recorded constant.
NCU_TRAFFIC_BYTES = {"decode_cfg2": 541_824_000}


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


# --------------------------------------------------------------------------- helpers
def decode_bytes(lens, heads, kv_heads, head_dim, page_size, elem=2, scale_bytes=0) -> int:
    from flashattntile_b200.autotune import bytes_decode_paged

    return bytes_decode_paged(lens, heads, kv_heads, head_dim, page_size, q_bytes=2, kv_bytes=elem,
                              scale_bytes=scale_bytes)


def time_steps(fn, steps: int, warmup: int, flush: torch.Tensor | None = None) -> list[float]:
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


def max_over_ranks(values: list[float], device, dist) -> list[float]:
    if dist is None:
        return values
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def roofline(bound: str, work: float, ms: float, peaks: dict, **extra) -> dict:
    """Roofline block: achieved = algorithmic work per launch / mean launch time."""
    if bound == "hbm":
        achieved, peak, unit, src = work / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s", "copy bandwidth (hbm_gbs)"
    else:
        achieved, peak, unit, src = (work / (ms * 1e-3) / 1e12, peaks["bf16_tflops"], "TFLOP/s",
                                     "cuBLAS bf16 burst (bf16_tflops)")
    out = {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": unit,
           "frac": round(achieved / peak, 4), "peak_source": f"{peaks['source']} {src}",
           "algorithmic": int(work), "kernel_ms": round(ms, 5)}
    out.update(extra)
    return out


def e2e_pipelined(device, steps: int, warmup: int, host_in: list, dev_sets: list, run, out_like: torch.Tensor,
                  views: list | None = None):
    """Device ms per step of ``run(inputs) -> output`` with every step's inputs
    uploaded from pinned host memory and its output read back to pinned host
    memory, inside the timed region.

    Two device input sets alternate: once step i's compute has finished, one
    copy stream reads its output back and uploads step i+2's inputs into the
    set step i used, so uploads and downloads overlap the next step's compute.
    The region starts before the first upload and ends after the last
    download.  ``views`` (per input set): what ``run`` gets instead of the set's
    buffers (views into one packed buffer: one copy per step).  Returns (median
    ms per step of three timed passes after a warm-up pass, last output on the
    host)."""
    comp = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    host_out = [torch.empty(out_like.shape, dtype=out_like.dtype).pin_memory() for _ in range(2)]

    def one_pass(n: int) -> float:
        ready = [torch.cuda.Event() for _ in range(n)]
        used = [torch.cuda.Event() for _ in range(n)]
        outs = []  # kept until the end of the pass: no output is freed under a pending copy
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(comp)
        with torch.cuda.stream(copy):
            copy.wait_event(start)
            for i in range(min(2, n)):
                for h, d in zip(host_in, dev_sets[i]):
                    d.copy_(h, non_blocking=True)
                ready[i].record(copy)
        for i in range(n):
            comp.wait_event(ready[i])
            o = run(dev_sets[i % 2] if views is None else views[i % 2])
            used[i].record(comp)
            outs.append(o)
            with torch.cuda.stream(copy):
                copy.wait_event(used[i])
                host_out[i % 2].copy_(o, non_blocking=True)
                if i + 2 < n:
                    for h, d in zip(host_in, dev_sets[i % 2]):
                        d.copy_(h, non_blocking=True)
                    ready[i + 2].record(copy)
        done = torch.cuda.Event()
        done.record(copy)
        comp.wait_event(done)
        end.record(comp)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n

    # The first passes of a process run slow (one warm-up pass of a few steps
    # left steps at ~1.4x the steady time on one B200 box): warm up with a
    # longer pass, then report the median of three timed passes.
    one_pass(max(warmup, 50))
    ms = statistics.median(one_pass(steps) for _ in range(3))
    return ms, host_out[(steps - 1) % 2]


def nbytes_of(tensors) -> int:
    return int(sum(t.numel() * t.element_size() for t in tensors))


def packed_inputs(device, tensors):
    """One pinned host buffer holding ``tensors`` back to back (16-byte aligned
    pieces) and two device buffers with views of the same layout, so a step's
    inputs go up in one copy: ``(host [buffer], dev_sets [[buffer]], views per set)``."""
    import numpy as np

    offs, n = [], 0
    for t in tensors:
        offs.append(n)
        n += (t.numel() * t.element_size() + 15) // 16 * 16
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    for t, o in zip(tensors, offs):
        b = t.numel() * t.element_size()
        host[o:o + b].copy_(torch.from_numpy(np.frombuffer(t.detach().cpu().contiguous().numpy().tobytes(),
                                                           dtype=np.uint8)))
    dev_bufs = [torch.empty(n, dtype=torch.uint8, device=device) for _ in range(2)]
    views = [[buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(tensors, offs)]
             for buf in dev_bufs]
    return [host], [[buf] for buf in dev_bufs], views


def _cpu_timed(fn, iters: int) -> tuple[float, float]:
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return min(times), statistics.median(times)


# --------------------------------------------------------------------------- workloads
def make_paged_shard(device, seed: int, batch: int, heads: int, kv_heads: int, head_dim: int, page_size: int,
                     lens: list[int], dtype=torch.float16):
    """q [B, H, D], K/V pools [P, ps, Hkv, D] N(0,1), a seeded permuted table, lengths."""
    gen = torch.Generator(device=device).manual_seed(seed)
    pages = [math.ceil(n / page_size) for n in lens]
    pool = sum(pages)
    shape = (pool, page_size, kv_heads, head_dim)
    k = torch.empty(shape, dtype=dtype, device=device)
    v = torch.empty_like(k)
    step = max(1, (1 << 28) // (page_size * kv_heads * head_dim))  # 256 Mi elements of fp32 per draw
    for p0 in range(0, pool, step):
        p1 = min(pool, p0 + step)
        k[p0:p1] = torch.randn((p1 - p0,) + shape[1:], generator=gen, device=device).to(dtype)
        v[p0:p1] = torch.randn((p1 - p0,) + shape[1:], generator=gen, device=device).to(dtype)
    q = torch.randn((batch, heads, head_dim), generator=gen, device=device).to(dtype)
    perm = torch.randperm(pool, generator=gen, device=device).to(torch.int32)
    table = torch.zeros((batch, max(pages)), dtype=torch.int32, device=device)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    return q, k, v, table, torch.tensor(lens, dtype=torch.int32, device=device)


def cfg2_shard_geometry(world: int, rank: int) -> dict:
    """This rank's share of the global cfg2-geometry problem with batch 32 * world."""
    from flashattntile_b200 import sharding

    c = CFG2
    plan = sharding.plan_shards(c["kv_heads"], world, "sequence")
    global_batch = c["batch"] * world
    sh = plan.shard(rank, global_batch)
    kvh = sh.kv_h1 - sh.kv_h0
    heads = kvh * (c["heads"] // c["kv_heads"])
    return {"plan": plan, "shard": sh, "global_batch": global_batch, "batch": sh.seq1 - sh.seq0,
            "kv_heads": kvh, "heads": heads}


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
    cpu_ok = rank == 0 and world == 1 and not args.no_cpu_baseline
    if args.only in ("quant", "prefill", "longctx", "loop", "comparators"):
        res = run_secondary(device, args, peaks, which=(args.only,), dist=dist, cpu=cpu_ok)
        if rank == 0:
            print(json.dumps({"only": args.only, "steps": args.steps, "warmup": args.warmup, "results": res}),
                  flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.only == "decode":
        args.no_secondary = True

    c = CFG2
    geo = cfg2_shard_geometry(world, rank)
    lens_list = [c["ctx"]] * geo["batch"]
    q, k, v, table, lens = make_paged_shard(device, 1 + rank, geo["batch"], geo["heads"], geo["kv_heads"],
                                            c["head_dim"], c["page_size"], lens_list)
    nbytes = decode_bytes(lens_list, geo["heads"], geo["kv_heads"], c["head_dim"], c["page_size"])
    scale = c["head_dim"] ** -0.5
    out = torch.empty_like(q)

    def step():
        launch_decode(q, k, v, table, lens, c["page_size"], scale, 1, out=out)

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        times = time_steps(step, args.steps, args.warmup)
    torch.cuda.synchronize()
    total_ms, kernel_ms = max_over_ranks([sum(times), statistics.mean(times)], device, dist)
    if dist is not None:
        dist.barrier()
    ms_per_step = total_ms / args.steps
    value = world * nbytes / (ms_per_step * 1e-3) / 1e9
    dev_err = _lib.read_device_error(device)

    # ---- e2e through the public op with host buffers ----
    host_in, dev_sets, views = packed_inputs(device, [q, table, lens])

    def e2e_run(d):
        return torch.ops.flashattn_tile.paged_decode(d[0], k, v, d[1], d[2], c["page_size"], scale, 1)

    e2e_steps = max(10, args.steps // 2)
    if dist is not None:
        dist.barrier()
    e2e_ms, o_h = e2e_pipelined(device, e2e_steps, args.warmup, host_in, dev_sets, e2e_run, q, views)
    (e2e_ms,) = max_over_ranks([e2e_ms], device, dist)
    e2e_ok = torch.equal(o_h.to(device), out)

    secondary = {}
    if not args.no_secondary:
        which = ("quant", "prefill", "longctx", "loop") if world == 1 else ("quant", "longctx")
        secondary = run_secondary(device, args, peaks, which=which, dist=dist, cpu=cpu_ok)
    if dist is not None:
        dist.barrier()

    if rank == 0:
        cpu = None
        if cpu_ok:
            cpu = cpu_decode_cfg2(q, k, v, table, lens, iters=3)
        plan = geo["plan"]
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
            "data": "synthetic N(0,1), seeded per rank shard",
            "config": {"workload": "cfg2 paged decode", "global_batch": geo["global_batch"],
                       "batch_per_gpu": geo["batch"], "ctx": c["ctx"], "heads": c["heads"],
                       "kv_heads": c["kv_heads"], "heads_per_gpu": geo["heads"], "kv_heads_per_gpu": geo["kv_heads"],
                       "head_dim": c["head_dim"], "page_size": c["page_size"],
                       "parallelism": f"shard by KV head ({plan.head_groups} groups) x sequence ({plan.splits}), "
                                      "no comm",
                       "l2": "inputs 537 MB per step per GPU > 126 MB L2; steps back to back, no flush"},
            "roofline": roofline("hbm", nbytes, kernel_ms, peaks, traffic=NCU_TRAFFIC_BYTES["decode_cfg2"],
                                 traffic_source="ncu dram read+write of one cfg2 launch (recorded capture)"),
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": nbytes_of(host_in),
                    "d2h_bytes_per_step": nbytes_of([q]),
                    "path": "torch.ops.flashattn_tile.paged_decode, default validation; q/table/lens packed in one "
                            "pinned host buffer, one upload per step (copy stream, two input sets), output to pinned "
                            "host (same copy stream)",
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


def run_secondary(device, args, peaks, which=("quant", "prefill", "longctx", "loop"), dist=None,
                  cpu: bool = False) -> dict:
    """Quantised decode (cfg4), varlen prefill (cfg3), long-context decode (cfg5), decode loop."""
    res = {}
    if "loop" in which:
        res.update(run_decode_loop(device, args))
    if "quant" in which:
        res.update(run_quant(device, args, peaks, dist, cpu))
    if "prefill" in which:
        res.update(run_prefill(device, args, peaks, cpu))
    if "longctx" in which:
        res.update(run_longctx(device, args, peaks, dist, cpu))
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
    q, k, v, table, lens = make_paged_shard(device, 1, c["batch"], c["heads"], c["kv_heads"], c["head_dim"],
                                            c["page_size"], [c["ctx"]] * c["batch"])
    nbytes = decode_bytes([c["ctx"]] * c["batch"], c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])
    scale = c["head_dim"] ** -0.5
    ours = launch_decode(q, k, v, table, lens, c["page_size"], scale, 1)
    out = torch.empty_like(q)

    def record(name, fn, ref, work, unit):
        try:
            o = fn()
            torch.cuda.synchronize()
            diff = float((o.float() - ref.float()).abs().max())
            ms = statistics.mean(time_steps(fn, steps, args.warmup))
            val = work / (ms * 1e-3) / (1e9 if unit == "GB/s" else 1e12)
            res[name] = {"value": round(val, 1), "unit": unit, "ms": round(ms, 4), "maxdiff_vs_ours": diff}
        except Exception as e:  # a library missing or failing on this box
            res[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}

    record("cfg2_decode_ours", lambda: launch_decode(q, k, v, table, lens, c["page_size"], scale, 1, out=out),
           ours, nbytes, "GB/s")
    # The reference's own CUDA C++ decode (csrc/paged_decode.cu), built for sm_100a by oracle/build_ref_native.py.
    try:
        from oracle import build_ref_native

        native = build_ref_native.load_module()
        if native is None:
            raise RuntimeError("oracle/_ref holds no build of the reference's native kernel")
        record("cfg2_decode_reference_native_cuda", lambda: native.paged_decode(q, k, v, table, lens, c["page_size"],
                                                                                 scale), ours, nbytes, "GB/s")
    except Exception as e:
        res["cfg2_decode_reference_native_cuda"] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
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

    flops = flops_attention_varlen(32, 128, CFG3_LENS, CFG3_LENS, causal=True)
    offs = [0] + torch.tensor(CFG3_LENS).cumsum(0).tolist()
    cu = torch.tensor(offs, dtype=torch.int32, device=device)
    g3 = torch.Generator(device=device).manual_seed(2)
    for dt, tag in ((torch.float16, ""), (torch.bfloat16, "_bf16")):
        sets = []
        for _ in range(2):
            sets.append(tuple(torch.randn((offs[-1], h, 128), generator=g3, device=device).to(dt) for h in (32, 8, 8)))
        ref3 = launch_prefill(*sets[1], cu, cu, 4096, 4096, True, 128 ** -0.5)

        def alternate(call):
            state = {"i": 0}  # the first call uses sets[1], the set ref3 was computed on

            def fn():
                state["i"] += 1
                return call(*sets[state["i"] & 1])
            return fn

        o3 = torch.empty_like(sets[0][0])
        record("cfg3_prefill_ours" + tag,
               alternate(lambda q3, k3, v3: launch_prefill(q3, k3, v3, cu, cu, 4096, 4096, True, 128 ** -0.5, out=o3)),
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

        record("cfg3_prefill_torch_sdpa" + tag, alternate(sdpa), ref3, flops, "TFLOP/s")
        try:
            from flash_attn import flash_attn_varlen_func

            record("cfg3_prefill_flash_attn2" + tag,
                   alternate(lambda q3, k3, v3: flash_attn_varlen_func(q3, k3, v3, cu, cu, 4096, 4096,
                                                                       softmax_scale=128 ** -0.5, causal=True)),
                   ref3, flops, "TFLOP/s")
        except Exception as e:
            res["cfg3_prefill_flash_attn2" + tag] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
        del sets, ref3, o3
        torch.cuda.empty_cache()
    # The reference's Triton kernels (cfg2 decode at split_k 1/2/4/8, cfg3 prefill), in a process of their own.
    import subprocess

    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "flashattn_tile").is_dir():
        run = subprocess.run([sys.executable, str(ROOT / "tests" / "ref_triton_runner.py"), str(ref_dir), "time",
                              str(steps), str(args.warmup)], capture_output=True, text=True, timeout=900,
                             env=dict(os.environ, PYTHONPATH=str(ROOT)))
        lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
        if run.returncode == 0 and lines:
            res.update(json.loads(lines[-1]))
        else:
            res["reference_triton"] = {"unavailable": (run.stderr or run.stdout)[-300:]}
    else:
        res["reference_triton"] = {"unavailable": "the reference is not installed under baseline/_ref"}
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


def run_longctx(device, args, peaks, dist=None, cpu: bool = False) -> dict:
    """cfg5: B8, H64/8, D128, ps64, ctx 131072 fp16, a fixed 4.3 GB cache (strong scaling).

    Head-first (the default plan): rank r holds KV heads [8r/N, 8(r+1)/N) of
    every sequence, all pages, and outputs their query heads; no data crosses
    GPUs at N <= 8.  Page split (reported beside it): every rank holds all KV
    heads of its page range of every sequence; fp32 partials meet their owner
    rank in one all-to-all (each rank receives only the rows it outputs) and
    merge by log-sum-exp.  Times are the slowest rank's."""
    from flashattntile_b200 import sharding
    from flashattntile_b200 import sequence_parallel as sp
    from flashattntile_b200._config import value_checks
    from flashattntile_b200.kernels.decode import launch_decode

    c = CFG5
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    g = c["heads"] // c["kv_heads"]
    scale = c["head_dim"] ** -0.5
    pages_per_seq = c["ctx"] // c["page_size"]
    total_bytes = decode_bytes([c["ctx"]] * c["batch"], c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])
    steps = max(10, args.steps // 2)
    gq = torch.Generator(device=device).manual_seed(49)  # the global q, identical on every rank
    q_all = torch.randn((c["batch"], c["heads"], c["head_dim"]), generator=gq, device=device).half()
    res = {}

    # ---- head-first ----
    plan = sharding.plan_shards(c["kv_heads"], world, "page")
    sh = plan.shard(rank)
    kvh = sh.kv_h1 - sh.kv_h0
    p0, p1 = sp.page_range(pages_per_seq, plan.splits, sh.split)
    q0, q1 = sh.query_heads(c["heads"], c["kv_heads"])
    q = q_all[:, q0:q1].contiguous()
    lq, k, v, table, lens = make_paged_shard(device, 50 + rank, c["batch"], q1 - q0, kvh, c["head_dim"],
                                             c["page_size"], [(p1 - p0) * c["page_size"]] * c["batch"])
    del lq
    local_bytes = decode_bytes([(p1 - p0) * c["page_size"]] * c["batch"], q1 - q0, kvh, c["head_dim"],
                               c["page_size"])
    out = torch.empty_like(q)
    with value_checks(False):
        if plan.splits == 1:
            def step():
                launch_decode(q, k, v, table, lens, c["page_size"], scale, 1, out=out)
        else:
            group = None
            if dist is not None:
                groups = [dist.new_group(plan.split_group_ranks(r0)) for r0 in range(0, world, plan.splits)]
                group = groups[rank // plan.splits]
            from flashattntile_b200.paging import PagedKVCache

            cache = PagedKVCache(k, v, table, lens, c["page_size"])

            def step():
                sharding.sharded_decode(q, cache, plan, rank, scale, group=group)
        if dist is not None:
            dist.barrier()
        times = time_steps(step, steps, args.warmup)
    ms, = max_over_ranks([statistics.mean(times)], device, dist)
    res["cfg5_longctx_decode"] = {
        "value": round(total_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms": round(ms, 4), "n_gpus": world,
        "scaling": "strong", "algorithmic_bytes": total_bytes,
        "plan": f"KV heads {plan.head_groups} groups x pages {plan.splits}",
        "per_gpu": {"kv_heads": kvh, "heads": q1 - q0, "pages_per_seq": p1 - p0, "bytes": local_bytes},
        "roofline": roofline("hbm", local_bytes, ms, peaks, note="per GPU: its share of the cache"),
        "exchange_bytes_per_rank": 0 if plan.splits == 1 else sp.packed_size(c["batch"], q1 - q0, c["head_dim"]) * 4,
        "step": "local decode only (no data crosses GPUs)" if plan.splits == 1
                else "local decode + all-to-all of partials to owners + LSE merge"}
    if cpu and world == 1:
        res["cfg5_longctx_decode"]["cpu_baseline"] = cpu_decode_sample(
            q, k, v, table, lens, c["page_size"], seqs=1, iters=3, what="cfg5 sequence 0 (ctx 131072, H64/8)",
            full_bytes=total_bytes, full_seqs=c["batch"])
    del k, v, table, lens
    torch.cuda.empty_cache()

    # ---- page split (every rank all KV heads, a page range of every sequence) ----
    pplan = sharding.plan_shards(c["kv_heads"], world, "page", head_groups=1)
    psh = pplan.shard(rank)
    p0, p1 = sp.page_range(pages_per_seq, pplan.splits, psh.split)
    lq, k, v, table, lens = make_paged_shard(device, 60 + rank, c["batch"], c["heads"], c["kv_heads"],
                                             c["head_dim"], c["page_size"], [(p1 - p0) * c["page_size"]] * c["batch"])
    del lq
    from flashattntile_b200.paging import PagedKVCache

    cache = PagedKVCache(k, v, table, lens, c["page_size"])
    packed = torch.empty(sp.packed_size(c["batch"], c["heads"], c["head_dim"]), dtype=torch.float32, device=device)
    rows = c["batch"] * c["heads"]
    r0, r1 = sharding.owner_rows(rows, world)[rank]

    def pstep():
        sp.decode_partial(q_all, cache, scale, packed=packed)
        if dist is not None:
            parts = sharding.exchange_to_owners(packed, c["batch"], c["heads"], c["head_dim"])
        else:
            parts = packed.view(1, -1)
        return sharding.merge_owned(parts, r1 - r0, c["head_dim"])

    with value_checks(False):
        if dist is not None:
            dist.barrier()
        times = time_steps(pstep, steps, args.warmup)
        dtimes = time_steps(lambda: sp.decode_partial(q_all, cache, scale, packed=packed), steps, args.warmup)
        merged = pstep()
        torch.cuda.synchronize()
    ms, dms = max_over_ranks([statistics.mean(times), statistics.mean(dtimes)], device, dist)
    check = pagesplit_check(device, dist, q_all, k, v, table, c, p0, p1, merged, rank, world, scale)
    res["cfg5_longctx_decode_pagesplit"] = {
        "value": round(total_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms": round(ms, 4), "n_gpus": world,
        "scaling": "strong", "local_decode_ms": round(dms, 4),
        "exchange_merge_share": round(max(0.0, ms - dms) / ms, 4),
        "exchange_bytes_received_per_rank": world * (r1 - r0) * (c["head_dim"] + 1) * 4,
        "check_max_abs_vs_unsplit": check,
        "step": "decode partial (fp32 o, lse) + all-to-all of rows to their owners + LSE merge"
                if world > 1 else "decode partial + LSE merge (1 part)"}
    del k, v, table, lens, cache
    torch.cuda.empty_cache()
    return res


def pagesplit_check(device, dist, q_all, k, v, table, c, p0, p1, merged, rank, world, scale) -> float | None:
    """Max-abs of rank 0's merged rows for (sequence 0, KV head 0) against one
    unsplit decode of that sequence and head, with every rank's pages of it
    brought to rank 0 (outside the timed region)."""
    from flashattntile_b200.kernels.decode import launch_decode

    g = c["heads"] // c["kv_heads"]
    n_local = p1 - p0
    mine_k = k[table[0, :n_local].long(), :, 0:1].contiguous()  # [n_local, ps, 1, D]
    mine_v = v[table[0, :n_local].long(), :, 0:1].contiguous()
    if dist is not None:
        gk = [torch.empty_like(mine_k) for _ in range(world)]
        gv = [torch.empty_like(mine_v) for _ in range(world)]
        dist.all_gather(gk, mine_k)
        dist.all_gather(gv, mine_v)
    else:
        gk, gv = [mine_k], [mine_v]
    if rank != 0:
        return None
    kc, vc = torch.cat(gk), torch.cat(gv)
    n = kc.shape[0]
    t = torch.arange(n, dtype=torch.int32, device=device).view(1, n)
    want = launch_decode(q_all[0:1, 0:g].contiguous(), kc, vc, t, torch.tensor([n * c["page_size"]],
                         dtype=torch.int32, device=device), c["page_size"], scale, 1, out_dtype=torch.float32)
    got = merged[0:g].float()
    return float((got - want[0]).abs().max())


def run_quant(device, args, peaks, dist=None, cpu: bool = False) -> dict:
    """cfg4: B128, H32/8, D128, ps32, ctx U[1024, 16384], INT8 and e4m3 caches.

    At N GPUs the global batch is 128 N (lengths from one seeded draw) and each
    rank holds its KV-head slice (head-first plan, weak scaling)."""
    from flashattntile_b200 import quant, sharding
    from flashattntile_b200.kernels.decode import launch_decode

    c = CFG4
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    plan = sharding.plan_shards(c["kv_heads"], world, "sequence")
    global_batch = c["batch"] * world
    sh = plan.shard(rank, global_batch)
    kvh = sh.kv_h1 - sh.kv_h0
    heads = kvh * (c["heads"] // c["kv_heads"])
    gen = torch.Generator(device="cpu").manual_seed(3)
    ctx_all = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (global_batch,), generator=gen)
    ctx = ctx_all[sh.seq0:sh.seq1]
    lens_list = [int(x) for x in ctx]
    batch, dim, ps = len(lens_list), c["head_dim"], c["page_size"]
    pages = [math.ceil(n / ps) for n in lens_list]
    pool = sum(pages)
    g2 = torch.Generator(device=device).manual_seed(3 + 1000 * rank)
    perm = torch.randperm(pool, generator=g2, device=device).to(torch.int32)
    table = torch.zeros((batch, max(pages)), dtype=torch.int32, device=device)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    lens = ctx.to(torch.int32).to(device)
    q = torch.randn((batch, heads, dim), generator=g2, device=device).half()
    res = {}
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
        nbytes = decode_bytes(lens_list, heads, kvh, dim, ps, elem=1, scale_bytes=4)

        def step():
            launch_decode(q, kq, vq, table, lens, ps, dim ** -0.5, 1, k_scale=ks, v_scale=vs, out=out)

        if dist is not None:
            dist.barrier()
        times = time_steps(step, max(10, args.steps // 2), args.warmup)
        ms, = max_over_ranks([statistics.mean(times)], device, dist)
        host_in, dev_sets, views = packed_inputs(device, [q, table, lens])

        def e2e_run(d):
            return torch.ops.flashattn_tile.paged_decode_quant(d[0], kq, vq, ks, vs, d[1], d[2], ps, dim ** -0.5, 1)

        e2e_ms, o_h = e2e_pipelined(device, max(10, args.steps // 4), args.warmup, host_in, dev_sets, e2e_run, q,
                                    views)
        e2e_ms, = max_over_ranks([e2e_ms], device, dist)
        entry = {"value": round(world * nbytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms": round(ms, 4),
                 "n_gpus": world, "scaling": "weak", "global_batch": global_batch, "batch_per_gpu": batch,
                 "kv_heads_per_gpu": kvh, "algorithmic_bytes": nbytes,
                 "roofline": roofline("hbm", nbytes, ms, peaks),
                 "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                         "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": nbytes_of(host_in),
                         "d2h_bytes_per_step": nbytes_of([q]),
                         "path": "torch.ops.flashattn_tile.paged_decode_quant, default validation, q/table/lens "
                                 "packed in one pinned upload per step, output to pinned host (one copy stream)",
                         "matches_device_path": bool(torch.equal(o_h.to(device), out))}}
        if cpu:
            entry["cpu_baseline"] = cpu_quant_sample(q, kq, vq, ks, vs, table, lens, ps, mode, seqs=8, iters=3,
                                                     full_bytes=nbytes, full_seqs=batch)
        res[f"cfg4_decode_{mode}"] = entry
        del kq, vq, ks, vs
    torch.cuda.empty_cache()
    return res


def run_prefill(device, args, peaks, cpu: bool = False) -> dict:
    """cfg3: varlen causal prefill, lens {512, 1024, 2048, 4096}, H32/8, D128, fp16 and bf16."""
    from flashattntile_b200.autotune import flops_attention_varlen
    from flashattntile_b200.kernels.prefill import launch_prefill

    res = {}
    lens = CFG3_LENS
    flops = flops_attention_varlen(32, 128, lens, lens, causal=True)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=device)
    g3 = torch.Generator(device=device).manual_seed(2)
    for dt in (torch.float16, torch.bfloat16):
        tag = "f16" if dt == torch.float16 else "bf16"
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

        times = time_steps(pstep, max(10, args.steps // 2), args.warmup)
        ms = statistics.mean(times)
        entry = {"value": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms": round(ms, 4),
                 "algorithmic_flops": flops, "roofline": roofline("tensor", flops, ms, peaks)}
        # e2e through the op: q/k/v/cu from pinned host, output back to pinned host.
        q3, k3, v3, _ = sets[0]
        host_in = [q3.cpu().pin_memory(), k3.cpu().pin_memory(), v3.cpu().pin_memory(), cu.cpu().pin_memory()]
        dev_sets = [[sets[i][0], sets[i][1], sets[i][2], torch.empty_like(cu)] for i in range(2)]

        def e2e_run(d):
            return torch.ops.flashattn_tile.prefill_varlen(d[0], d[1], d[2], d[3], d[3], 4096, 4096, True,
                                                           128 ** -0.5)

        e2e_ms, o_h = e2e_pipelined(device, 10, args.warmup, host_in, dev_sets, e2e_run, q3)
        ref = launch_prefill(q3, k3, v3, cu, cu, 4096, 4096, True, 128 ** -0.5)
        entry["e2e"] = {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                        "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": nbytes_of(host_in),
                        "d2h_bytes_per_step": nbytes_of([q3]),
                        "path": "torch.ops.flashattn_tile.prefill_varlen, default validation, pinned host q/k/v/cu "
                                "in and output out (one copy stream); bound by PCIe, not the kernel",
                        "matches_device_path": bool(torch.equal(o_h.to(device), ref))}
        if cpu:
            entry["cpu_baseline"] = cpu_prefill_cfg3(q3, k3, v3, cu, tag, flops, iters=3)
        res[f"cfg3_prefill_{tag}"] = entry
        del sets, dev_sets, host_in
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
        times = time_steps(ppstep, max(10, args.steps // 2), args.warmup)
    ms = statistics.mean(times)
    res["cfg3_prefill_paged_f16_ps16"] = {
        "value": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms": round(ms, 4),
        "algorithmic_flops": flops, "roofline": roofline("tensor", flops, ms, peaks), "page_size": ps}
    del caches
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------- CPU baselines (oracle/)
def _threads() -> int:
    return os.cpu_count() or 1


def cpu_decode_cfg2(q, k, v, table, lens, iters: int) -> dict:
    """The oracle (numpy port of the reference's fp32 paged path) on the whole cfg2 batch."""
    from oracle import attention as oatt
    from oracle import work as owork

    qn, tn, ln = q.cpu().numpy(), table.cpu().numpy(), lens.cpu().numpy()
    kn, vn = k.cpu().numpy(), v.cpu().numpy()
    nbytes = owork.bytes_decode_paged(ln.tolist(), q.shape[1], k.shape[2], k.shape[3], k.shape[1])
    threads = _threads()
    best, med = _cpu_timed(lambda: oatt.attention_paged(qn, kn, vn, tn, ln, int(k.shape[1]), dtype="f16",
                                                        threads=threads), iters)
    return {"value": round(nbytes / best / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"the whole cfg2 batch ({q.shape[0]} x ctx {int(ln[0])}), fp16 inputs upcast to fp32; "
                      f"sequences on {threads} threads, BLAS one thread each; min of {iters}",
            "seconds_min": round(best, 4), "seconds_median": round(med, 4)}


def cpu_decode_sample(q, k, v, table, lens, page_size, seqs: int, iters: int, what: str, full_bytes: int,
                      full_seqs: int) -> dict:
    """The oracle on the first ``seqs`` sequences (only their pages copied to the host)."""
    import numpy as np

    from oracle import attention as oatt
    from oracle import work as owork

    tn = table[:seqs].cpu().numpy()
    ln = lens[:seqs].cpu().numpy()
    used = np.unique(tn.reshape(-1))
    remap = np.full(int(k.shape[0]), -1, dtype=np.int64)
    remap[used] = np.arange(used.size)
    idx = torch.from_numpy(used).to(k.device)
    kn = k.index_select(0, idx).cpu().numpy()
    vn = v.index_select(0, idx).cpu().numpy()
    tn = remap[tn].astype(np.int32)
    qn = q[:seqs].cpu().numpy()
    nbytes = owork.bytes_decode_paged(ln.tolist(), q.shape[1], k.shape[2], k.shape[3], page_size)
    threads = _threads()
    best, med = _cpu_timed(lambda: oatt.attention_paged(qn, kn, vn, tn, ln, page_size, dtype="f16",
                                                        threads=threads), iters)
    return {"value": round(nbytes / best / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{what}: {seqs} of {full_seqs} sequences ({nbytes} of {full_bytes} algorithmic bytes), "
                      f"fp16 upcast to fp32; min of {iters}",
            "seconds_min": round(best, 4), "seconds_median": round(med, 4)}


def cpu_quant_sample(q, kq, vq, ks, vs, table, lens, page_size, mode, seqs: int, iters: int, full_bytes: int,
                     full_seqs: int) -> dict:
    """``dequantize_cache(float32)`` + ``ref_attention_paged`` (quant.py:178, reference.py:145),
    restated by the oracle, on the first ``seqs`` sequences; each step dequantises and attends."""
    import numpy as np

    from oracle import attention as oatt
    from oracle import quant as oquant
    from oracle import work as owork

    tn = table[:seqs].cpu().numpy()
    ln = lens[:seqs].cpu().numpy()
    used = np.unique(np.concatenate([tn[b, :math.ceil(int(ln[b]) / page_size)] for b in range(seqs)]))
    remap = np.zeros(int(kq.shape[0]), dtype=np.int64)
    remap[used] = np.arange(used.size)
    idx = torch.from_numpy(used).to(kq.device)
    codes_k = kq.index_select(0, idx).cpu()
    codes_v = vq.index_select(0, idx).cpu()
    if mode != "int8":
        codes_k, codes_v = codes_k.view(torch.uint8), codes_v.view(torch.uint8)
    ck, cv = codes_k.numpy(), codes_v.numpy()
    sk, sv = ks.index_select(0, idx).cpu().numpy(), vs.index_select(0, idx).cpu().numpy()
    tn = remap[tn].astype(np.int32)
    qn = q[:seqs].float().cpu().numpy()
    nbytes = owork.bytes_decode_paged(ln.tolist(), q.shape[1], kq.shape[2], kq.shape[3], page_size, 2, 1, 4)
    threads = _threads()

    def run():
        dk, dv = oquant.dequantize_kv_pages(ck, cv, sk, sv, mode)
        oatt.attention_paged(qn, dk, dv, tn, ln, page_size, dtype="f32", threads=threads)

    best, med = _cpu_timed(run, iters)
    return {"value": round(nbytes / best / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"cfg4 {mode}: {seqs} of {full_seqs} sequences ({nbytes} of {full_bytes} algorithmic "
                      f"bytes); dequantise to fp32 then the fp32 paged oracle; min of {iters}",
            "seconds_min": round(best, 4), "seconds_median": round(med, 4)}


def _storage(t: torch.Tensor):
    import numpy as np

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def cpu_prefill_cfg3(q, k, v, cu, tag: str, flops: int, iters: int) -> dict:
    """``ref_attention_varlen`` (reference.py:50) restated by the oracle on the whole cfg3 batch."""
    from oracle import attention as oatt

    qn, kn, vn, cn = _storage(q), _storage(k), _storage(v), cu.cpu().numpy()
    threads = _threads()
    best, med = _cpu_timed(lambda: oatt.attention_varlen(qn, kn, vn, cn, cn, True, dtype=tag, threads=threads),
                           iters)
    return {"value": round(flops / best / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"the whole cfg3 batch ({tag}, lens {CFG3_LENS}), upcast to fp32; (sequence, 256-row) "
                      f"blocks on {threads} threads, BLAS one thread each; min of {iters}",
            "seconds_min": round(best, 4), "seconds_median": round(med, 4)}


# --------------------------------------------------------------------------- reference arm
def run_reference_arm(args, rank: int, world: int) -> None:
    """The reference's CPU path (the oracle port of reference.py's fp32 paged
    attention) on rank 0 only, all host threads, the whole cfg2 batch per step.
    Nothing here imports or loads this repository's library."""
    if rank != 0:
        return
    import numpy as np

    from oracle import attention as oatt
    from oracle import work as owork

    c = CFG2
    gen = torch.Generator().manual_seed(1)
    pages_per_seq = c["ctx"] // c["page_size"]
    shape = (c["batch"] * pages_per_seq, c["page_size"], c["kv_heads"], c["head_dim"])
    k = torch.randn(shape, generator=gen).half().numpy()
    v = torch.randn(shape, generator=gen).half().numpy()
    q = torch.randn((c["batch"], c["heads"], c["head_dim"]), generator=gen).half().numpy()
    table = torch.randperm(shape[0], generator=gen).view(c["batch"], pages_per_seq).to(torch.int32).numpy()
    lens = np.full(c["batch"], c["ctx"], dtype=np.int32)
    threads = _threads()
    nbytes = owork.bytes_decode_paged(lens.tolist(), c["heads"], c["kv_heads"], c["head_dim"], c["page_size"])

    def call():
        oatt.attention_paged(q, k, v, table, lens, c["page_size"], dtype="f16", threads=threads)

    for _ in range(args.warmup):
        call()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call()
    dt = (time.perf_counter() - t0) / args.steps
    value = nbytes / dt / 1e9
    sample = (f"the whole cfg2 batch (32 x ctx 4096, H32/8, D128, ps16) every step, fp16 inputs upcast to fp32; "
              f"sequences on {threads} threads, BLAS one thread each")
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
        "config": {"workload": "cfg2 paged decode", "global_batch": c["batch"], "batch_per_gpu": c["batch"],
                   "ctx": c["ctx"], "heads": c["heads"], "kv_heads": c["kv_heads"], "head_dim": c["head_dim"],
                   "page_size": c["page_size"]},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
