"""Generate the golden vectors in this folder by running the reference itself.

Usage (on a machine with a FlashAttnTile checkout; the GPU box does not need
one, it only reads the committed ``.npz`` files)::

    python tests/golden/make_golden.py --reference /path/to/FlashAttnTile

Every case draws seeded inputs on the CPU, runs the reference's own CPU
functions (``flashattn_tile.reference`` / ``paging`` / ``quant``) and stores
inputs and outputs as raw storage arrays: fp16 as float16, bf16 as uint16 bit
patterns, float8_e4m3fn as uint8 codes.  ``tests/test_oracle_golden.py``
pins the numpy oracle to these files; the GPU tests compare the CUDA kernels
against them as well.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _store(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == getattr(torch, "float8_e4m3fn", None):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def _tag(dtype: torch.dtype) -> str:
    return {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[dtype]


def _paged_inputs(gen, batch, lens, heads, kv_heads, dim, page_size, dtype, pool_extra=0):
    max_pages = max(1, -(-max(lens) // page_size))
    pool = batch * max_pages + pool_extra
    k = torch.randn(pool, page_size, kv_heads, dim, generator=gen).to(dtype)
    v = torch.randn(pool, page_size, kv_heads, dim, generator=gen).to(dtype)
    q = torch.randn(batch, heads, dim, generator=gen).to(dtype)
    table = torch.randperm(pool, generator=gen)[: batch * max_pages].view(batch, max_pages).to(torch.int32)
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    return q, k, v, table, seq_lens


def make_cases(ref_root: Path) -> dict[str, dict[str, np.ndarray]]:
    sys.path.insert(0, str(ref_root))
    from flashattn_tile import paging, quant, reference  # noqa: E402

    cases: dict[str, dict[str, np.ndarray]] = {}

    # cfg1 of the benchmark contract: B2, H8/Hkv2, D64, ps16, lens U[1,256],
    # fp32 N(0,1), permuted table over a B*ceil(256/16) = 32-page pool.
    gen = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 257, (2,), generator=gen).tolist()
    pool, max_pages = 2 * 16, 16
    k = torch.randn(pool, 16, 2, 64, generator=gen)
    v = torch.randn(pool, 16, 2, 64, generator=gen)
    q = torch.randn(2, 8, 64, generator=gen)
    table = torch.randperm(pool, generator=gen)[: 2 * max_pages].view(2, max_pages).to(torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    out = reference.ref_attention_paged(q, k, v, table, sl)
    cases["cfg1_decode_f32"] = dict(q=_store(q), k_cache=_store(k), v_cache=_store(v), page_table=_store(table),
                                    seq_lens=_store(sl), out=_store(out),
                                    meta=np.array(json.dumps({"dtype": "f32", "page_size": 16})))

    # Ragged decode in the 16-bit dtypes; "out" is the reference's output in the
    # input dtype, "out_f32" the same math on fp32 upcasts (no output rounding).
    decode_specs = [
        ("decode_f16_gqa4", torch.float16, [1, 15, 17, 35, 65], 8, 2, 64, 16, 1),
        ("decode_bf16_gqa4", torch.bfloat16, [1, 15, 17, 35, 65], 8, 2, 64, 16, 2),
        ("decode_f16_mqa_d128", torch.float16, [1, 33, 100], 8, 1, 128, 32, 3),
        ("decode_bf16_mha_d128", torch.bfloat16, [7, 40, 70], 2, 2, 128, 16, 4),
        ("decode_f16_ps8", torch.float16, [3, 8, 9, 40], 4, 2, 64, 8, 5),
    ]
    for name, dtype, lens, h, hkv, d, ps, seed in decode_specs:
        gen = torch.Generator().manual_seed(100 + seed)
        q, k, v, table, sl = _paged_inputs(gen, len(lens), lens, h, hkv, d, ps, dtype, pool_extra=3)
        out = reference.ref_attention_paged(q, k, v, table, sl)
        out32 = reference.ref_attention_paged(q.float(), k.float(), v.float(), table, sl)
        cases[name] = dict(q=_store(q), k_cache=_store(k), v_cache=_store(v), page_table=_store(table),
                           seq_lens=_store(sl), out=_store(out), out_f32=_store(out32),
                           meta=np.array(json.dumps({"dtype": _tag(dtype), "page_size": ps})))

    # Varlen prefill (packed, cu_seqlens), causal and not, incl. kv_len > q_len.
    prefill_specs = [
        ("prefill_f16_causal", torch.float16, [1, 7, 33, 64, 129], None, 4, 2, 64, True, 11),
        ("prefill_bf16_causal_mqa", torch.bfloat16, [5, 40, 90], None, 4, 1, 128, True, 12),
        ("prefill_f16_noncausal", torch.float16, [3, 17, 70], None, 4, 4, 128, False, 13),
        ("prefill_f16_kv_longer", torch.float16, [3, 5, 20], [10, 5, 47], 4, 2, 64, True, 14),
    ]
    for name, dtype, qlens, klens, h, hkv, d, causal, seed in prefill_specs:
        gen = torch.Generator().manual_seed(200 + seed)
        klens = klens or qlens
        q = torch.randn(sum(qlens), h, d, generator=gen).to(dtype)
        k = torch.randn(sum(klens), hkv, d, generator=gen).to(dtype)
        v = torch.randn(sum(klens), hkv, d, generator=gen).to(dtype)
        cu_q = torch.tensor([0] + np.cumsum(qlens).tolist(), dtype=torch.int32)
        cu_k = torch.tensor([0] + np.cumsum(klens).tolist(), dtype=torch.int32)
        out = reference.ref_attention_varlen(q, k, v, cu_q, cu_k, causal=causal)
        out32 = reference.ref_attention_varlen(q.float(), k.float(), v.float(), cu_q, cu_k, causal=causal)
        cases[name] = dict(q=_store(q), k=_store(k), v=_store(v), cu_q=_store(cu_q), cu_k=_store(cu_k),
                           out=_store(out), out_f32=_store(out32),
                           meta=np.array(json.dumps({"dtype": _tag(dtype), "causal": causal})))

    # Quantisation: scales, codes, dequantised values, and the reference's
    # quantised-decode parity target (dequantise, then the fp32 oracle).
    for mode, seed in (("int8", 21), ("float8_e4m3fn", 22)):
        gen = torch.Generator().manual_seed(300 + seed)
        lens = [1, 17, 33, 50]
        q, k, v, table, sl = _paged_inputs(gen, len(lens), lens, 8, 2, 64, 32, torch.float32, pool_extra=2)
        k[0] *= 0.0  # an all-zero page exercises the 1e-8 scale floor
        qk, qv, sk, sv, info = quant.quantize_kv_pages(k, v, mode=mode)
        dk, dv = quant.dequantize_kv_pages(qk, qv, sk, sv, out_dtype=torch.float32)
        q16 = q.to(torch.float16)
        cache = paging.PagedKVCache(k_cache=qk, v_cache=qv, page_table=table, seq_lens=sl, page_size=32)
        deq = quant.dequantize_cache(cache, quant.QuantScales(k=sk, v=sv, mode=mode), out_dtype=torch.float16)
        out = reference.ref_attention_paged(q16, deq.k_cache, deq.v_cache, table, sl)
        cases[f"quant_{mode}"] = dict(k_f32=_store(k), v_f32=_store(v), qk=_store(qk), qv=_store(qv),
                                      scale_k=_store(sk), scale_v=_store(sv), deq_k=_store(dk[:3]), deq_v=_store(dv[:3]),
                                      q=_store(q16), page_table=_store(table), seq_lens=_store(sl), out=_store(out),
                                      meta=np.array(json.dumps({"mode": mode, "page_size": 32,
                                                                "scale_min": info["scale_min"]})))

    # Page-table gather with zero-length rows and a permuted table (bit-exact).
    gen = torch.Generator().manual_seed(400)
    lens = [3, 0, 2, 17, 8]
    q, k, v, table, sl = _paged_inputs(gen, len(lens), lens, 4, 2, 16, 8, torch.float16, pool_extra=1)
    table[1] = -1  # entries of an empty sequence are never read
    gk, gv = paging.gather_paged(k, v, table, sl, 8)
    cases["gather_f16"] = dict(k_cache=_store(k), v_cache=_store(v), page_table=_store(table), seq_lens=_store(sl),
                               gather_k=_store(gk), gather_v=_store(gv), meta=np.array(json.dumps({"page_size": 8})))

    # One-token appends through a permuted table (paging.append_tokens).
    gen = torch.Generator().manual_seed(401)
    cache = paging.allocate(3, 13, 2, 8, 4, dtype=torch.float16)
    perm = torch.randperm(cache.num_pages, generator=gen)
    cache.page_table = perm[cache.page_table.long()].to(torch.int32)
    start_table = cache.page_table.clone()
    steps_k = torch.randn(13, 3, 2, 8, generator=gen).to(torch.float16)
    steps_v = torch.randn(13, 3, 2, 8, generator=gen).to(torch.float16)
    for t in range(13):
        paging.append_tokens(cache, steps_k[t], steps_v[t])
    cases["append_f16"] = dict(page_table=_store(start_table), steps_k=_store(steps_k), steps_v=_store(steps_v),
                               k_cache=_store(cache.k_cache), v_cache=_store(cache.v_cache),
                               seq_lens=_store(cache.seq_lens), meta=np.array(json.dumps({"page_size": 4})))
    return cases


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path of the FlashAttnTile checkout to run")
    args = ap.parse_args()
    cases = make_cases(Path(args.reference))
    for name, arrays in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
    total = sum((HERE / f"{n}.npz").stat().st_size for n in cases)
    print(f"wrote {len(cases)} cases, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
