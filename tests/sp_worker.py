"""One rank of the two-GPU sequence-parallel decode test (launched by torchrun).

Each rank keeps only its own page range of every sequence, in its own page
pool on its own GPU; ``sequence_parallel_decode`` exchanges the fp32 partials
over NCCL and merges them.  Every rank checks the result against the oracle's
unsplit attention and prints ``sp_worker ok``.
"""

from __future__ import annotations

import datetime
import math
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from flashattntile_b200 import sequence_parallel as sp  # noqa: E402
from flashattntile_b200.paging import PagedKVCache  # noqa: E402
from oracle import attention as oatt  # noqa: E402
from tests.helpers import assert_parity_16bit, paged_case, to_np  # noqa: E402


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        lens, heads, kvh, dim, ps = [1000, 4096, 77], 16, 2, 128, 64
        q, k, v, table, lens_t = paged_case(99, lens, heads, kvh, dim, ps, torch.float16)
        p0, p1 = sp.page_range(table.shape[1], world, rank)
        # This rank's pool: only the pages its range uses, renumbered 0..n-1.
        mine = table[:, p0:p1].reshape(-1).long()
        local_table = torch.arange(mine.numel(), dtype=torch.int32).view(table.shape[0], p1 - p0)
        local = PagedKVCache(k[mine].to(dev), v[mine].to(dev), local_table.to(dev),
                             sp.local_lengths(lens_t, ps, p0, p1).to(dev), ps)
        out = sp.sequence_parallel_decode(q.to(dev), local)
        torch.cuda.synchronize()
        want = oatt.attention_paged(to_np(q), to_np(k), to_np(v), to_np(table), to_np(lens_t), ps, dtype="f16")
        worst = assert_parity_16bit(out, want, torch.float16)
        print(f"rank {rank}: max-abs {worst:.3e} over {math.prod(out.shape)} outputs")

        # Head-first plan: this rank keeps a compact copy of its KV-head slice
        # (sequence split inside the head group) and decodes with no exchange.
        from flashattntile_b200 import sharding

        cache = PagedKVCache(k.to(dev), v.to(dev), table.to(dev), lens_t.to(dev), ps)
        plan = sharding.plan_shards(kvh, world, "sequence")
        sh = plan.shard(rank, len(lens))
        mine_cache = sharding.shard_cache(cache, plan, rank, copy=True)
        h0, h1 = sh.query_heads(heads, kvh)
        part = sharding.sharded_decode(sharding.shard_query(q.to(dev), plan, rank).contiguous(), mine_cache, plan,
                                       rank)
        assert_parity_16bit(part, want[sh.seq0:sh.seq1, h0:h1], torch.float16)

        # Page split over all ranks: partial rows go to their owners (all-to-all), LSE merge.
        pplan = sharding.plan_shards(kvh, world, "page", head_groups=1)
        rows = sharding.sharded_decode(q.to(dev), sharding.shard_cache(cache, pplan, rank), pplan, rank)
        r0, r1 = sharding.owner_rows(len(lens) * heads, world)[rank]
        assert_parity_16bit(rows, want.reshape(len(lens) * heads, dim)[r0:r1], torch.float16)
        dist.barrier()
        print("sp_worker ok")
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
