"""Multi-GPU decode: shard by KV head first, then by sequence or by page range.

One process per GPU.  A decode unit is (sequence, KV head): its query heads,
its K/V rows and its output rows belong to it alone, so the units split across
GPUs with no communication.  The plan here cuts them two ways:

1. **KV heads** (first): the ``world_size`` ranks form ``head_groups`` groups;
   group ``g`` owns the contiguous KV heads ``kv_head_range(...)`` and the
   query heads that map to them (GQA ``h // G``).  Each rank keeps only its
   slice ``[num_pages, page_size, Hkv / head_groups, head_dim]`` of the cache --
   the tensor-parallel layout a serving engine already holds -- plus the whole
   page table and lengths (small).
2. **Second axis** (the ``splits = world_size / head_groups`` ranks of a
   group): ``"sequence"`` gives each a contiguous range of sequences (no
   communication; the normal serving batch), ``"page"`` gives each a
   contiguous range of every sequence's logical pages (long contexts with a
   small batch).  Page splits produce fp32 partials ``(o, lse)`` that meet
   their owner rank in one ``all_to_all`` (each rank receives only the rows it
   outputs, not every rank's full partial) and merge by log-sum-exp
   (``merge_partials``; the combine of FlashAttnTile's split-K reduce,
   ``kernels/decode.py:316-356``).

``head_groups`` is the largest divisor of ``num_kv_heads`` that also divides
``world_size``: with 8 KV heads and 1, 2, 4 or 8 GPUs every split is by KV
head and nothing crosses GPUs; page ranges come in only beyond that (16 GPUs,
or fewer KV heads than GPUs).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .paging import PagedKVCache
from .sequence_parallel import (decode_partial, local_lengths, merge_partials, packed_size, page_range,
                                unpack)


def _even_range(n: int, parts: int, i: int) -> tuple[int, int]:
    """``[lo, hi)`` of part ``i`` when ``n`` items are cut into ``parts`` contiguous, near-equal parts."""
    return (i * n) // parts, ((i + 1) * n) // parts


def kv_head_range(num_kv_heads: int, head_groups: int, group: int) -> tuple[int, int]:
    """KV heads ``[h0, h1)`` of head group ``group`` (``head_groups`` must divide ``num_kv_heads``)."""
    if head_groups < 1 or num_kv_heads % head_groups != 0:
        raise ValueError(f"head_groups {head_groups} must divide num_kv_heads {num_kv_heads}")
    if not 0 <= group < head_groups:
        raise ValueError(f"group {group} out of range for {head_groups} head groups")
    per = num_kv_heads // head_groups
    return group * per, (group + 1) * per


@dataclass(frozen=True)
class RankShard:
    """What one rank owns: KV heads ``[kv_h0, kv_h1)`` and, on the second axis,
    sequences ``[seq0, seq1)`` (``"sequence"``) or split ``split`` of the pages."""

    rank: int
    head_group: int
    split: int
    kv_h0: int
    kv_h1: int
    second: str
    seq0: int = 0
    seq1: int = 0

    def query_heads(self, num_heads: int, num_kv_heads: int) -> tuple[int, int]:
        """Query heads ``[q0, q1)`` that read this rank's KV heads (GQA ``h // G``)."""
        group = num_heads // num_kv_heads
        return self.kv_h0 * group, self.kv_h1 * group


@dataclass(frozen=True)
class ShardPlan:
    world_size: int
    num_kv_heads: int
    head_groups: int
    splits: int
    second: str  # "sequence" or "page"

    def shard(self, rank: int, batch: int | None = None) -> RankShard:
        if not 0 <= rank < self.world_size:
            raise ValueError(f"rank {rank} out of range for world_size {self.world_size}")
        g, s = divmod(rank, self.splits)
        h0, h1 = kv_head_range(self.num_kv_heads, self.head_groups, g)
        seq0 = seq1 = 0
        if self.second == "sequence":
            if batch is None:
                raise ValueError("a sequence split needs the batch size")
            seq0, seq1 = _even_range(batch, self.splits, s)
        return RankShard(rank, g, s, h0, h1, self.second, seq0, seq1)

    def split_group_ranks(self, rank: int) -> list[int]:
        """Ranks that share ``rank``'s KV heads (they split its pages or sequences)."""
        g = rank // self.splits
        return list(range(g * self.splits, (g + 1) * self.splits))


def plan_shards(num_kv_heads: int, world_size: int, second: str = "sequence",
                head_groups: int | None = None) -> ShardPlan:
    """Head-first plan: ``head_groups`` = the largest divisor of ``num_kv_heads``
    that divides ``world_size`` (or the one given), the rest of the ranks on
    ``second`` ("sequence" or "page")."""
    if world_size < 1:
        raise ValueError(f"world_size must be >= 1, got {world_size}")
    if num_kv_heads < 1:
        raise ValueError(f"num_kv_heads must be >= 1, got {num_kv_heads}")
    if second not in ("sequence", "page"):
        raise ValueError(f"second axis must be 'sequence' or 'page', got {second!r}")
    if head_groups is None:
        head_groups = max(d for d in range(1, num_kv_heads + 1)
                          if num_kv_heads % d == 0 and world_size % d == 0)
    if num_kv_heads % head_groups or world_size % head_groups:
        raise ValueError(f"head_groups {head_groups} must divide num_kv_heads {num_kv_heads} "
                         f"and world_size {world_size}")
    return ShardPlan(world_size, num_kv_heads, head_groups, world_size // head_groups, second)


def kv_head_slice(cache: PagedKVCache, kv_h0: int, kv_h1: int, copy: bool = False) -> PagedKVCache:
    """The cache restricted to KV heads ``[kv_h0, kv_h1)``: ``[P, ps, h1 - h0, D]``.

    A view of the same pools by default (the decode kernel takes any head
    stride); ``copy=True`` returns a compact copy, i.e. what a rank holding
    only its slice stores.  Scales of an 8-bit cache slice the same way
    (``scales[:, kv_h0:kv_h1]``)."""
    if not 0 <= kv_h0 < kv_h1 <= cache.num_kv_heads:
        raise ValueError(f"KV heads [{kv_h0}, {kv_h1}) out of range for {cache.num_kv_heads}")
    k = cache.k_cache[:, :, kv_h0:kv_h1]
    v = cache.v_cache[:, :, kv_h0:kv_h1]
    if copy:
        k, v = k.contiguous(), v.contiguous()
    return PagedKVCache(k, v, cache.page_table, cache.seq_lens, cache.page_size)


def sequence_slice(cache: PagedKVCache, seq0: int, seq1: int) -> PagedKVCache:
    """Sequences ``[seq0, seq1)`` of the cache (the page table and lengths are row slices)."""
    return PagedKVCache(cache.k_cache, cache.v_cache, cache.page_table[seq0:seq1], cache.seq_lens[seq0:seq1],
                        cache.page_size)


def shard_cache(cache: PagedKVCache, plan: ShardPlan, rank: int, copy: bool = False) -> PagedKVCache:
    """Rank ``rank``'s share of a whole cache under ``plan`` (views unless ``copy``).

    Sequence splits take the rank's rows of the table; page splits keep every
    sequence with the rank's page columns and lengths (``page_range``)."""
    sh = plan.shard(rank, cache.batch_size)
    c = kv_head_slice(cache, sh.kv_h0, sh.kv_h1, copy=copy)
    if plan.second == "sequence":
        return sequence_slice(c, sh.seq0, sh.seq1)
    p0, p1 = page_range(cache.max_pages_per_seq, plan.splits, sh.split)
    if p1 == p0:
        return PagedKVCache(c.k_cache, c.v_cache, c.page_table[:, :1], torch.zeros_like(c.seq_lens), c.page_size)
    return PagedKVCache(c.k_cache, c.v_cache, c.page_table[:, p0:p1], local_lengths(c.seq_lens, c.page_size, p0, p1),
                        c.page_size)


def shard_query(q: torch.Tensor, plan: ShardPlan, rank: int) -> torch.Tensor:
    """Rank ``rank``'s query rows ``q[seqs, heads]`` of ``q [B, H, D]`` (a view)."""
    sh = plan.shard(rank, q.shape[0])
    h0, h1 = sh.query_heads(q.shape[1], plan.num_kv_heads)
    q = q[:, h0:h1]
    return q[sh.seq0:sh.seq1] if plan.second == "sequence" else q


def owner_rows(rows: int, splits: int) -> list[tuple[int, int]]:
    """Rows ``[r0, r1)`` of a flattened ``[B * H]`` partial that split ``i`` owns and outputs."""
    return [_even_range(rows, splits, i) for i in range(splits)]


def exchange_to_owners(packed: torch.Tensor, batch: int, num_heads: int, head_dim: int, group=None) -> torch.Tensor:
    """Send every row of this rank's packed partial to the rank that outputs it.

    ``packed`` is ``decode_partial``'s buffer (``o [B*H, D]`` then ``lse [B*H]``).
    Split rank ``i`` of ``group`` owns rows ``owner_rows(B*H, R)[i]`` and
    receives those rows from every rank (rank order): the result is a packed
    buffer ``[R, rows_i * (D + 1)]`` (per source rank: ``o`` rows then ``lse``)
    for ``merge_owned``.  Each rank receives ``R * rows_i * (D + 1) * 4`` bytes,
    ``1 / R`` of what an all-gather of the full partials would bring."""
    world = dist.get_world_size(group)
    me = dist.get_rank(group)
    rows = batch * num_heads
    spans = owner_rows(rows, world)
    o, lse = unpack(packed, batch, num_heads, head_dim)
    o = o.reshape(rows, head_dim)
    lse = lse.reshape(rows)
    mine = spans[me][1] - spans[me][0]
    recv_o = torch.empty((world, mine, head_dim), dtype=torch.float32, device=packed.device)
    recv_l = torch.empty((world, mine), dtype=torch.float32, device=packed.device)
    o_splits = [(r1 - r0) * head_dim for r0, r1 in spans]
    l_splits = [r1 - r0 for r0, r1 in spans]
    dist.all_to_all_single(recv_o.view(-1), o.reshape(-1), [mine * head_dim] * world, o_splits, group=group)
    dist.all_to_all_single(recv_l.view(-1), lse, [mine] * world, l_splits, group=group)
    return torch.cat([recv_o.view(world, -1), recv_l], dim=1)


def merge_owned(parts: torch.Tensor, rows: int, head_dim: int, out_dtype: torch.dtype = torch.float16,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge ``exchange_to_owners``' ``[R, rows * (D + 1)]`` into ``[rows, D]`` (LSE-merge kernel)."""
    return merge_partials(parts.contiguous(), 1, rows, head_dim, out_dtype,
                          out=None if out is None else out.view(1, rows, head_dim)).view(rows, head_dim)


def sharded_decode(q: torch.Tensor, local_cache: PagedKVCache, plan: ShardPlan, rank: int,
                   softmax_scale: float | None = None, scales=None, group=None,
                   out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """One decode step on this rank's shard.

    ``q`` is the rank's query slice (``shard_query``) and ``local_cache`` its
    cache shard.  Sequence splits (and page splits with one split per group)
    run the decode kernel alone and return ``[seqs, heads, D]``; page splits
    return the rows this rank owns, ``[rows_i, D]`` of the flattened
    ``[B * H_rank]`` output (``owner_rows``).  ``group`` is the process group of
    ``plan.split_group_ranks(rank)`` for page splits."""
    from .kernels.decode import launch_decode

    scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
    if plan.second == "sequence" or plan.splits == 1:
        k_scale = v_scale = None
        if scales is not None:
            k_scale = scales["k"] if isinstance(scales, dict) else scales.k
            v_scale = scales["v"] if isinstance(scales, dict) else scales.v
        return launch_decode(q, local_cache.k_cache, local_cache.v_cache, local_cache.page_table,
                             local_cache.seq_lens, local_cache.page_size, scale, k_scale=k_scale, v_scale=v_scale,
                             out_dtype=out_dtype)
    batch, heads, dim = q.shape
    packed = decode_partial(q, local_cache, scale, scales)
    parts = exchange_to_owners(packed, batch, heads, dim, group)
    rows = parts.shape[1] // (dim + 1)
    return merge_owned(parts, rows, dim, out_dtype or q.dtype)


__all__ = [
    "RankShard",
    "ShardPlan",
    "exchange_to_owners",
    "kv_head_range",
    "kv_head_slice",
    "merge_owned",
    "owner_rows",
    "packed_size",
    "plan_shards",
    "sequence_slice",
    "shard_cache",
    "shard_query",
    "sharded_decode",
]
