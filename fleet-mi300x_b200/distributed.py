"""Multi-GPU decode over one process per GPU (torch.distributed, NCCL over NVLink).

Two partitions of the attention task:

* **By request** (many independent sequences, BASELINE config 5a): each rank owns
  whole requests, their pages and block-table rows. There is no collective in the
  step; `request_shard` picks a rank's requests, balanced by cache rows.
* **By sequence** (one very long sequence, config 5b): each rank owns a
  page-aligned contiguous range of the sequence's cache rows; the rank owning the
  last range also stores the new token's row. Every rank runs K1/K2/K3 on its range
  with the global RoPE position and emits a 8.4 KB partial per request (y = W_UV o_c
  normalised within the range, plus the log2-domain max m and sum of exps L per
  head; W_UV is linear, so applying it before the exchange is exact). One
  all-gather moves the partials, and every rank combines them in sequence order
  (`mla_combine_shards`): the LSE merge the reference runs over its KV chunks
  inside one GPU (src/kernels/attention.h:358-401), one level up.
"""
from __future__ import annotations

import torch

from . import native
from .attention import MlaDecodeAttention, combine_shards
from .cache import PagedLatentCache
from .native import PAGE_SIZE


def sequence_shards(cached_rows: int, world: int, page: int = PAGE_SIZE) -> list[tuple[int, int]]:
    """Page-aligned contiguous ranges [start, end) of a sequence's cached rows over
    `world` ranks, as equal as whole pages allow. The new token (row `cached_rows`)
    belongs to the last range. Ranges may be empty when there are fewer pages than
    ranks (only the last rank is then guaranteed a row, the new one)."""
    if world <= 0 or cached_rows < 0:
        raise ValueError("world must be positive and cached_rows non-negative")
    total = cached_rows + 1                         # rows attended, the new one included
    pages = (total + page - 1) // page
    bounds = [min(cached_rows, (pages * r // world) * page) for r in range(world)] + [cached_rows]
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def request_shard(seq_lens, world: int, rank: int) -> list[int]:
    """Requests of `rank` when independent requests are spread over `world` ranks:
    greedy longest-first assignment to the least-loaded rank (by attended rows)."""
    order = sorted(range(len(seq_lens)), key=lambda b: -int(seq_lens[b]))
    load = [0] * world
    owner = [0] * len(seq_lens)
    for b in order:
        r = min(range(world), key=lambda x: (load[x], x))
        owner[b] = r
        load[r] += int(seq_lens[b]) + 1
    return [b for b in range(len(seq_lens)) if owner[b] == rank]


class SequenceShardedAttention:
    """The attention task of one layer for sequences split over ranks by KV range.

    Every rank holds a PagedLatentCache with its range of each sequence (local rows
    0..seq_lens[b]-1) and calls `step` with the same x_n and the global positions.
    Returns R(out) bf16 [B, 2048] on every rank.
    """

    def __init__(self, runner: MlaDecodeAttention, rank: int, world: int, group=None):
        self.runner = runner
        self.rank, self.world = rank, world
        self.group = group
        self._parts = None
        self._local = None

    def step(self, x_n: torch.Tensor, cache: PagedLatentCache, global_pos: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
        import torch.distributed as dist
        B = x_n.shape[0]
        dev = x_n.device
        if self._local is None or self._local.shape[0] != B:
            self._local = torch.empty(B, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
            self._parts = torch.empty(self.world, B, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
        q, kv_a = self.runner.project(x_n)
        owns_new = self.rank == self.world - 1
        self.runner.attend(q, kv_a, cache, rope_pos=global_pos, shard_out=self._local, new_row=owns_new)
        if self.world > 1:
            dist.all_gather_into_tensor(self._parts, self._local, group=self.group)
            parts = self._parts
        else:
            parts = self._local[None]
        return combine_shards(parts, out)


def emulate_sequence_shards(runner: MlaDecodeAttention, q: torch.Tensor, kv_a: torch.Tensor,
                            caches: list[PagedLatentCache], global_pos: torch.Tensor) -> torch.Tensor:
    """All ranges of a sequence-sharded step run one after another on one GPU
    (the last range owns the new token), then combined: the multi-GPU arithmetic
    without the all-gather, for testing on a single device."""
    B = q.shape[0]
    parts = torch.empty(len(caches), B, 16, native.SHARD_STRIDE, dtype=torch.float32, device=q.device)
    for r, cache in enumerate(caches):
        runner.attend(q, kv_a, cache, rope_pos=global_pos, shard_out=parts[r], new_row=(r == len(caches) - 1))
    return combine_shards(parts)
