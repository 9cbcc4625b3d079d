"""Multi-GPU decode over one process per GPU (torch.distributed, NCCL over NVLink).

Two partitions of the attention task:

* **By request** (many independent sequences, config 5a): each rank owns
  whole requests, their pages and block-table rows. There is no collective in the
  step; `request_shard` picks a rank's requests, balanced by cache rows.
* **By sequence** (one very long sequence, config 5b): each rank owns a
  page-aligned contiguous range of the sequence's cache rows; the rank owning the
  last range also stores the new token's row. Every rank runs K1/K2/K3 on its range
  with the global RoPE position and emits a 8.4 KB partial per request (y = W_UV o_c
  normalised within the range, plus the log2-domain max m and sum of exps L per
  head; W_UV is linear, so applying it before the exchange is exact). The partials
  reach every rank and are combined there in sequence order: the LSE merge the
  reference runs over its KV chunks inside one GPU (src/kernels/attention.h:358-401),
  one level up. Two ways to move them:
  - peer exchange (`ExchangeBuffers`, the default): K3 stores its partial straight
    into every rank's exchange buffer over NVLink and raises flags there; K4 waits
    for the flags and combines. The whole step is one library call, no NCCL.
  - NCCL: K3 writes a local partial, `all_gather_into_tensor` moves it and
    `mla_combine_shards` combines.
"""
from __future__ import annotations

import ctypes

import torch

from . import native
from .attention import MlaDecodeAttention, combine_shards
from .cache import PagedLatentCache
from .native import PAGE_SIZE


def exchange_bytes(world: int, max_batch: int) -> int:
    """Bytes of one rank's exchange buffer (mla_exchange_bytes)."""
    n = ctypes.c_uint64()
    native.check(native.load_library().mla_exchange_bytes(world, max_batch, ctypes.byref(n)), "mla_exchange_bytes")
    return int(n.value)


def gather_handles(handle: bytes, world: int, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order (a collective over `group`). The
    bytes travel as a uint8 tensor: on the current CUDA device for NCCL, on the
    CPU for gloo."""
    import torch.distributed as dist
    if len(handle) != native.IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {native.IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    mine = torch.frombuffer(bytearray(handle), dtype=torch.uint8).to(dev)
    allh = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allh, mine, group=group)
    return [bytes(t.cpu().numpy().tobytes()) for t in allh]


class ExchangeBuffers:
    """The exchange buffers of a sequence-sharded step as one rank sees them: the
    address of every rank's buffer in this process, this rank's index, the world
    and the batch the buffers hold. `apply` puts them into a step's params; the
    step then ends with the peer exchange and the combine (K3 stores, K4 combines).

    `create` is the multi-process form (one process per GPU, a collective over the
    process group); `local` makes `world` buffers on one device, one view per
    emulated rank, for running all shards of a step on one GPU.
    """

    def __init__(self, ptrs: list[int], rank: int, world: int, max_batch: int, *, timeout_us: int = 0,
                 owned: tuple[int, ...] = (), opened: tuple[int, ...] = ()):
        if not 1 <= world <= native.MAX_RANKS or not 0 <= rank < world or len(ptrs) != world:
            raise ValueError(f"need 1 <= world <= {native.MAX_RANKS}, 0 <= rank < world and one pointer per rank")
        self.ptrs, self.rank, self.world, self.max_batch = list(ptrs), rank, world, max_batch
        self.timeout_us = int(timeout_us)
        self._owned, self._opened = list(owned), list(opened)

    @property
    def key(self) -> tuple:
        return (tuple(self.ptrs), self.rank, self.world, self.max_batch, self.timeout_us)

    def apply(self, p: native.MlaDecodeParams) -> None:
        for r in range(native.MAX_RANKS):
            p.exchange[r] = self.ptrs[r] if r < self.world else None
        p.rank, p.world = self.rank, self.world
        p.exchange_batch = self.max_batch
        p.exchange_timeout_us = self.timeout_us

    @classmethod
    def create(cls, rank: int, world: int, max_batch: int, group=None, *, timeout_us: int = 0) -> "ExchangeBuffers":
        """Allocate this rank's buffer on the current device and map every other
        rank's (CUDA IPC). Collective: every rank of `group` calls it with the same
        world and max_batch. Ends with a barrier, so that no rank's first step
        writes into a buffer that its owner has not yet zeroed."""
        import torch.distributed as dist
        lib = native.load_library()
        buf = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * native.IPC_HANDLE_BYTES)()
        native.check(lib.mla_exchange_alloc(exchange_bytes(world, max_batch), ctypes.byref(buf), handle),
                     "mla_exchange_alloc")
        handles = gather_handles(bytes(handle), world, group)
        ptrs, opened = [], []
        try:
            for r, h in enumerate(handles):
                if r == rank:
                    ptrs.append(buf.value)
                    continue
                peer = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * native.IPC_HANDLE_BYTES).from_buffer_copy(h)
                native.check(lib.mla_exchange_open(hb, ctypes.byref(peer)), f"mla_exchange_open (rank {r})")
                ptrs.append(peer.value)
                opened.append(peer.value)
        except Exception:
            for q in opened:
                lib.mla_exchange_close(q)
            lib.mla_exchange_free(buf)
            raise
        dist.barrier(group=group)
        return cls(ptrs, rank, world, max_batch, timeout_us=timeout_us, owned=(buf.value,), opened=tuple(opened))

    @classmethod
    def local(cls, world: int, max_batch: int, *, timeout_us: int = 0) -> list["ExchangeBuffers"]:
        """`world` buffers on the current device and one view per emulated rank; the
        first view owns (and frees) them all."""
        lib = native.load_library()
        ptrs = []
        for _ in range(world):
            buf = ctypes.c_void_p()
            native.check(lib.mla_exchange_alloc(exchange_bytes(world, max_batch), ctypes.byref(buf), None),
                         "mla_exchange_alloc")
            ptrs.append(buf.value)
        return [cls(ptrs, r, world, max_batch, timeout_us=timeout_us, owned=tuple(ptrs) if r == 0 else ())
                for r in range(world)]

    def close(self) -> None:
        """Unmap the peers' buffers and free the owned ones (after the last step has
        completed on every rank)."""
        lib = native.load_library()
        for q in self._opened:
            native.check(lib.mla_exchange_close(q), "mla_exchange_close")
        for q in self._owned:
            native.check(lib.mla_exchange_free(q), "mla_exchange_free")
        self._opened, self._owned = [], []


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
    Returns R(out) bf16 [B, 2048] on every rank. With `exchange` (ExchangeBuffers of
    this rank) the partials move by the peer exchange inside the library step;
    without, by an NCCL all-gather over `group`.
    """

    def __init__(self, runner: MlaDecodeAttention, rank: int, world: int, group=None,
                 exchange: ExchangeBuffers | None = None):
        if exchange is not None and (exchange.rank != rank or exchange.world != world):
            raise ValueError("the exchange buffers belong to another rank or world")
        self.runner = runner
        self.rank, self.world = rank, world
        self.group = group
        self.exchange = exchange
        self._parts = None
        self._local = None

    def step(self, x_n: torch.Tensor, cache: PagedLatentCache, global_pos: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
        import torch.distributed as dist
        B = x_n.shape[0]
        dev = x_n.device
        owns_new = self.rank == self.world - 1
        if self.exchange is not None:
            q, kv_a = self.runner.project(x_n)
            return self.runner.attend(q, kv_a, cache, out, rope_pos=global_pos, new_row=owns_new,
                                      exchange=self.exchange)
        if self._local is None or self._local.shape[0] != B:
            self._local = torch.empty(B, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
            self._parts = torch.empty(self.world, B, 16, native.SHARD_STRIDE, dtype=torch.float32, device=dev)
        q, kv_a = self.runner.project(x_n)
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


def emulate_exchange_step(runner: MlaDecodeAttention, q: torch.Tensor, kv_a: torch.Tensor,
                          caches: list[PagedLatentCache], global_pos: torch.Tensor,
                          exchange: list[ExchangeBuffers]) -> list[torch.Tensor]:
    """A peer-exchange step with all ranks on one GPU (`ExchangeBuffers.local`):
    K1-K3 of every rank one after another (each K3 stores into every rank's buffer),
    then every rank's K4. Each K4 thus starts after all flags it waits for are set;
    nothing waits on a kernel that runs at the same time. Returns every rank's R(out)."""
    world = len(caches)
    outs = [torch.empty(q.shape[0], 2048, dtype=torch.bfloat16, device=q.device) for _ in range(world)]
    for r in range(world):
        for stage in ("prologue", "attention", "merge"):
            runner.attend(q, kv_a, caches[r], outs[r], stage, rope_pos=global_pos, new_row=(r == world - 1),
                          exchange=exchange[r])
    for r in range(world):
        runner.attend(q, kv_a, caches[r], outs[r], "combine", rope_pos=global_pos, new_row=(r == world - 1),
                      exchange=exchange[r])
    return outs
