"""Paged latent KV cache of one layer and its block table.

The reference keeps one flat cache per layer, `[max_pos][kv_lora + qk_rope]` bf16
(src/runtime/fleet_types.h:106-111, src/host/kv_convert.py:36-59), appended in place
at `pos` (reference_decode.py:236-237). Here the same 576-wide rows (c_kv | k_pe,
k_pe already RoPE'd) live in 64-row pages `[n_pages][64][576]` bf16; request b's
logical row t is page `block_table[b][t // 64]`, slot `t % 64`. `seq_lens[b]` is the
number of rows already cached, i.e. the position of the token being decoded.
"""
from __future__ import annotations

import torch

from .native import PAGE_SIZE, ROW


class PagedLatentCache:
    def __init__(self, n_pages: int, batch: int, max_blocks: int, device: torch.device | str = "cuda",
                 zero: bool = True):
        if n_pages <= 0 or batch <= 0 or max_blocks <= 0:
            raise ValueError("n_pages, batch and max_blocks must be positive")
        alloc = torch.zeros if zero else torch.empty
        self.pages = alloc(n_pages, PAGE_SIZE, ROW, dtype=torch.bfloat16, device=device)
        self.block_table = torch.zeros(batch, max_blocks, dtype=torch.int32, device=device)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=device)

    @property
    def batch(self) -> int:
        return self.block_table.shape[0]

    @property
    def n_pages(self) -> int:
        return self.pages.shape[0]

    @property
    def max_blocks(self) -> int:
        return self.block_table.shape[1]

    @property
    def device(self) -> torch.device:
        return self.pages.device

    @classmethod
    def for_lengths(cls, lengths, *, extra_tokens: int = 1, spare_pages: int = 0, permute: bool = True,
                    generator: torch.Generator | None = None, device="cuda", zero: bool = True
                    ) -> "PagedLatentCache":
        """A cache whose request b can hold lengths[b] + extra_tokens rows, with
        seq_lens = lengths. Pages are handed out in a random permutation when
        `permute` (the fragmented layout of a long-running server)."""
        lengths = [int(x) for x in lengths]
        need = [(n + extra_tokens + PAGE_SIZE - 1) // PAGE_SIZE for n in lengths]
        total = max(1, sum(need) + spare_pages)
        max_blocks = max(1, max(need))
        cache = cls(total, len(lengths), max_blocks, device=device, zero=zero)
        order = (torch.randperm(total, generator=generator) if permute else torch.arange(total))
        order = order.to(torch.int32)
        bt = torch.zeros(len(lengths), max_blocks, dtype=torch.int32)
        off = 0
        for b, n in enumerate(need):
            bt[b, :n] = order[off:off + n]
            off += n
        cache.block_table.copy_(bt)
        cache.seq_lens.copy_(torch.tensor(lengths, dtype=torch.int32))
        return cache

    def _flat_index(self, b: int, start: int, n: int) -> torch.Tensor:
        t = torch.arange(start, start + n, device=self.device)
        pages = self.block_table[b].to(torch.int64)[t // PAGE_SIZE]
        return pages * PAGE_SIZE + (t % PAGE_SIZE)

    def write_rows(self, b: int, start: int, rows: torch.Tensor) -> None:
        """Store rows [n, 576] as request b's logical rows start..start+n-1 (set-up helper)."""
        flat = self.pages.view(-1, ROW)
        flat[self._flat_index(b, start, rows.shape[0])] = rows.to(device=self.device, dtype=torch.bfloat16)

    def read_rows(self, b: int, start: int, n: int) -> torch.Tensor:
        """Request b's logical rows start..start+n-1, [n, 576] bf16."""
        return self.pages.view(-1, ROW)[self._flat_index(b, start, n)]

    def advance(self, n: int = 1) -> None:
        """Count the rows appended by the last step (the reference's caller advances pos)."""
        self.seq_lens += n
