"""Prefill hand-off: a prefill's latent rows into the paged cache.

The reference hands prefill states to decode as one flat cache per layer,
[max_pos][576] bf16 rows c (after kv_a_layernorm) | k_pe (after RoPE), written by
src/host/kv_convert.py:124-139 as raw bf16 [layers][max_pos][576] (positions past the
prefill are zero) and uploaded as-is by src/host/fleet_launch.hip:651-669. Here the
cache is paged: `rows_to_pages` scatters each request's rows into its pages on the GPU
(libmla_decode.so: mla_rows_to_pages), either finished rows (the file's format) or raw
kv_a rows, to which it applies kv_a_layernorm and RoPE at each row's position with the
arithmetic of the decode step's own appended row.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import torch

from . import native
from .attention import _ptr
from .cache import PagedLatentCache
from .native import ROW

ROW_BYTES = ROW * 2


def rows_to_pages(cache: PagedLatentCache, rows: torch.Tensor, row_start, first_pos=None, *, raw: bool = False,
                  norm_w: torch.Tensor | None = None, cos: torch.Tensor | None = None,
                  sin: torch.Tensor | None = None, eps: float = 1e-6,
                  error_word: torch.Tensor | None = None) -> None:
    """Write rows[row_start[b]:row_start[b+1]] of request b at positions first_pos[b] + i.

    rows: bf16 [total, >= 576] on the cache's device; row_start: [batch + 1] (host or
    device, int); first_pos: [batch] or None (= 0). raw=True takes kv_a rows and needs
    norm_w (kv_a_layernorm weight) and the YaRN tables cos/sin. Does not change seq_lens.
    """
    dev = cache.device
    if rows.dtype != torch.bfloat16 or rows.dim() != 2 or rows.shape[1] < ROW or rows.stride(1) != 1:
        raise ValueError("rows must be bf16 [n, >= 576] with contiguous rows")
    starts = torch.as_tensor(row_start, dtype=torch.int64).to(dev)
    if starts.dim() != 1 or starts.numel() != cache.batch + 1:
        raise ValueError(f"row_start needs batch + 1 = {cache.batch + 1} entries")
    total = int(starts[-1].item())
    if total > rows.shape[0]:
        raise ValueError(f"row_start ends at {total} but only {rows.shape[0]} rows were given")
    pos = None if first_pos is None else torch.as_tensor(first_pos, dtype=torch.int32).to(dev)
    r = native.new_rows()
    r.mode = native.ROWS_RAW if raw else native.ROWS_FINAL
    r.batch = cache.batch
    r.total_rows = total
    r.rows, r.rows_stride = _ptr(rows), rows.stride(0) if rows.shape[0] > 1 else rows.shape[1]
    r.row_start, r.first_pos = _ptr(starts), _ptr(pos)
    r.block_table, r.max_blocks, r.n_pages = _ptr(cache.block_table), cache.max_blocks, cache.n_pages
    r.kv_cache = _ptr(cache.pages)
    if raw:
        if norm_w is None or cos is None or sin is None:
            raise ValueError("raw rows need norm_w, cos and sin")
        r.kv_a_norm_w, r.rope_cos, r.rope_sin = _ptr(norm_w), _ptr(cos), _ptr(sin)
        r.max_pos, r.rms_eps = cos.shape[0], eps
    r.error_word = _ptr(error_word)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    native.check(native.load_library().mla_rows_to_pages(ctypes.byref(r), stream), "mla_rows_to_pages")


def read_flat_cache(path: str | Path, layers: int, max_pos: int) -> torch.Tensor:
    """The reference's cache file (raw bf16 [layers][max_pos][576], C order) as a CPU
    bf16 tensor [layers, max_pos, 576]."""
    data = np.fromfile(path, dtype=np.int16)
    if data.size != layers * max_pos * ROW:
        raise ValueError(f"{path}: {data.size * 2} bytes, expected {layers * max_pos * ROW_BYTES}")
    return torch.from_numpy(data.reshape(layers, max_pos, ROW)).view(torch.bfloat16)


def write_flat_cache(path: str | Path, flat: torch.Tensor) -> None:
    """Write bf16 [layers, max_pos, 576] in the reference's cache-file layout."""
    if flat.dtype != torch.bfloat16 or flat.dim() != 3 or flat.shape[2] != ROW:
        raise ValueError("flat must be bf16 [layers, max_pos, 576]")
    flat.contiguous().view(torch.int16).numpy().tofile(path)


def caches_from_flat(flat: torch.Tensor, prefill_len: int, *, extra_tokens: int = 1, device="cuda",
                     permute: bool = True, generator: torch.Generator | None = None) -> list[PagedLatentCache]:
    """One single-request PagedLatentCache per layer holding rows 0..prefill_len-1 of the
    flat cache [layers, max_pos, 576] (e.g. from read_flat_cache), with seq_lens =
    prefill_len and room for extra_tokens more rows."""
    layers, max_pos, _ = flat.shape
    if not 0 <= prefill_len <= max_pos:
        raise ValueError(f"prefill_len {prefill_len} outside [0, {max_pos}]")
    out = []
    for l in range(layers):
        cache = PagedLatentCache.for_lengths([prefill_len], extra_tokens=extra_tokens, permute=permute,
                                             generator=generator, device=device)
        if prefill_len:
            rows = flat[l, :prefill_len].to(device)
            rows_to_pages(cache, rows, [0, prefill_len])
        out.append(cache)
    return out
