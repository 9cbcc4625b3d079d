"""One decode step of a layer as a CUDA graph.

The eager step costs one Python call, a ctypes call and three kernel launches on the
host per layer; at batch 1 that host time is longer than the kernels. `DecodeGraph`
captures the step once over fixed device buffers and replays it with one launch.
The reference avoids the same per-task launch cost with its persistent kernel
(src/kernels/fleet_kernel.hip:938-1043).

The captured kernels read `seq_lens`, the block table and the cache pages from
device memory when they run, so one graph serves every step of a decode loop: write
the next x_n into `graph.x_n` (or q / kv_a into `graph.q` / `graph.kv_a`), replay,
read `graph.out`. With `advance=True` the graph also adds 1 to `seq_lens`, as the
caller of the eager step does after each call.
"""
from __future__ import annotations

import torch

from .attention import MlaDecodeAttention
from .cache import PagedLatentCache


class DecodeGraph:
    """`runner`'s step over `cache` captured as a CUDA graph.

    inputs="x_n": the step from the post-RMSNorm hidden state (q|kv_a GEMM + K1-K3).
    inputs="qkv": the step from q [B, 3072] and kv_a [B, 576] (K1-K3 only).
    Set-up runs the step once eagerly on a side stream (library set-up, workspace,
    cuBLAS state), which writes a row into each request's next slot; the first
    replay writes that slot again.
    """

    def __init__(self, runner: MlaDecodeAttention, cache: PagedLatentCache, *, inputs: str = "x_n",
                 advance: bool = False, x_n: torch.Tensor | None = None, q: torch.Tensor | None = None,
                 kv_a: torch.Tensor | None = None, out: torch.Tensor | None = None):
        if inputs not in ("x_n", "qkv"):
            raise ValueError("inputs must be 'x_n' or 'qkv'")
        cfg, dev, B = runner.cfg, runner.device, cache.batch
        bf = torch.bfloat16
        self.runner, self.cache, self.inputs = runner, cache, inputs
        self.x_n = self.q = self.kv_a = None
        if inputs == "x_n":
            self.x_n = x_n if x_n is not None else torch.zeros(B, cfg.hidden, dtype=bf, device=dev)
        else:
            self.q = q if q is not None else torch.zeros(B, cfg.heads * cfg.q_head_dim, dtype=bf, device=dev)
            self.kv_a = kv_a if kv_a is not None else torch.zeros(B, cfg.kv_lora_rank + cfg.qk_rope, dtype=bf,
                                                                  device=dev)
        self.out = out if out is not None else torch.empty(B, cfg.heads * cfg.v_head, dtype=bf, device=dev)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
            if advance:
                cache.seq_lens.add_(1)

    def _step(self) -> None:
        if self.inputs == "x_n":
            self.runner(self.x_n, self.cache, self.out)
        else:
            self.runner.attend(self.q, self.kv_a, self.cache, self.out)

    def replay(self) -> torch.Tensor:
        """Run the captured step on the current stream; returns `out`."""
        self.graph.replay()
        return self.out
