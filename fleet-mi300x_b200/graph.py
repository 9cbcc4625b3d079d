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

Device errors (a bad block-table entry or position, a timed-out wait) reach the host
without a synchronisation: the captured kernels store the code into the runner's
pinned host word (MlaDecodeParams.error_host), and every replay / submit / wait here
raises MlaError if an earlier step recorded one (MlaDecodeAttention.raise_pending).
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
        """Run the captured step on the current stream; returns `out`. Raises first if
        an earlier step recorded a device error."""
        self.runner.raise_pending()
        self.graph.replay()
        return self.out

    def synchronize(self) -> None:
        """Wait for the current stream and raise if a step recorded a device error."""
        torch.cuda.current_stream(self.runner.device).synchronize()
        self.runner.raise_pending()


class HostPipeline:
    """The host-facing decode loop of one layer: x_n from pinned host memory in, R(out)
    to pinned host memory out, with the copies of neighbouring steps overlapping the
    compute of this one.

    Two DecodeGraphs over double-buffered device x_n / out are replayed on a compute
    stream; the host-to-device copy of step k+1 and the device-to-host copy of step k-1
    run on two copy streams meanwhile, ordered by events. `submit(x_host)` queues one step
    and returns the pinned host tensor that will hold its R(out); that tensor is reused
    two steps later, so read it (after `wait()` or `synchronize()`) before then.
    """

    def __init__(self, runner: MlaDecodeAttention, cache: PagedLatentCache, *, advance: bool = False):
        cfg, dev, B = runner.cfg, runner.device, cache.batch
        bf = torch.bfloat16
        self.device = dev
        self.runner = runner
        self.x_dev = [torch.zeros(B, cfg.hidden, dtype=bf, device=dev) for _ in range(2)]
        self.out_dev = [torch.empty(B, cfg.heads * cfg.v_head, dtype=bf, device=dev) for _ in range(2)]
        self.out_host = [torch.empty(B, cfg.heads * cfg.v_head, dtype=bf).pin_memory() for _ in range(2)]
        self.graphs = [DecodeGraph(runner, cache, inputs="x_n", advance=advance, x_n=self.x_dev[i],
                                   out=self.out_dev[i]) for i in range(2)]
        self.compute = torch.cuda.Stream(dev)
        self.h2d = torch.cuda.Stream(dev)  # separate from d2h: the input copy of step k+1 must not
        self.d2h = torch.cuda.Stream(dev)  # queue behind the output copy of step k
        self.x_ready = [torch.cuda.Event() for _ in range(2)]
        self.done = [torch.cuda.Event() for _ in range(2)]
        self.out_read = [torch.cuda.Event() for _ in range(2)]
        self.k = 0
        self._used = [False, False]

    def submit(self, x_host: torch.Tensor) -> torch.Tensor:
        """Queue one step whose input is the pinned host tensor x_host [B, hidden] bf16.
        Raises first if an earlier step recorded a device error."""
        self.runner.raise_pending()
        i = self.k % 2
        with torch.cuda.stream(self.h2d):
            if self._used[i]:
                self.h2d.wait_event(self.done[i])  # x_dev[i] is free once step k-2 has computed
            self.x_dev[i].copy_(x_host, non_blocking=True)
            self.x_ready[i].record(self.h2d)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(self.x_ready[i])
            if self._used[i]:
                self.compute.wait_event(self.out_read[i])  # out_dev[i] copied out by step k-2
            self.graphs[i].replay()
            self.done[i].record(self.compute)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.done[i])
            self.out_host[i].copy_(self.out_dev[i], non_blocking=True)
            self.out_read[i].record(self.d2h)
        self._used[i] = True
        self.k += 1
        return self.out_host[i]

    def wait(self) -> None:
        """Block until every submitted step's R(out) is in host memory; raise MlaError
        if any of them recorded a device error."""
        for st in (self.h2d, self.compute, self.d2h):
            st.synchronize()
        self.runner.raise_pending()


class HostStepGraph:
    """One decode step of a layer from pinned host memory to pinned host memory as a
    single CUDA graph: the copy of x_n in, the step (the kernels DecodeGraph runs) and
    the copy of R(out) back, in order on one stream.

    For latency-bound use (one request or a few), where HostPipeline's overlap of
    neighbouring steps buys nothing and its hand-offs between three streams cost
    more than the copies themselves. Write the next input into `x_host`, call
    `replay()` on the current stream, synchronise, read `out_host`. The copies are
    real copies on every replay (graph memcpy nodes from and to pinned memory).
    """

    def __init__(self, runner: MlaDecodeAttention, cache: PagedLatentCache, *, advance: bool = False):
        cfg, dev, B = runner.cfg, runner.device, cache.batch
        bf = torch.bfloat16
        self.runner, self.cache = runner, cache
        self.x_host = torch.zeros(B, cfg.hidden, dtype=bf).pin_memory()
        self.out_host = torch.empty(B, cfg.heads * cfg.v_head, dtype=bf).pin_memory()
        self.x_dev = torch.zeros(B, cfg.hidden, dtype=bf, device=dev)
        self.out_dev = torch.empty(B, cfg.heads * cfg.v_head, dtype=bf, device=dev)
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
        self.x_dev.copy_(self.x_host, non_blocking=True)
        self.runner(self.x_dev, self.cache, self.out_dev)
        self.out_host.copy_(self.out_dev, non_blocking=True)

    def replay(self) -> torch.Tensor:
        """Queue the step on the current stream; returns `out_host` (valid once the
        stream has reached this point). Raises first if an earlier step recorded a
        device error."""
        self.runner.raise_pending()
        self.graph.replay()
        return self.out_host

    def synchronize(self) -> None:
        """Wait for the current stream and raise if a step recorded a device error."""
        torch.cuda.current_stream(self.runner.device).synchronize()
        self.runner.raise_pending()


def rms_norm_bf16(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """DeepseekV2RMSNorm of a bf16 hidden state with HF's two bf16 roundings
    (reference_decode.py:51-65): fp32 normalisation rounded to bf16, times the weight."""
    x32 = x.float()
    y = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return weight * y.to(torch.bfloat16)


class LayerStackGraph:
    """One decode step over a stack of layers as a single CUDA graph.

    The reference runs every layer of a token in one persistent launch
    (src/kernels/fleet_kernel.hip:938-1043). Here the layers' kernels are captured in
    order into one graph, so a step pays one graph launch instead of one per layer, and
    each layer's first kernel, a programmatic dependent launch, becomes resident while
    the previous layer's last kernel still runs (its weight copies start before its wait).

    mode="slice": layer l runs its attention task K1-K3 from its own q / kv_a buffers
      (self.q[l], self.kv_a[l]) over caches[l] into self.out[l]: the attention slice of
      every layer with its own weights and cache, the unit the per-layer-step metric counts.
      `attend_kw` is passed to every layer's MlaDecodeAttention.attend, e.g. rope_pos,
      new_row and exchange for one shard of a sequence-sharded step (the layers then
      share the exchange buffers: each layer's step is one step of its protocol).
    mode="block": the hidden state self.h [B, 2048] flows through the layers: for each l,
      x_n = RMSNorm(h, in_norms[l]) (torch), then runners[l].attention_block(x_n, caches[l],
      residual=h, h_out=h) (K0-K5: projection, attention, o_proj and the residual add in the
      library for batches up to 64), then `ffn(l, h)` if given (capturable torch ops that
      update h in place, e.g. the layer's FFN with its residual).

    With advance=True the graph also adds 1 to every cache's seq_lens. Device errors of any
    layer are raised by replay() / synchronize() (each runner's pinned host error word).
    """

    def __init__(self, runners, caches, *, mode: str = "slice", q=None, kv_a=None, h=None, in_norms=None,
                 ffn=None, advance: bool = False, attend_kw: dict | None = None):
        if mode not in ("slice", "block"):
            raise ValueError("mode must be 'slice' or 'block'")
        if len(runners) != len(caches) or not runners:
            raise ValueError("one cache per runner, at least one layer")
        self.runners, self.caches, self.mode, self.ffn = list(runners), list(caches), mode, ffn
        self.attend_kw = dict(attend_kw or {})
        r0, dev, B = runners[0], runners[0].device, caches[0].batch
        cfg, bf = r0.cfg, torch.bfloat16
        if any(c.batch != B for c in caches):
            raise ValueError("every layer's cache must hold the same batch")
        n = len(runners)
        if mode == "slice":
            self.q = q if q is not None else [torch.zeros(B, cfg.heads * cfg.q_head_dim, dtype=bf, device=dev)
                                              for _ in range(n)]
            self.kv_a = kv_a if kv_a is not None else [
                torch.zeros(B, cfg.kv_lora_rank + cfg.qk_rope, dtype=bf, device=dev) for _ in range(n)]
            self.out = [torch.empty(B, cfg.heads * cfg.v_head, dtype=bf, device=dev) for _ in range(n)]
        else:
            if in_norms is None or len(in_norms) != n:
                raise ValueError("mode 'block' needs one input RMSNorm weight per layer")
            self.in_norms = list(in_norms)
            self.h = h if h is not None else torch.zeros(B, cfg.hidden, dtype=bf, device=dev)
            self.x_n = torch.empty(B, cfg.hidden, dtype=bf, device=dev)
            self.attn = torch.empty(B, cfg.heads * cfg.v_head, dtype=bf, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # library set-up and workspaces before the capture
            self._params_warm()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
            if advance:
                for c in self.caches:
                    c.seq_lens.add_(1)

    def _params_warm(self) -> None:
        """Run each layer's library call once outside the capture (workspace allocation,
        per-device set-up); state that a step changes (rows, h) is restored after."""
        if self.mode == "slice":
            self._step()
            return
        h0 = self.h.clone()
        self._step()
        self.h.copy_(h0)

    def _step(self) -> None:
        if self.mode == "slice":
            for l, (r, c) in enumerate(zip(self.runners, self.caches)):
                r.attend(self.q[l], self.kv_a[l], c, self.out[l], **self.attend_kw)
            return
        for l, (r, c) in enumerate(zip(self.runners, self.caches)):
            self.x_n.copy_(rms_norm_bf16(self.h, self.in_norms[l], r.cfg.rms_eps))
            r.attention_block(self.x_n, c, self.h, h_out=self.h, out=self.attn)
            if self.ffn is not None:
                self.ffn(l, self.h)

    def _raise_pending(self) -> None:
        for r in self.runners:
            r.raise_pending()

    def replay(self) -> None:
        """Run the captured step on the current stream (raises first if an earlier step of
        any layer recorded a device error)."""
        self._raise_pending()
        self.graph.replay()

    def synchronize(self) -> None:
        """Wait for the current stream and raise if a step recorded a device error."""
        torch.cuda.current_stream(self.runners[0].device).synchronize()
        self._raise_pending()
