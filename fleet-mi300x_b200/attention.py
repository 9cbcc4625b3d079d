"""Host side of the attention task: the drop-in for reference_decode.attention_absorbed.

The reference's `attention_absorbed(cfg, w, x, cache, pos, cos, sin)`
(src/host/reference_decode.py:210-256) normalises x, projects q and kv_a, appends
this token's cache row, attends and returns o_proj of the result. The north-star
slice kept here starts at the post-RMSNorm hidden state x_n (:224) and ends at the
head-concatenated bf16 output R(out) before o_proj (:256):

    K0 project   q, kv_a = R(W_q x_n), R(W_kv_a x_n) with the fused [W_q; W_kv_a]: a
                 weight stream up to 64 requests, a tcgen05 GEMM beyond   (libmla_decode.so;
                 above 64 requests __call__ uses cuBLAS instead, measured faster here)
    K1 prologue  kv_post + cache append + q_pe RoPE + q_c = q_nope W_UK      (libmla_decode.so)
    K2 attention split-KV scores, online softmax, P c_kv (m16n8k16 MMAs)    (libmla_decode.so)
    K3 merge     fixed-order LSE merge + W_UV up-projection, bf16 out       (libmla_decode.so)

All of it runs in the C-ABI library; there is no CPU path. project() below is a
cuBLAS GEMM through torch: __call__ takes it above 64 requests, where the library's
own tcgen05 GEMM is slower (17.4 against 12.9 us at 256 requests: it uses no cluster
multicast loads, so each of its CTAs streams its rows of x_n itself), and callers that
want q / kv_a themselves use it.
"""
from __future__ import annotations

import ctypes
import weakref
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from . import native
from .cache import PagedLatentCache
from .config import ModelConfig, rope_tables


@dataclass
class LayerWeights:
    """The attention weights of one layer, as device tensors (names follow HF /
    reference_decode.LayerWeights, reference_decode.py:139-159)."""

    q_proj: torch.Tensor               # [heads*192, hidden] bf16
    kv_a_proj_with_mqa: torch.Tensor   # [576, hidden] bf16
    kv_a_layernorm: torch.Tensor       # [512] bf16
    kv_b_proj: torch.Tensor            # [heads*256, 512] bf16
    o_proj: torch.Tensor | None = None  # [hidden, heads*v_head] bf16 (optional: attention_block)

    def fused_qkv(self) -> torch.Tensor:
        return torch.cat([self.q_proj, self.kv_a_proj_with_mqa], dim=0).contiguous()


def device_rope_tables(cfg: ModelConfig, max_pos: int, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    cos, sin = rope_tables(cfg, max_pos)
    return (torch.from_numpy(np.ascontiguousarray(cos)).to(device),
            torch.from_numpy(np.ascontiguousarray(sin)).to(device))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _row_stride(t: torch.Tensor) -> int:
    """Elements between rows of a [B, n] tensor. For B = 1 torch may report any
    stride for the batch dimension (0 for a broadcast view), so use the row length."""
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


class MlaDecodeAttention:
    """One layer's attention task over a PagedLatentCache.

    Owns the fused q|kv_a weight, the workspace and a device error word; the
    library itself allocates nothing. Calls are stream-ordered on the current
    torch stream and can be captured in a CUDA graph.
    """

    def __init__(self, cfg: ModelConfig, w: LayerWeights, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                 *, num_ctas: int = 0, check_kernel: bool = False, kernel: str = "mma", qc_hilo: bool = False,
                 p_hilo: bool = False):
        """qc_hilo / p_hilo (default kernel only): keep the absorbed query, and the
        probabilities of P c_kv, as bf16 hi/lo pairs instead of rounding them to bf16
        (MLA_FLAG_QC_HILO / MLA_FLAG_P_HILO), closer to the reference's fp32 q_c and P
        (reference_decode.py:250-253) at the cost of more tensor-core issue in K2."""
        cfg.check_supported()
        self.cfg = cfg
        self.lib = native.load_library()
        dev = w.kv_b_proj.device
        if dev.type != "cuda":
            raise RuntimeError("MlaDecodeAttention needs CUDA tensors (sm_100a); there is no CPU path")
        self.device = dev
        self.w = w
        self.w_qkv = w.fused_qkv()
        self.w_o = None if w.o_proj is None else w.o_proj.contiguous()
        self.kv_b = w.kv_b_proj.contiguous()
        self.norm_w = w.kv_a_layernorm.contiguous()
        self.cos = rope_cos.contiguous().float()
        self.sin = rope_sin.contiguous().float()
        self.num_ctas = int(num_ctas)
        if kernel not in ("mma", "tcgen05"):
            raise ValueError("kernel must be 'mma' (m16n8k16, default) or 'tcgen05'")
        self.flags = native.FLAG_CHECK_KERNEL if check_kernel else (native.FLAG_TCGEN05 if kernel == "tcgen05" else 0)
        if (qc_hilo or p_hilo) and self.flags:
            raise ValueError("qc_hilo / p_hilo exist in the default (mma) kernel only")
        self.flags |= (native.FLAG_QC_HILO if qc_hilo else 0) | (native.FLAG_P_HILO if p_hilo else 0)
        self.error_word = torch.zeros(1, dtype=torch.int32, device=dev)
        # pinned host copy of the error word: the kernels store a code into it when they
        # record one (MlaDecodeParams.error_host), so the host sees a failed step
        # without synchronising, also when the step was replayed from a CUDA graph
        self.error_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._ws: torch.Tensor | None = None
        self._step_key: tuple | None = None   # attend(): params of the last call, reused for the same tensors
        self._step_p: native.MlaDecodeParams | None = None

    # ------------------------------------------------------------------ params
    def params(self, q: torch.Tensor | None, kv_a: torch.Tensor | None, cache: PagedLatentCache,
               out: torch.Tensor | None, *, rope_pos: torch.Tensor | None = None,
               shard_out: torch.Tensor | None = None, new_row: bool = True,
               x_n: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               h_out: torch.Tensor | None = None, exchange=None) -> native.MlaDecodeParams:
        """The C-ABI params of one step. With `x_n` (and q = kv_a = None) the library
        projects q | kv_a itself with the fused [W_q; W_kv_a] weight (K0); with
        `residual` and `h_out` it ends with h_out = R(residual + R(W_o R(out))) (K5);
        with `exchange` (distributed.ExchangeBuffers) the step is one shard of a
        sequence-sharded step and ends with the peer exchange and combine (K4)."""
        B = (x_n if x_n is not None else q).shape[0]
        p = native.new_params()
        p.softmax_scale = self.cfg.softmax_scale
        p.rms_eps = self.cfg.rms_eps
        p.batch = B
        p.max_blocks = cache.max_blocks
        p.n_pages = cache.n_pages
        p.max_pos = self.cos.shape[0]
        if x_n is not None:
            p.x_n, p.x_stride, p.w_qkv = _ptr(x_n), _row_stride(x_n), _ptr(self.w_qkv)
        else:
            p.q, p.q_stride = _ptr(q), _row_stride(q)
            p.kv_a, p.kv_a_stride = _ptr(kv_a), _row_stride(kv_a)
        p.kv_a_norm_w = _ptr(self.norm_w)
        p.kv_b = _ptr(self.kv_b)
        p.rope_cos, p.rope_sin = _ptr(self.cos), _ptr(self.sin)
        p.block_table = _ptr(cache.block_table)
        p.seq_lens = _ptr(cache.seq_lens)
        p.kv_cache = _ptr(cache.pages)
        p.out = _ptr(out)
        p.out_stride = _row_stride(out) if out is not None else self.cfg.heads * self.cfg.v_head
        p.error_word = _ptr(self.error_word)
        p.error_host = _ptr(self.error_host)
        p.num_ctas = self.num_ctas
        p.flags = self.flags | (0 if new_row else native.FLAG_NO_NEW_ROW)
        p.rope_pos = _ptr(rope_pos)
        p.shard_out = _ptr(shard_out)
        if exchange is not None:
            exchange.apply(p)
        if h_out is not None:
            if self.w_o is None:
                raise ValueError("o_proj + residual needs LayerWeights.o_proj")
            p.w_o = _ptr(self.w_o)
            p.residual, p.residual_stride = _ptr(residual), _row_stride(residual)
            p.h_out, p.h_out_stride = _ptr(h_out), _row_stride(h_out)
        need = ctypes.c_uint64()
        native.check(self.lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(need)), "mla_workspace_size")
        if self._ws is None or self._ws.numel() < need.value:
            self._ws = torch.empty(int(need.value), dtype=torch.uint8, device=self.device)
        p.workspace = _ptr(self._ws)
        p.workspace_bytes = self._ws.numel()
        return p

    def _check_inputs(self, q, kv_a, cache):
        if q.dtype != torch.bfloat16 or kv_a.dtype != torch.bfloat16:
            raise TypeError("q and kv_a must be bf16")
        if q.shape[0] != cache.batch or kv_a.shape[0] != cache.batch:
            raise ValueError(f"batch {q.shape[0]} does not match the cache's {cache.batch} requests")
        if q.dim() != 2 or kv_a.dim() != 2 or q.shape[1] != self.cfg.heads * self.cfg.q_head_dim or \
                kv_a.shape[1] != self.cfg.kv_lora_rank + self.cfg.qk_rope:
            raise ValueError(f"q must be [B, 3072] and kv_a [B, 576], got {tuple(q.shape)} and {tuple(kv_a.shape)}")
        if q.stride(-1) != 1 or kv_a.stride(-1) != 1:
            raise ValueError("q and kv_a rows must be contiguous")

    # ------------------------------------------------------------------ calls
    def attend(self, q: torch.Tensor, kv_a: torch.Tensor, cache: PagedLatentCache,
               out: torch.Tensor | None = None, stage: str = "all", *, rope_pos: torch.Tensor | None = None,
               shard_out: torch.Tensor | None = None, new_row: bool = True, exchange=None,
               check: bool | str = True) -> torch.Tensor:
        """K1+K2+K3 from q [B, 3072] and kv_a [B, 576] (bf16 views allowed).
        Appends each request's row at seq_lens[b]; does not advance seq_lens.

        Sequence-sharded use: `rope_pos` gives the new token's global position,
        `new_row=False` marks a shard that does not own the new token, and either
        `shard_out` (f32 [B, 16, 132]) receives this shard's partial instead of
        R(out), to be gathered and combined with `combine_shards`, or `exchange`
        (this rank's distributed.ExchangeBuffers) moves the partials between the
        ranks' GPUs inside the step, which then returns the combined R(out) (stage
        "combine" runs K4 alone).

        `check` (see raise_pending): True raises, before launching, a device error
        that an earlier call recorded (no synchronisation); "sync" also waits for this
        call and raises its own error; False skips both."""
        self._pre_check(check)
        self._check_inputs(q, kv_a, cache)
        if exchange is not None:
            if shard_out is not None:
                raise ValueError("shard_out and exchange are exclusive")
            if q.shape[0] > exchange.max_batch:
                raise ValueError(f"batch {q.shape[0]} exceeds the exchange buffers' {exchange.max_batch}")
        if shard_out is not None:
            if shard_out.dtype != torch.float32 or tuple(shard_out.shape) != (q.shape[0], 16, native.SHARD_STRIDE):
                raise ValueError(f"shard_out must be f32 [{q.shape[0]}, 16, {native.SHARD_STRIDE}]")
            out = None
        elif out is None:
            out = torch.empty(q.shape[0], self.cfg.heads * self.cfg.v_head, dtype=torch.bfloat16,
                              device=self.device)
        key = (q.data_ptr(), _row_stride(q), kv_a.data_ptr(), _row_stride(kv_a), cache.pages.data_ptr(),
               cache.block_table.data_ptr(), cache.seq_lens.data_ptr(), cache.n_pages, cache.max_blocks,
               q.shape[0], _ptr(out), None if out is None else _row_stride(out), _ptr(rope_pos), _ptr(shard_out),
               new_row, self.flags, self.num_ctas, self.cos.data_ptr(), self.cos.shape[0], self.kv_b.data_ptr(),
               None if exchange is None else exchange.key)
        p = self._step_p
        if key != self._step_key or self._ws is None or p.workspace != self._ws.data_ptr():
            p = self.params(q, kv_a, cache, out, rope_pos=rope_pos, shard_out=shard_out, new_row=new_row,
                            exchange=exchange)
            self._step_key, self._step_p = key, p
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        fn = {"all": self.lib.mla_decode_step, "prologue": self.lib.mla_prologue,
              "attention": self.lib.mla_attention, "merge": self.lib.mla_merge_uv,
              "combine": self.lib.mla_exchange_combine}[stage]
        native.check(fn(ctypes.byref(p), stream), f"mla {stage}", p)
        self._post_check(check)
        return out if shard_out is None else shard_out

    def attend_x(self, x_n: torch.Tensor, cache: PagedLatentCache, out: torch.Tensor | None = None,
                 stage: str = "all", *, check: bool | str = True) -> torch.Tensor:
        """The whole slice in the library, from the post-RMSNorm hidden state x_n
        [B, 2048] bf16: K0 projects q | kv_a, then K1-K3 as in attend()."""
        self._pre_check(check)
        self._check_x(x_n, cache)
        if out is None:
            out = torch.empty(x_n.shape[0], self.cfg.heads * self.cfg.v_head, dtype=torch.bfloat16,
                              device=self.device)
        key = ("x", x_n.data_ptr(), _row_stride(x_n), cache.pages.data_ptr(), cache.block_table.data_ptr(),
               cache.seq_lens.data_ptr(), cache.n_pages, cache.max_blocks, x_n.shape[0], out.data_ptr(),
               _row_stride(out), self.flags, self.num_ctas, self.cos.data_ptr(), self.cos.shape[0],
               self.kv_b.data_ptr())
        p = self._step_p
        if key != self._step_key or self._ws is None or p.workspace != self._ws.data_ptr():
            p = self.params(None, None, cache, out, x_n=x_n)
            self._step_key, self._step_p = key, p
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        fn = {"all": self.lib.mla_decode_step, "project": self.lib.mla_project, "prologue": self.lib.mla_prologue,
              "attention": self.lib.mla_attention, "merge": self.lib.mla_merge_uv}[stage]
        native.check(fn(ctypes.byref(p), stream), f"mla {stage}", p)
        self._post_check(check)
        return out

    def attention_block(self, x_n: torch.Tensor, cache: PagedLatentCache, residual: torch.Tensor,
                        h_out: torch.Tensor | None = None, out: torch.Tensor | None = None, *,
                        check: bool | str = True) -> torch.Tensor:
        """The attention half of a decoder layer (reference_decode.py:300):
        h_out = R(residual + R(W_o R(attention(x_n)))), with R(out) left in `out`.
        Decode batches (<= 64 requests) run as one library call, K0 through K5;
        larger ones (and inputs that break the library's alignment rules) use cuBLAS
        for the two projections around attend(), as __call__ does."""
        B = x_n.shape[0]
        if self.w_o is None:
            raise ValueError("attention_block needs LayerWeights.o_proj")
        if residual.dtype != torch.bfloat16 or tuple(residual.shape) != (B, self.cfg.hidden):
            raise ValueError(f"residual must be bf16 [{B}, {self.cfg.hidden}]")
        if h_out is None:
            h_out = torch.empty_like(residual)
        if out is None:
            out = torch.empty(B, self.cfg.heads * self.cfg.v_head, dtype=torch.bfloat16, device=self.device)
        fused = (B <= native.MAX_PROJECT_BATCH and x_n.stride(-1) == 1 and x_n.data_ptr() % 16 == 0
                 and _row_stride(x_n) % 8 == 0 and out.data_ptr() % 16 == 0 and _row_stride(out) % 8 == 0
                 and residual.stride(-1) == 1 and h_out.stride(-1) == 1 and _row_stride(residual) % 4 == 0
                 and _row_stride(h_out) % 4 == 0)
        if not fused:
            attn = self(x_n, cache, out, check=check)
            h_out.copy_(residual + torch.nn.functional.linear(attn, self.w_o))
            return h_out
        self._pre_check(check)
        self._check_x(x_n, cache)
        p = self.params(None, None, cache, out, x_n=x_n, residual=residual, h_out=h_out)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        native.check(self.lib.mla_decode_step(ctypes.byref(p), stream), "mla attention block", p)
        self._post_check(check)
        return h_out

    def _check_x(self, x_n: torch.Tensor, cache: PagedLatentCache) -> None:
        if x_n.dtype != torch.bfloat16 or x_n.dim() != 2 or x_n.shape[1] != self.cfg.hidden:
            raise ValueError(f"x_n must be bf16 [B, {self.cfg.hidden}], got {x_n.dtype} {tuple(x_n.shape)}")
        if x_n.stride(-1) != 1:
            raise ValueError("x_n rows must be contiguous")
        if x_n.shape[0] != cache.batch:
            raise ValueError(f"batch {x_n.shape[0]} does not match the cache's {cache.batch} requests")

    def project(self, x_n: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """q = R(W_q x_n), kv_a = R(W_kv_a x_n) as views of one bf16 GEMM output.
        (torch.mm against the transposed view: at B = 256 with cold weights cuBLAS runs
        it in 13.3 us against 17.1 us for F.linear; inside the pipelined decode loop the
        two measured the same within run-to-run noise.)"""
        qkv = torch.mm(x_n, self.w_qkv.t())
        nq = self.cfg.heads * self.cfg.q_head_dim
        return qkv[:, :nq], qkv[:, nq:]

    def __call__(self, x_n: torch.Tensor, cache: PagedLatentCache,
                 out: torch.Tensor | None = None, *, check: bool | str = True) -> torch.Tensor:
        """x_n -> R(out). Decode batches (<= 64 requests) run the projection in the
        library (attend_x: a weight stream at HBM rate); larger batches project with
        cuBLAS (see project()) and then attend(). `check` as in attend()."""
        if x_n.shape[0] <= native.MAX_PROJECT_BATCH and x_n.stride(-1) == 1 and \
                x_n.data_ptr() % 16 == 0 and _row_stride(x_n) % 8 == 0:
            return self.attend_x(x_n, cache, out, check=check)
        self._pre_check(check)
        q, kv_a = self.project(x_n)
        return self.attend(q, kv_a, cache, out, check=check)

    # ------------------------------------------------------------------ device errors
    def raise_pending(self) -> None:
        """Raise MlaError if a kernel of an earlier call (eager or replayed from a graph)
        has recorded a device error. Reads the pinned host word the kernels store the
        code into; no synchronisation, so a step still running is seen once it has
        stored. Clears both words before raising."""
        code = int(self.error_host[0])
        if code:
            self.error_host.zero_()
            if not torch.cuda.is_current_stream_capturing():
                self.error_word.zero_()
            raise native.MlaError(code, "device (a step since the last check)")

    def _pre_check(self, check) -> None:
        if check and not torch.cuda.is_current_stream_capturing():
            self.raise_pending()

    def _post_check(self, check) -> None:
        if check == "sync" and not torch.cuda.is_current_stream_capturing():
            torch.cuda.current_stream(self.device).synchronize()
            self.raise_pending()

    def check_errors(self, reset: bool = True) -> None:
        """Raise if a kernel recorded a device error (synchronises with the device)."""
        code = int(self.error_word.item()) or int(self.error_host[0])
        if reset and code:
            self.error_word.zero_()
            self.error_host.zero_()
        if code:
            raise native.MlaError(code, "device")

    def workspace_bytes(self, batch: int) -> int:
        p = native.new_params()
        p.batch = batch
        p.num_ctas = self.num_ctas
        p.flags = self.flags
        need = ctypes.c_uint64()
        native.check(self.lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(need)), "mla_workspace_size")
        return int(need.value)


def combine_shards(parts: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Fixed-order LSE combine of gathered shard partials f32 [n_shards, B, 16, 132]
    (sequence order) into R(out) bf16 [B, 2048] (libmla_decode.so: mla_combine_shards)."""
    if parts.dtype != torch.float32 or parts.dim() != 4 or parts.shape[2:] != (16, native.SHARD_STRIDE):
        raise ValueError("parts must be f32 [n_shards, B, 16, 132]")
    parts = parts.contiguous()
    n, B = parts.shape[0], parts.shape[1]
    if out is None:
        out = torch.empty(B, 2048, dtype=torch.bfloat16, device=parts.device)
    lib = native.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream(parts.device).cuda_stream)
    native.check(lib.mla_combine_shards(parts.data_ptr(), n, B, out.data_ptr(), _row_stride(out), stream),
                 "mla_combine_shards")
    return out


def attention_absorbed(cfg: ModelConfig, w: LayerWeights, x_n: torch.Tensor, cache: PagedLatentCache,
                       pos=None, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                       *, runner: MlaDecodeAttention | None = None) -> torch.Tensor:
    """Drop-in for the attention slice of reference_decode.attention_absorbed.

    x_n: post-RMSNorm hidden state, bf16 [hidden] or [B, hidden], on the GPU.
    cache: PagedLatentCache; request b's new row is written at `pos` (an int for
    B = 1, a sequence, or None to use cache.seq_lens) and attention runs over rows
    0..pos inclusive. As in the reference, the cache is appended in place and the
    caller advances positions (cache.advance()).
    Returns R(out): bf16 [B, heads*v_head] (or [heads*v_head] for 1-D x_n), the
    head-concatenated attention output before o_proj.
    Without `runner`, one MlaDecodeAttention per weight set is kept (up to 64, the
    layers of a model), so that repeated calls reuse its fused weight and workspace.
    A device error that an earlier call recorded (bad page, bad position) is raised
    at the next call, without synchronising (MlaDecodeAttention.raise_pending).
    """
    squeeze = x_n.dim() == 1
    if squeeze:
        x_n = x_n[None, :]
    if pos is not None:
        pos_t = torch.as_tensor(np.atleast_1d(np.asarray(pos, dtype=np.int32)))
        cache.seq_lens.copy_(pos_t.to(cache.device))
    if runner is None:
        if cos is None or sin is None:
            raise ValueError("cos/sin tables are required (device_rope_tables)")
        runner = _cached_runner(cfg, w, cos, sin)
    out = runner(x_n, cache)
    return out[0] if squeeze else out


# attention_absorbed without `runner=`: one MlaDecodeAttention per weight set (the layers
# of a model), so that a decode loop does not rebuild the 14.9 MB fused [W_q; W_kv_a] and
# a workspace at every token. An entry is reused only for the very same tensor objects,
# unmodified since (torch's in-place version counter) and the same config; the runner
# holds them alive, so the cache is bounded.
_RUNNER_CACHE_SIZE = 64
_runners: "OrderedDict[tuple, tuple[list, MlaDecodeAttention]]" = OrderedDict()


def _cached_runner(cfg: ModelConfig, w: LayerWeights, cos: torch.Tensor, sin: torch.Tensor) -> MlaDecodeAttention:
    tensors = (w.q_proj, w.kv_a_proj_with_mqa, w.kv_a_layernorm, w.kv_b_proj, cos, sin)
    key = tuple((t.data_ptr(), tuple(t.shape), t.dtype, t._version) for t in tensors) + (
        cfg.softmax_scale, cfg.rms_eps)
    hit = _runners.get(key)
    if hit is not None and all(r() is t for r, t in zip(hit[0], tensors)):
        _runners.move_to_end(key)
        return hit[1]
    runner = MlaDecodeAttention(cfg, w, cos, sin)
    _runners[key] = ([weakref.ref(t) for t in tensors], runner)
    while len(_runners) > _RUNNER_CACHE_SIZE:
        _runners.popitem(last=False)
    return runner
