"""ctypes binding of libmla_decode.so, the C ABI declared in include/mla_decode.h.

The library is the product: there is no Python or CPU implementation behind this
module. If the shared library is missing, loading fails loudly with the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libmla_decode.so"

ABI_VERSION = 6
HEADS, QK_NOPE, QK_ROPE, V_HEAD, KV_LORA, PAGE_SIZE = 16, 128, 64, 128, 512, 64
ROW = KV_LORA + QK_ROPE
MAX_BATCH = 65536

FLAG_CHECK_KERNEL = 0x2
FLAG_TCGEN05 = 0x4
FLAG_NO_NEW_ROW = 0x8
FLAG_EXCHANGE_SPLIT = 0x10  # peer exchange as K3 + K4 even where the fused K3 applies
FLAG_QC_HILO = 0x20  # q_c as a bf16 hi/lo pair in the score MMAs (default kernel)
FLAG_P_HILO = 0x40   # probabilities as a bf16 hi/lo pair in P c_kv, row sums unrounded (default kernel)
SHARD_STRIDE = 132
MAX_PROJECT_BATCH = 64  # MLA_MAX_PROJECT_BATCH: weight-stream projection up to here, tcgen05 GEMM beyond
STATIC_SCRATCH_BYTES = 32 << 20  # MLA_STATIC_SCRATCH_BYTES, the workspace of mla_decode_step_static
MAX_RANKS = 8              # MLA_MAX_RANKS: shards of a step with the peer exchange
IPC_HANDLE_BYTES = 64      # MLA_IPC_HANDLE_BYTES

STATUS = {
    0: "MLA_OK", -1: "MLA_E_INVALID_ARG", -2: "MLA_E_UNSUPPORTED_DIMS", -3: "MLA_E_MISALIGNED",
    -4: "MLA_E_WORKSPACE", -5: "MLA_E_ARCH", -6: "MLA_E_LAUNCH", -7: "MLA_E_DRIVER", -8: "MLA_E_LIMIT",
}
DEV_ERRORS = {0: "ok", 1: "MLA_DEV_BAD_PAGE", 2: "MLA_DEV_BAD_POSITION", 3: "MLA_DEV_TIMEOUT",
              4: "MLA_DEV_PEER_TIMEOUT"}

EXPORTED = (
    "mla_abi_version", "mla_status_string", "mla_device_error_string", "mla_params_init",
    "mla_workspace_size", "mla_decode_step", "mla_prologue", "mla_attention", "mla_merge_uv",
    "mla_plan_info", "mla_launches_per_step", "mla_combine_shards", "mla_decode_step_static", "mla_project",
    "mla_rows_init", "mla_rows_to_pages", "mla_o_proj", "mla_exchange_bytes", "mla_exchange_alloc",
    "mla_exchange_free", "mla_exchange_open", "mla_exchange_close", "mla_exchange_combine",
)


def _field_str(v) -> str:
    return str(list(v)) if isinstance(v, ctypes.Array) else str(v)


class MlaError(RuntimeError):
    """A nonzero mla_status from the C ABI, or a device error word."""

    def __init__(self, code: int, what: str, params: "MlaDecodeParams | None" = None):
        self.code = code
        msg = f"{what}: {STATUS.get(code, DEV_ERRORS.get(code, code))} ({code})"
        if params is not None:
            fields = ", ".join(f"{n}={_field_str(getattr(params, n))}" for n, _ in params._fields_)
            msg += f" [params: {fields}]"
        super().__init__(msg)


class MlaDecodeParams(ctypes.Structure):
    """Field-for-field mirror of `MlaDecodeParams` in include/mla_decode.h."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
        ("heads", ctypes.c_int32), ("qk_nope", ctypes.c_int32), ("qk_rope", ctypes.c_int32),
        ("v_head", ctypes.c_int32), ("kv_lora", ctypes.c_int32), ("page_size", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("batch", ctypes.c_int32), ("max_blocks", ctypes.c_int32), ("n_pages", ctypes.c_int32),
        ("max_pos", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_stride", ctypes.c_int64),
        ("kv_a", ctypes.c_void_p), ("kv_a_stride", ctypes.c_int64),
        ("kv_a_norm_w", ctypes.c_void_p), ("kv_b", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p), ("seq_lens", ctypes.c_void_p),
        ("kv_cache", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("out_stride", ctypes.c_int64),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
        ("error_word", ctypes.c_void_p),
        ("num_ctas", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("rope_pos", ctypes.c_void_p), ("shard_out", ctypes.c_void_p),
        ("x_n", ctypes.c_void_p), ("x_stride", ctypes.c_int64), ("w_qkv", ctypes.c_void_p),
        ("w_o", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("residual_stride", ctypes.c_int64),
        ("h_out", ctypes.c_void_p), ("h_out_stride", ctypes.c_int64),
        ("exchange", ctypes.c_void_p * MAX_RANKS), ("rank", ctypes.c_int32), ("world", ctypes.c_int32),
        ("exchange_batch", ctypes.c_int32), ("exchange_timeout_us", ctypes.c_int32),
        ("error_host", ctypes.c_void_p),
    ]


ROWS_FINAL = 0  # MLA_ROWS_FINAL: finished cache rows, copied
ROWS_RAW = 1    # MLA_ROWS_RAW: raw kv_a rows, kv_a_layernorm + RoPE applied


class MlaRowsToPages(ctypes.Structure):
    """Mirror of MlaRowsToPages (include/mla_decode.h), field for field."""
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
        ("mode", ctypes.c_int32), ("batch", ctypes.c_int32), ("total_rows", ctypes.c_int64),
        ("rows", ctypes.c_void_p), ("rows_stride", ctypes.c_int64),
        ("row_start", ctypes.c_void_p), ("first_pos", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p), ("max_blocks", ctypes.c_int32), ("n_pages", ctypes.c_int32),
        ("kv_cache", ctypes.c_void_p), ("kv_a_norm_w", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
        ("max_pos", ctypes.c_int32), ("rms_eps", ctypes.c_float),
        ("error_word", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def load_library(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libmla_decode.so (once) and declare the prototypes."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else Path(os.environ.get("MLA_DECODE_LIB", LIB_PATH))
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python fleet-mi300x_b200/build.py` "
                "(nvcc, sm_100a). There is no fallback implementation.")
        lib = ctypes.CDLL(str(p))
        P = ctypes.POINTER(MlaDecodeParams)
        lib.mla_abi_version.restype = ctypes.c_int
        lib.mla_status_string.restype = ctypes.c_char_p
        lib.mla_status_string.argtypes = [ctypes.c_int]
        lib.mla_device_error_string.restype = ctypes.c_char_p
        lib.mla_device_error_string.argtypes = [ctypes.c_int]
        lib.mla_params_init.restype = None
        lib.mla_params_init.argtypes = [P]
        lib.mla_workspace_size.restype = ctypes.c_int
        lib.mla_workspace_size.argtypes = [P, ctypes.POINTER(ctypes.c_uint64)]
        lib.mla_plan_info.restype = ctypes.c_int
        lib.mla_plan_info.argtypes = [P, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
        lib.mla_launches_per_step.restype = ctypes.c_int
        lib.mla_combine_shards.restype = ctypes.c_int
        lib.mla_combine_shards.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_void_p]
        R = ctypes.POINTER(MlaRowsToPages)
        lib.mla_rows_init.restype = None
        lib.mla_rows_init.argtypes = [R]
        lib.mla_rows_to_pages.restype = ctypes.c_int
        lib.mla_rows_to_pages.argtypes = [R, ctypes.c_void_p]
        lib.mla_exchange_bytes.restype = ctypes.c_int
        lib.mla_exchange_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64)]
        lib.mla_exchange_alloc.restype = ctypes.c_int
        lib.mla_exchange_alloc.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        lib.mla_exchange_open.restype = ctypes.c_int
        lib.mla_exchange_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        for fn in ("mla_exchange_free", "mla_exchange_close"):
            getattr(lib, fn).restype = ctypes.c_int
            getattr(lib, fn).argtypes = [ctypes.c_void_p]
        for fn in ("mla_decode_step", "mla_prologue", "mla_attention", "mla_merge_uv", "mla_decode_step_static",
                   "mla_project", "mla_o_proj", "mla_exchange_combine"):
            f = getattr(lib, fn)
            f.restype = ctypes.c_int
            f.argtypes = [P, ctypes.c_void_p]
        if lib.mla_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{p}: ABI version {lib.mla_abi_version()} != {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def check(code: int, what: str, params: "MlaDecodeParams | None" = None) -> None:
    if code != 0:
        raise MlaError(code, what, params)


def new_rows() -> MlaRowsToPages:
    r = MlaRowsToPages()
    load_library().mla_rows_init(ctypes.byref(r))
    return r


def new_params() -> MlaDecodeParams:
    p = MlaDecodeParams()
    load_library().mla_params_init(ctypes.byref(p))
    return p
