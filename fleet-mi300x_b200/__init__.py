"""B200-native (sm_100a) absorbed-MLA decode attention.

A drop-in for the attention task of the cklxx/fleet-mi300x reference's task-by-task
decode (src/host/reference_decode.py:attention_absorbed): post-RMSNorm hidden state
in, paged latent cache c_kv | k_pe appended and attended, head-concatenated bf16
output before o_proj out. The work runs in hand-written CUDA kernels behind the C
ABI of libmla_decode.so (include/mla_decode.h); this package is the host side.

The directory name is not a Python identifier; import it with
`importlib.import_module("fleet-mi300x_b200")`.
"""
from .config import ModelConfig, rope_tables, yarn_cos_sin, yarn_get_mscale
from .cache import PagedLatentCache
from .attention import LayerWeights, MlaDecodeAttention, attention_absorbed, combine_shards, device_rope_tables
from .graph import DecodeGraph, HostPipeline, HostStepGraph, LayerStackGraph
from .handoff import caches_from_flat, read_flat_cache, rows_to_pages, write_flat_cache
from .native import MlaError, load_library

__all__ = [
    "ModelConfig", "rope_tables", "yarn_cos_sin", "yarn_get_mscale", "PagedLatentCache",
    "LayerWeights", "MlaDecodeAttention", "attention_absorbed", "combine_shards", "device_rope_tables",
    "DecodeGraph", "HostPipeline", "HostStepGraph", "LayerStackGraph", "MlaError", "load_library", "caches_from_flat", "read_flat_cache", "rows_to_pages",
    "write_flat_cache",
]
