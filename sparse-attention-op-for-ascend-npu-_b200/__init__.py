"""B200-native TriangleMix paged sparse prefill attention.

Import name: ``trianglemix_b200`` (the directory name is not a valid Python
identifier; ``load_package()`` in ``__graft_entry__.py`` registers it).

Layers, bottom up:
  csrc/tpsa_kernel.cu   sm_100a kernel + C ABI (include/tpsa.h) -> libtpsa.so
  csrc/torch_adapter.cpp torch ops trianglemix::triangle_paged_sparse_attention.out,
                         trianglemix_reference::triangle_paged_sparse_attention[_workspace_size]
                         -> _tpsa_torch.so
  _native.py            ctypes binding of the C ABI
  kernel.py             reference-compatible direct-path API
  sharding.py           KV-head partition across 1/2/4/8 GPUs
  config.py, planning.py, stats.py, plugin.py
                        serving integration: configuration, per-step plans,
                        counters, and the router / vLLM FlashAttention hook
"""

from . import _native, config, planning, plugin, sharding, stats
from ._native import TpsaError, load_adapter
from .kernel import (
    TriangleMixConfig,
    TriangleSparseSpan,
    estimate_tile_counts,
    extract_layer_index,
    load_triangle_mix_adapter,
    load_triangle_mix_adapter_if_enabled,
    parse_layer_indices,
    triangle_direct_eligible,
    triangle_direct_paged_attention,
    triangle_mix_adapter_loaded,
    triangle_saved_qk,
    triangle_sparse_query_rows,
    triangle_sparse_span,
    triangle_streaming_start,
)

__all__ = [
    "TpsaError",
    "TriangleMixConfig",
    "TriangleSparseSpan",
    "estimate_tile_counts",
    "extract_layer_index",
    "load_adapter",
    "load_triangle_mix_adapter",
    "load_triangle_mix_adapter_if_enabled",
    "parse_layer_indices",
    "triangle_direct_eligible",
    "triangle_direct_paged_attention",
    "triangle_mix_adapter_loaded",
    "triangle_saved_qk",
    "triangle_sparse_query_rows",
    "triangle_sparse_span",
    "triangle_streaming_start",
    "_native",
    "config",
    "planning",
    "plugin",
    "sharding",
    "stats",
]
