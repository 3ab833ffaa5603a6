"""Direct-path Python API for single-launch TriangleMix paged prefill on B200.

Same names, argument meanings and error behaviour as the reference's direct
path (package/src/vllm_ascend_trianglemix/kernel.py in the reference
project; line citations below are into that file).  The launch goes to the
CUDA operator ``torch.ops.trianglemix.triangle_paged_sparse_attention.out``
registered by ``_tpsa_torch.so`` (which calls libtpsa.so's C ABI); there is
no CPU or eager fallback in this module.
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass

import torch

from . import _native

SUPPORTED_HEAD_SIZE = 128
SUPPORTED_CACHE_BLOCK_SIZE = 128
SUPPORTED_QUERY_HEADS = 32
SUPPORTED_KV_HEADS = 8
SUPPORTED_SINK_TOKENS = 8
SUPPORTED_LOCAL_WINDOW = 512
SUPPORTED_LAST_ROWS = 128


@dataclass(frozen=True)
class TriangleMixConfig:
    """Runtime configuration (reference kernel.py:54-105).

    The crossover thresholds keep the reference defaults (calibrated on
    Ascend 910B3); ``harness``-style B200 sweeps may override them.
    """

    enabled: bool
    layer_indices: frozenset[int]
    sink_tokens: int = SUPPORTED_SINK_TOKENS
    local_window: int = SUPPORTED_LOCAL_WINDOW
    last_rows: int = SUPPORTED_LAST_ROWS
    direct_min_seq_len: int = 0
    direct_min_sparse_rows: int = 128
    direct_min_saved_qk: int = 913_152
    direct_split_min_sparse_rows: int = 192
    direct_split_min_saved_qk: int = 1_299_264

    def __post_init__(self) -> None:
        if self.sink_tokens <= 0:
            raise ValueError("TriangleMix sink_tokens must be positive")
        if self.local_window < 0:
            raise ValueError("TriangleMix local_window must be non-negative")
        if self.last_rows <= 0:
            raise ValueError("TriangleMix last_rows must be positive")
        for name in ("direct_min_seq_len", "direct_min_sparse_rows", "direct_min_saved_qk",
                     "direct_split_min_sparse_rows", "direct_split_min_saved_qk"):
            if getattr(self, name) < 0:
                raise ValueError(f"TriangleMix {name} must be non-negative")

    @property
    def has_supported_geometry(self) -> bool:
        return (self.sink_tokens == SUPPORTED_SINK_TOKENS
                and self.local_window == SUPPORTED_LOCAL_WINDOW
                and self.last_rows == SUPPORTED_LAST_ROWS)

    def uses_layer(self, layer_name: str) -> bool:
        index = extract_layer_index(layer_name)
        return index is not None and index in self.layer_indices


@dataclass(frozen=True)
class TriangleSparseSpan:
    """Absolute-coordinate plan of one prefill call (reference kernel.py:108-142).

    Rows ``[q0, q1)`` are the query chunk; ``[s0, s1)`` its sparse rows.
    """

    q0: int
    q1: int
    s0: int
    s1: int

    @property
    def query_rows(self) -> int:
        return self.q1 - self.q0

    @property
    def sparse_rows(self) -> int:
        return max(0, self.s1 - self.s0)

    @property
    def has_sparse_middle(self) -> bool:
        return self.s0 < self.s1

    @property
    def has_dense_prefix(self) -> bool:
        return self.has_sparse_middle and self.q0 < self.s0

    @property
    def has_dense_tail(self) -> bool:
        return self.has_sparse_middle and self.s1 < self.q1

    @property
    def is_split(self) -> bool:
        return self.has_dense_prefix or self.has_dense_tail

    @property
    def saved_qk(self) -> int:
        return triangle_saved_qk(self.s0, self.s1)


_LAYER_RE = re.compile(r"(?:^|\.)layers\.(\d+)(?:\.|$)")


def extract_layer_index(layer_name: str) -> int | None:
    """``model.layers.17.self_attn.attn`` -> 17 (reference kernel.py:145-151)."""
    match = _LAYER_RE.search(layer_name)
    return int(match.group(1)) if match else None


def parse_layer_indices(value: str) -> frozenset[int]:
    """Parse ``"5,7,10,15-35"`` (reference kernel.py:154-177)."""
    out: set[int] = set()
    for item in (part.strip() for part in value.split(",")):
        if not item:
            continue
        if "-" in item:
            lo_text, hi_text = item.split("-", 1)
            lo, hi = int(lo_text), int(hi_text)
            if lo < 0 or hi < lo:
                raise ValueError(f"Invalid TriangleMix layer range: {item!r}")
            out.update(range(lo, hi + 1))
        else:
            idx = int(item)
            if idx < 0:
                raise ValueError(f"Invalid TriangleMix layer index: {item!r}")
            out.add(idx)
    return frozenset(out)


def triangle_streaming_start(config: TriangleMixConfig) -> int:
    """First row that can skip keys: sink + window + 1 (521)."""
    return config.sink_tokens + config.local_window + 1


def triangle_sparse_span(*, query_len: int, seq_len: int, prompt_len: int,
                         config: TriangleMixConfig) -> TriangleSparseSpan:
    """Sparse interval ``[s0, s1)`` of a chunk (reference kernel.py:185-208)."""
    if query_len < 0:
        raise ValueError("TriangleMix query_len must be non-negative")
    if seq_len < query_len:
        raise ValueError("TriangleMix seq_len must be at least query_len")
    if prompt_len < seq_len:
        raise ValueError("TriangleMix prompt_len must be at least seq_len")
    q0, q1 = seq_len - query_len, seq_len
    s0 = max(q0, triangle_streaming_start(config))
    s1 = min(q1, max(0, prompt_len - config.last_rows))
    return TriangleSparseSpan(q0=q0, q1=q1, s0=s0, s1=s1)


def triangle_sparse_query_rows(*, query_len: int, seq_len: int, prompt_len: int,
                               config: TriangleMixConfig) -> int:
    return triangle_sparse_span(query_len=query_len, seq_len=seq_len, prompt_len=prompt_len,
                                config=config).sparse_rows


def triangle_saved_qk(sparse_start: int, sparse_end: int) -> int:
    """Causal QK pairs skipped by rows ``[sparse_start, sparse_end)``.

    Row q skips q - 520 keys, so the sum is an arithmetic series
    (reference kernel.py:227-237).
    """
    if sparse_end <= sparse_start:
        return 0
    rows = sparse_end - sparse_start
    return rows * (sparse_start + sparse_end - 1041) // 2


def triangle_direct_eligible(*, query_len: int, seq_len: int, prompt_len: int,
                             config: TriangleMixConfig) -> bool:
    """Performance / geometry gates (reference kernel.py:240-269)."""
    if not config.has_supported_geometry:
        return False
    span = triangle_sparse_span(query_len=query_len, seq_len=seq_len, prompt_len=prompt_len,
                                config=config)
    if not span.has_sparse_middle:
        return False
    if seq_len < config.direct_min_seq_len:
        return False
    if span.sparse_rows < config.direct_min_sparse_rows:
        return False
    if span.saved_qk < config.direct_min_saved_qk:
        return False
    if span.is_split and (span.sparse_rows < config.direct_split_min_sparse_rows
                          or span.saved_qk < config.direct_split_min_saved_qk):
        return False
    return True


def load_triangle_mix_adapter(path=None) -> str:
    """Load the torch adapter once per process; default is the in-tree build.

    Reusing the same path is idempotent; a different second path is refused
    (reference kernel.py:296-322).
    """
    if path is not None and not str(path).strip():
        raise ValueError("TriangleMix adapter path is empty")
    return _native.load_adapter(path)


def load_triangle_mix_adapter_if_enabled(enabled: bool, path=None) -> bool:
    if not enabled:
        return False
    load_triangle_mix_adapter(path)
    return True


def triangle_mix_adapter_loaded() -> bool:
    return _native.adapter_loaded()


def _validate_direct_tensors(*, query: torch.Tensor, key_cache: torch.Tensor,
                             value_cache: torch.Tensor, block_table: torch.Tensor,
                             output: torch.Tensor, seq_len: int) -> None:
    """Pre-launch checks with the reference's ValueError contract (kernel.py:342-416)."""
    if query.ndim != 3 or tuple(query.shape[1:]) != (SUPPORTED_QUERY_HEADS, SUPPORTED_HEAD_SIZE):
        raise ValueError("TriangleMix query must be [Tq, 32, 128]")
    if query.dtype != torch.bfloat16:
        raise ValueError("TriangleMix query must be BF16")
    if output.shape != query.shape or output.dtype != query.dtype:
        raise ValueError("TriangleMix output must match query shape and dtype")
    tail = (SUPPORTED_CACHE_BLOCK_SIZE, SUPPORTED_KV_HEADS, SUPPORTED_HEAD_SIZE)
    if key_cache.ndim != 4 or tuple(key_cache.shape[1:]) != tail or value_cache.shape != key_cache.shape:
        raise ValueError("TriangleMix KV caches must be [pages, 128, 8, 128]")
    if key_cache.dtype != query.dtype or value_cache.dtype != query.dtype:
        raise ValueError("TriangleMix query and KV cache dtypes must match")
    if block_table.ndim != 2 or block_table.shape[0] != 1 or block_table.dtype != torch.int32:
        raise ValueError("TriangleMix block table must be INT32 [1, max_pages]")
    if any(not t.is_contiguous() for t in (query, key_cache, value_cache, block_table, output)):
        raise ValueError("TriangleMix tensors must be contiguous")
    if any(t.device != query.device for t in (key_cache, value_cache, block_table, output)):
        raise ValueError("TriangleMix tensors must share one device")
    if block_table.shape[1] < math.ceil(seq_len / SUPPORTED_CACHE_BLOCK_SIZE):
        raise ValueError("TriangleMix block table is too short for seq_len")


def _run_triangle_single_launch_out(*, query, key_cache, value_cache, block_table, query_start: int,
                                    seq_len: int, prompt_len: int, softmax_scale: float,
                                    output) -> None:
    torch.ops.trianglemix.triangle_paged_sparse_attention.out(
        query, key_cache, value_cache, block_table, query_start, seq_len, prompt_len,
        softmax_scale, out=output)


def triangle_direct_paged_attention(*, query: torch.Tensor, key_cache: torch.Tensor,
                                    value_cache: torch.Tensor, block_table: torch.Tensor,
                                    seq_len: int, prompt_len: int, output: torch.Tensor,
                                    softmax_scale: float, config: TriangleMixConfig) -> torch.Tensor:
    """Dense prefix, sparse middle and dense tail in one launch (reference kernel.py:445-489)."""
    span = triangle_sparse_span(query_len=query.shape[0], seq_len=seq_len, prompt_len=prompt_len,
                                config=config)
    if not config.has_supported_geometry:
        raise ValueError("TriangleMix operator geometry does not match config")
    if not span.has_sparse_middle:
        raise ValueError("TriangleMix direct path requires a non-empty sparse middle")
    _validate_direct_tensors(query=query, key_cache=key_cache, value_cache=value_cache,
                             block_table=block_table, output=output, seq_len=seq_len)
    _run_triangle_single_launch_out(query=query, key_cache=key_cache, value_cache=value_cache,
                                    block_table=block_table, query_start=span.q0, seq_len=span.q1,
                                    prompt_len=prompt_len, softmax_scale=softmax_scale, output=output)
    return output


def estimate_tile_counts(seq_len: int, config: TriangleMixConfig) -> tuple[int, int]:
    """``(triangle, dense)`` key-tile counts of one KV head for a full prompt of
    ``seq_len`` tokens run as one chunk, in this kernel's tiling.

    The reference's helper (kernel.py:492-522) counts its own 32-row x
    512-key tiles; here ``triangle`` is the plan this library launches
    (``tpsa_make_plan``: 64-token blocks, 128- and 64-key tiles, the sink and
    band edge of a sparse block in one composite tile) and ``dense`` the tiles
    the same blocks would run over their whole causal prefix.
    """
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    if (config.sink_tokens, config.local_window, config.last_rows) != (8, 512, 128):
        raise ValueError("the kernel's geometry is sink 8, window 512, dense tail 128")
    if seq_len == 0:
        return 0, 0
    triangle = _native.make_plan(seq_len, 0, seq_len, seq_len, 1, 148).total_tiles
    dense = 0
    for q_lo in range(0, seq_len, 64):
        keys = -(-min(seq_len, q_lo + 64) // 64) * 64
        dense += -(-keys // 128)
    return triangle, dense
