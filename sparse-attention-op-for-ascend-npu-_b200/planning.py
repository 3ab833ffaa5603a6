"""Per-scheduler-step routing plans for TriangleMix prefill.

The reason codes, plan records and per-request eligibility rules follow the
reference planner (package/src/vllm_ascend_trianglemix/planning.py:14-207 in
the reference project); the reason values are the reference's so that
counters and logs read the same.  One difference: the reference op takes a
single request, so its planner sends every batch of more than one request
to the stock backend (``batch_unsupported``, planning.py:149-150).  Here a
packed batch runs through one varlen launch
(``tpsa_paged_attention_varlen``), so a batch is direct when every request
in it is eligible; ``BATCH_UNSUPPORTED`` is kept for API compatibility.
"""

from __future__ import annotations

import itertools
import time
from dataclasses import dataclass
from enum import Enum
from typing import Sequence

from .kernel import TriangleMixConfig, TriangleSparseSpan, triangle_sparse_span


class FallbackReason(str, Enum):
    NONE = "none"
    STATE_UNSUPPORTED = "state_unsupported"
    MIXED_DECODE = "mixed_decode"
    BATCH_UNSUPPORTED = "batch_unsupported"
    MISSING_METADATA = "missing_metadata"
    INVALID_LENGTHS = "invalid_lengths"
    NO_SPARSE_MIDDLE = "no_sparse_middle"
    BELOW_MIN_SEQ_LEN = "below_min_seq_len"
    BELOW_MIN_SPARSE_ROWS = "below_min_sparse_rows"
    BELOW_MIN_SAVED_QK = "below_min_saved_qk"
    BELOW_SPLIT_MIN_SPARSE_ROWS = "below_split_min_sparse_rows"
    BELOW_SPLIT_MIN_SAVED_QK = "below_split_min_saved_qk"
    GEOMETRY_UNSUPPORTED = "geometry_unsupported"
    ADAPTER_UNAVAILABLE = "adapter_unavailable"
    DIRECT_LAUNCH_ERROR = "direct_launch_error"
    STATIC_CAPABILITY = "static_capability"
    GRAPH_CAPTURE = "graph_capture"
    CONTEXT_PARALLEL = "context_parallel"
    TENSOR_PARALLEL = "tensor_parallel"
    NON_CAUSAL = "non_causal"
    MODEL_UNSUPPORTED = "model_unsupported"
    QUERY_UNSUPPORTED = "query_unsupported"
    KV_CACHE_UNSUPPORTED = "kv_cache_unsupported"
    BLOCK_TABLE_UNSUPPORTED = "block_table_unsupported"


@dataclass(frozen=True)
class TriangleRequestPlan:
    request_index: int
    q_begin: int
    q_end: int
    seq_len: int
    prompt_len: int
    span: TriangleSparseSpan | None
    eligible: bool
    reason: FallbackReason

    @property
    def query_len(self) -> int:
        return self.q_end - self.q_begin

    @property
    def saved_qk(self) -> int:
        return 0 if self.span is None else self.span.saved_qk


@dataclass(frozen=True)
class TriangleBatchPlan:
    """One immutable plan per scheduler step, reused by every selected layer."""

    plan_id: int
    state_name: str
    batch_size: int
    requests: tuple[TriangleRequestPlan, ...]
    direct: bool
    routing_ns: int

    @property
    def primary_reason(self) -> FallbackReason:
        for request in self.requests:
            if request.reason is not FallbackReason.NONE:
                return request.reason
        return FallbackReason.NONE

    @property
    def cu_seqlens_q(self) -> list[int]:
        """Packed query offsets of the batch (host), for the varlen launch."""
        out = [0]
        for request in self.requests[:self.batch_size]:
            out.append(out[-1] + request.query_len)
        return out

    @property
    def saved_qk(self) -> int:
        return sum(r.saved_qk for r in self.requests[:self.batch_size])


_PLAN_IDS = itertools.count(1)
PREFILL_STATES = frozenset({"PrefillNoCache", "PrefillCacheHit", "ChunkedPrefill"})


def request_reason(*, query_len: int, seq_len: int, prompt_len: int,
                   config: TriangleMixConfig) -> tuple[TriangleSparseSpan | None, FallbackReason]:
    """Eligibility of one request, checked in the reference's order (planning.py:88-117)."""
    if query_len <= 0 or seq_len < query_len or prompt_len < seq_len:
        return None, FallbackReason.INVALID_LENGTHS
    span = triangle_sparse_span(query_len=query_len, seq_len=seq_len, prompt_len=prompt_len,
                                config=config)
    if not config.has_supported_geometry:
        return span, FallbackReason.GEOMETRY_UNSUPPORTED
    if not span.has_sparse_middle:
        return span, FallbackReason.NO_SPARSE_MIDDLE
    if seq_len < config.direct_min_seq_len:
        return span, FallbackReason.BELOW_MIN_SEQ_LEN
    if span.sparse_rows < config.direct_min_sparse_rows:
        return span, FallbackReason.BELOW_MIN_SPARSE_ROWS
    if span.saved_qk < config.direct_min_saved_qk:
        return span, FallbackReason.BELOW_MIN_SAVED_QK
    if span.is_split:
        if span.sparse_rows < config.direct_split_min_sparse_rows:
            return span, FallbackReason.BELOW_SPLIT_MIN_SPARSE_ROWS
        if span.saved_qk < config.direct_split_min_saved_qk:
            return span, FallbackReason.BELOW_SPLIT_MIN_SAVED_QK
    return span, FallbackReason.NONE


def build_batch_plan(*, state_name: str, cumulative_query_ends: Sequence[int] | None,
                     seq_lens: Sequence[int] | None, prompt_lens: Sequence[int] | None,
                     num_decodes: int, num_prefills: int,
                     config: TriangleMixConfig) -> TriangleBatchPlan:
    """Build the step's plan: a batch-wide reason first, then each request's."""
    started = time.perf_counter_ns()
    ends = tuple(int(x) for x in (cumulative_query_ends or ()))
    seqs = tuple(int(x) for x in (seq_lens or ()))
    prompts = tuple(int(x) for x in (prompt_lens or ()))
    batch = len(seqs)
    if state_name not in PREFILL_STATES:
        batch_reason = FallbackReason.STATE_UNSUPPORTED
    elif num_decodes:
        batch_reason = FallbackReason.MIXED_DECODE
    elif not ends or not seqs or not prompts or len(ends) != batch or len(prompts) != batch \
            or num_prefills != batch:
        batch_reason = FallbackReason.MISSING_METADATA
    else:
        batch_reason = FallbackReason.NONE
    requests: list[TriangleRequestPlan] = []
    prev = 0
    for i in range(batch):
        end = ends[i] if i < len(ends) else prev
        qlen = end - prev
        prompt = prompts[i] if i < len(prompts) else seqs[i]
        span, own = request_reason(query_len=qlen, seq_len=seqs[i], prompt_len=prompt,
                                   config=config)
        reason = batch_reason if batch_reason is not FallbackReason.NONE else own
        requests.append(TriangleRequestPlan(i, seqs[i] - qlen, seqs[i], seqs[i], prompt, span,
                                            reason is FallbackReason.NONE, reason))
        prev = end
    if not requests:
        # A placeholder keeps the reason when every piece of metadata is absent.
        reason = batch_reason if batch_reason is not FallbackReason.NONE \
            else FallbackReason.MISSING_METADATA
        requests.append(TriangleRequestPlan(0, 0, 0, 0, 0, None, False, reason))
    direct = batch > 0 and all(r.eligible for r in requests)
    return TriangleBatchPlan(plan_id=next(_PLAN_IDS), state_name=state_name, batch_size=batch,
                             requests=tuple(requests), direct=direct,
                             routing_ns=time.perf_counter_ns() - started)
