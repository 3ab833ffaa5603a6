"""Routing of selected attention layers to the TriangleMix kernel, and a vLLM hook.

The reference plugin patches vllm-ascend's attention backend so that the
layers named in the configuration run the TriangleMix operator when the
step's plan allows it, and the stock fused-infer-attention path otherwise
(package/src/vllm_ascend_trianglemix/plugin.py:1358-1535 in the reference
project), with ``strict`` turning launch errors into exceptions instead of
fallbacks (:1406-1535).  This module does the same for vLLM's CUDA
FlashAttention backend:

* ``TriangleMixRouter`` builds one plan per scheduler step (planning.py),
  checks a layer call's tensors against what the kernel supports, launches
  the kernel (batch-one or varlen), records counters (stats.py) and tells
  the caller whether the stock backend must run instead;
* ``install_vllm_flash_attention_hook`` wraps
  ``vllm.v1.attention.backends.flash_attn.FlashAttentionImpl.forward``.  In
  vLLM's v1 engine the KV cache write is a separate step, so ``forward`` only
  reads the paged cache ``[2, num_blocks, block_size, kv_heads, head_size]``,
  which is this kernel's BSND layout when ``block_size`` is 128.

Differences from the reference, both enabled by this kernel: a packed batch
of prefills is direct when every request is eligible (one varlen launch),
and a tensor-parallel shard of the heads (1, 2, 4 or 8 KV heads) is direct
for a single request (the reference sends tensor-parallel calls to its
fallback, plugin.py:1251-1253).
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable, Sequence

import torch

from . import _native
from .config import PluginConfig
from .kernel import (SUPPORTED_CACHE_BLOCK_SIZE, SUPPORTED_HEAD_SIZE, extract_layer_index)
from .planning import FallbackReason, TriangleBatchPlan, build_batch_plan
from .stats import TriangleMixRuntimeStats, runtime_stats

GROUP_SIZE = 4  # query heads per KV head (GQA 4:1)


def step_state(query_lens: Sequence[int], seq_lens: Sequence[int]) -> tuple[str, int]:
    """Attention state name and decode count of a step from its lengths.

    The names are the vllm-ascend states the reference planner accepts
    (planning.py:78-82); vLLM's CUDA metadata has no state field, so it is
    derived: a request with one query row is a decode, a request whose rows
    cover its whole sequence is a cache-miss prefill, and a request with
    earlier tokens already cached is a chunked prefill.
    """
    decodes = sum(1 for q in query_lens if q == 1)
    if query_lens and decodes == len(query_lens):
        return "DecodeOnly", decodes
    if all(q == s for q, s in zip(query_lens, seq_lens)):
        return "PrefillNoCache", decodes
    return "ChunkedPrefill", decodes


class TriangleMixRouter:
    """Per-process router: plans steps, checks layer calls, launches, counts."""

    def __init__(self, config: PluginConfig, stats: TriangleMixRuntimeStats | None = None):
        self.config = config
        self.stats = stats if stats is not None else runtime_stats()
        self.stats.configure(config.stats_recent_capacity, config.stats_log_interval)
        self._workspaces: dict[tuple[int, int], torch.Tensor] = {}
        self._lock = threading.Lock()
        self._plans: dict[int, tuple[Any, TriangleBatchPlan]] = {}

    # ------------------------------------------------------------ planning
    def selects(self, layer_name: str) -> bool:
        return self.config.enabled and self.config.kernel.uses_layer(layer_name)

    def plan_step(self, *, query_lens: Sequence[int], seq_lens: Sequence[int],
                  prompt_lens: Sequence[int] | None = None) -> TriangleBatchPlan:
        """The step's plan from host lengths (prompt_lens default to seq_lens)."""
        query_lens = [int(x) for x in query_lens]
        seq_lens = [int(x) for x in seq_lens]
        prompts = [int(x) for x in prompt_lens] if prompt_lens is not None else list(seq_lens)
        state, decodes = step_state(query_lens, seq_lens)
        ends, total = [], 0
        for q in query_lens:
            total += q
            ends.append(total)
        plan = build_batch_plan(state_name=state, cumulative_query_ends=ends, seq_lens=seq_lens,
                                prompt_lens=prompts, num_decodes=decodes,
                                num_prefills=len(query_lens) - decodes, config=self.config.kernel)
        self.stats.record_planner_decision(plan)
        return plan

    def plan_for_metadata(self, metadata: Any,
                          prompt_lens_provider: Callable[[Any], Sequence[int]] | None = None
                          ) -> TriangleBatchPlan:
        """One plan per metadata object (shared by all layers of a step).

        The lengths are read to the host once per step (``query_start_loc``
        and ``seq_lens`` of vLLM's FlashAttention metadata).  Prompt lengths
        come from ``prompt_lens_provider(metadata)``; without one, each
        request's prompt is taken to end at its sequence end.
        """
        key = id(metadata)
        with self._lock:
            hit = self._plans.get(key)
            if hit is not None and hit[0] is metadata:
                return hit[1]
        starts = [int(x) for x in metadata.query_start_loc.tolist()]
        seq_lens = [int(x) for x in metadata.seq_lens.tolist()]
        query_lens = [b - a for a, b in zip(starts, starts[1:])]
        prompts = prompt_lens_provider(metadata) if prompt_lens_provider is not None else None
        plan = self.plan_step(query_lens=query_lens, seq_lens=seq_lens, prompt_lens=prompts)
        with self._lock:
            if len(self._plans) > 64:
                self._plans.clear()
            self._plans[key] = (metadata, plan)
        return plan

    # ------------------------------------------------------------ checks
    def dispatch_reason(self, plan: TriangleBatchPlan, query: torch.Tensor,
                        key_cache: torch.Tensor, value_cache: torch.Tensor,
                        block_table: torch.Tensor, out: torch.Tensor, *, causal: bool = True,
                        unsupported_features: bool = False) -> FallbackReason:
        """Why this layer call cannot run the kernel (NONE when it can)."""
        if not plan.direct:
            return plan.primary_reason
        if not causal:
            return FallbackReason.NON_CAUSAL
        if unsupported_features:
            return FallbackReason.MODEL_UNSUPPORTED
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            return FallbackReason.GRAPH_CAPTURE
        rows = plan.cu_seqlens_q[-1]
        if (query.dtype != torch.bfloat16 or query.dim() != 3 or query.shape[0] != rows
                or query.shape[2] != SUPPORTED_HEAD_SIZE or not query.is_contiguous()
                or not query.is_cuda):
            return FallbackReason.QUERY_UNSUPPORTED
        if (out.dtype != torch.bfloat16 or out.shape != query.shape or not out.is_contiguous()):
            return FallbackReason.QUERY_UNSUPPORTED
        for cache in (key_cache, value_cache):
            if (cache.dtype != torch.bfloat16 or cache.dim() != 4
                    or cache.shape[1] != SUPPORTED_CACHE_BLOCK_SIZE
                    or cache.shape[3] != SUPPORTED_HEAD_SIZE or not cache.is_contiguous()
                    or cache.device != query.device):
                return FallbackReason.KV_CACHE_UNSUPPORTED
        if key_cache.shape != value_cache.shape:
            return FallbackReason.KV_CACHE_UNSUPPORTED
        kv_heads = key_cache.shape[2]
        if kv_heads not in (1, 2, 4, 8) or query.shape[1] != GROUP_SIZE * kv_heads:
            return FallbackReason.MODEL_UNSUPPORTED
        if plan.batch_size > 1 and kv_heads != 8:
            return FallbackReason.TENSOR_PARALLEL
        if (block_table.dtype != torch.int32 or block_table.dim() != 2
                or block_table.shape[0] < plan.batch_size or not block_table.is_contiguous()
                or block_table.device != query.device):
            return FallbackReason.BLOCK_TABLE_UNSUPPORTED
        pages_needed = max(-(-r.seq_len // SUPPORTED_CACHE_BLOCK_SIZE)
                           for r in plan.requests[:plan.batch_size])
        if block_table.shape[1] < pages_needed:
            return FallbackReason.BLOCK_TABLE_UNSUPPORTED
        return FallbackReason.NONE

    # ------------------------------------------------------------ launch
    def _workspace(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index or 0, nbytes)
        ws = self._workspaces.get(key)
        if ws is None:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._workspaces[key] = ws
        return ws

    def _launch(self, plan: TriangleBatchPlan, query, key_cache, value_cache, block_table,
                out) -> int:
        reqs = plan.requests[:plan.batch_size]
        scale = SUPPORTED_HEAD_SIZE ** -0.5
        stream = torch.cuda.current_stream(query.device).cuda_stream
        if plan.batch_size == 1:
            r = reqs[0]
            kv_heads = key_cache.shape[2]
            nbytes = _native.make_plan(r.query_len, r.q_begin, r.seq_len, r.prompt_len,
                                       kv_heads).workspace_bytes
            _native.paged_attention(query, key_cache, value_cache, block_table[:1], out,
                                    r.q_begin, r.seq_len, r.prompt_len, scale,
                                    kv_heads=kv_heads,
                                    workspace=self._workspace(query.device, nbytes),
                                    stream=stream)
            return 1
        cu = plan.cu_seqlens_q
        seqs = [r.seq_len for r in reqs]
        prompts = [r.prompt_len for r in reqs]
        nbytes = _native.varlen_workspace_size(cu, seqs, prompts)
        _native.paged_attention_varlen(query, key_cache, value_cache, block_table, out, cu, seqs,
                                       prompts, scale,
                                       workspace=self._workspace(query.device, nbytes),
                                       stream=stream)
        return -(-plan.batch_size // 16)

    def attend(self, plan: TriangleBatchPlan, layer_name: str, query: torch.Tensor,
               key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
               out: torch.Tensor, *, causal: bool = True,
               unsupported_features: bool = False) -> bool:
        """Run the kernel into ``out`` if the call qualifies; False: run the stock backend.

        With ``strict`` configured, a launch error raises instead of falling
        back (reference plugin.py:1406-1535).
        """
        layer_index = extract_layer_index(layer_name)
        reason = self.dispatch_reason(plan, query, key_cache, value_cache, block_table, out,
                                      causal=causal, unsupported_features=unsupported_features)
        if reason is not FallbackReason.NONE:
            self.stats.record_layer_fallback(plan_id=plan.plan_id, layer_index=layer_index,
                                             reason=reason)
            return False
        started = time.perf_counter_ns()
        try:
            launches = self._launch(plan, query, key_cache, value_cache, block_table, out)
        except Exception:
            self.stats.record_runtime_error(stage="direct_launch")
            if self.config.strict:
                raise
            self.stats.record_layer_fallback(plan_id=plan.plan_id, layer_index=layer_index,
                                             reason=FallbackReason.DIRECT_LAUNCH_ERROR)
            return False
        self.stats.record_layer_dispatch(plan_id=plan.plan_id, layer_index=layer_index,
                                         saved_qk=plan.saved_qk,
                                         host_enqueue_ns=time.perf_counter_ns() - started,
                                         launches=launches)
        return True


_HOOK_ATTR = "_trianglemix_original_forward"


def install_vllm_flash_attention_hook(router: TriangleMixRouter, *, impl_cls: type | None = None,
                                      prompt_lens_provider: Callable[[Any], Sequence[int]]
                                      | None = None) -> bool:
    """Wrap FlashAttentionImpl.forward so selected layers take the TriangleMix kernel.

    ``impl_cls`` defaults to vLLM's ``FlashAttentionImpl``; returns False when
    vLLM is not importable.  Installing twice replaces the router.
    """
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl as impl_cls
        except Exception:  # vLLM absent or incompatible: nothing to hook
            return False
    original = getattr(impl_cls, _HOOK_ATTR, None) or impl_cls.forward

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        name = str(getattr(layer, "layer_name", ""))
        if (attn_metadata is None or output_scale is not None or output_block_scale is not None
                or not router.selects(name)):
            return original(self, layer, query, key, value, kv_cache, attn_metadata, output,
                             output_scale, output_block_scale)
        plan = router.plan_for_metadata(attn_metadata, prompt_lens_provider)
        key_cache, value_cache = kv_cache.unbind(0)
        rows = int(getattr(attn_metadata, "num_actual_tokens", query.shape[0]))
        q = query[:rows]
        out = output[:rows].view(rows, q.shape[1], -1)
        extras = (getattr(self, "sliding_window", None) not in (None, (-1, -1))
                  or getattr(self, "alibi_slopes", None) is not None
                  or bool(getattr(self, "logits_soft_cap", 0) or 0)
                  or getattr(self, "sinks", None) is not None)
        if router.attend(plan, name, q, key_cache, value_cache, attn_metadata.block_table, out,
                         causal=bool(getattr(attn_metadata, "causal", True)),
                         unsupported_features=extras):
            return output
        return original(self, layer, query, key, value, kv_cache, attn_metadata, output,
                        output_scale, output_block_scale)

    setattr(impl_cls, _HOOK_ATTR, original)
    impl_cls.forward = forward
    return True


def uninstall_vllm_flash_attention_hook(impl_cls: type | None = None) -> bool:
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl as impl_cls
        except Exception:
            return False
    original = getattr(impl_cls, _HOOK_ATTR, None)
    if original is None:
        return False
    impl_cls.forward = original
    delattr(impl_cls, _HOOK_ATTR)
    return True
