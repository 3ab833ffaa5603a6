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
  which is this kernel's BSND layout when ``block_size`` is 128;
  ``install_vllm_triton_attention_hook`` does the same for vLLM's Triton
  backend, whose cache ``[num_blocks, 2, block_size, kv_heads, head_size]``
  the kernel reads in place as interleaved K and V pages;
* ``install_vllm_metadata_patch`` puts each step's host lengths and the
  scheduler's final prompt lengths on the backend's metadata (the
  reference attaches the runner's prompt lengths the same way,
  plugin.py:523-570, 946); ``install_vllm_v2_runner_patch`` publishes the
  prompt lengths from vLLM's V2 model runner (the default for Qwen3 in vLLM
  0.22);
* ``register`` is the ``vllm.general_plugins`` entry point (pyproject.toml;
  reference setup.py:292-294, plugin.py:1705-1741): it installs both, with
  the configuration read from ``additional_config.trianglemix`` when vLLM
  builds its first attention layer.

Differences from the reference, both enabled by this kernel: a packed batch
of prefills is direct when every request is eligible (one varlen launch),
and a tensor-parallel shard of the heads (1, 2, 4 or 8 KV heads) is direct
for a single request (the reference sends tensor-parallel calls to its
fallback, plugin.py:1251-1253).
"""

from __future__ import annotations

import contextvars
import logging
import os
import threading
import time
from typing import Any, Callable, Sequence

import torch

from . import _native
from .config import PluginConfig, coerce_bool, resolve_plugin_config
from .kernel import (SUPPORTED_CACHE_BLOCK_SIZE, SUPPORTED_HEAD_SIZE, extract_layer_index)
from .planning import FallbackReason, TriangleBatchPlan, build_batch_plan
from .stats import TriangleMixRuntimeStats, runtime_stats

GROUP_SIZE = 4  # query heads per KV head (GQA 4:1)
logger = logging.getLogger(__name__)


class _NvtxRange:
    """An NVTX range on the host timeline (``trianglemix.plan``,
    ``trianglemix.attend``), so a profiler shows where the router spends
    host time; a no-op where NVTX is unavailable."""

    __slots__ = ("name", "pushed")

    def __init__(self, name: str):
        self.name, self.pushed = name, False

    def __enter__(self):
        try:
            torch.cuda.nvtx.range_push(self.name)
            self.pushed = True
        except Exception:
            pass
        return self

    def __exit__(self, *exc):
        if self.pushed:
            try:
                torch.cuda.nvtx.range_pop()
            except Exception:
                pass
        return False

# Attributes this module puts on vLLM's FlashAttention metadata (host lists).
QUERY_START_ATTR = "trianglemix_query_start_loc"
SEQ_LENS_ATTR = "trianglemix_seq_lens"
PROMPT_LENS_ATTR = "trianglemix_prompt_lens"


def _int_list(value: Any) -> list[int] | None:
    """A host integer sequence as a list, or None (device tensors are not read)."""
    if value is None:
        return None
    if isinstance(value, torch.Tensor):
        if value.device.type != "cpu":
            return None
        value = value.tolist()
    try:
        out = [int(x) for x in value]
    except (TypeError, ValueError):
        return None
    return out or None


def metadata_prompt_lens(metadata: Any) -> tuple[list[int] | None, str]:
    """The scheduler's final prompt length of each request of a step, and where
    it came from; ``(None, "missing")`` when the metadata carries none.

    Same order of sources as the reference (plugin.py:523-570): fields of the
    metadata itself, then the lengths this module attached from the model
    runner's input batch.
    """
    for name in ("prompt_lens_list", "prompt_lens_cpu", "num_prompt_tokens_cpu"):
        value = _int_list(getattr(metadata, name, None))
        if value:
            return value, f"metadata:{name}"
    value = _int_list(getattr(metadata, PROMPT_LENS_ATTR, None))
    if value:
        return value, "runner"
    return None, "missing"


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
        self._workspaces: dict[int, torch.Tensor] = {}  # one buffer per device
        self._lock = threading.Lock()
        self._plans: dict[int, tuple[Any, TriangleBatchPlan]] = {}

    # ------------------------------------------------------------ planning
    def selects(self, layer_name: str) -> bool:
        return self.config.enabled and self.config.kernel.uses_layer(layer_name)

    def plan_step(self, *, query_lens: Sequence[int], seq_lens: Sequence[int],
                  prompt_lens: Sequence[int] | None = None) -> TriangleBatchPlan:
        """The step's plan from host lengths, for a caller that knows each
        request's whole prompt (prompt_lens default to seq_lens)."""
        return self._plan([int(x) for x in query_lens], [int(x) for x in seq_lens],
                          prompt_lens if prompt_lens is not None else seq_lens)

    def _plan(self, query_lens: list[int], seq_lens: list[int],
              prompt_lens: Sequence[int] | None) -> TriangleBatchPlan:
        """The step's plan (prompt_lens None: missing, the step falls back)."""
        state, decodes = step_state(query_lens, seq_lens)
        ends, total = [], 0
        for q in query_lens:
            total += q
            ends.append(total)
        prompts = [int(x) for x in prompt_lens] if prompt_lens is not None else None
        plan = build_batch_plan(state_name=state, cumulative_query_ends=ends, seq_lens=seq_lens,
                                prompt_lens=prompts, num_decodes=decodes,
                                num_prefills=len(query_lens) - decodes, config=self.config.kernel)
        self.stats.record_planner_decision(plan)
        return plan

    def plan_for_metadata(self, metadata: Any,
                          prompt_lens_provider: Callable[[Any], Sequence[int]] | None = None
                          ) -> TriangleBatchPlan:
        """One plan per metadata object (shared by all layers of a step).

        Lengths come from the host lists ``install_vllm_metadata_patch`` puts
        on the metadata; without them ``query_start_loc`` and ``seq_lens`` are
        read from the device once per step.  Prompt lengths come from the
        metadata (``metadata_prompt_lens``), else from
        ``prompt_lens_provider(metadata)``.  With no prompt length the step
        falls back with ``missing_metadata``, as the reference does
        (plugin.py:523-570): a chunk's sparse range depends on where the
        prompt ends, which the sequence end does not tell.
        """
        key = id(metadata)
        with self._lock:
            hit = self._plans.get(key)
            if hit is not None and hit[0] is metadata:
                return hit[1]
        starts = _int_list(getattr(metadata, QUERY_START_ATTR, None))
        if starts is None:
            starts = [int(x) for x in metadata.query_start_loc.tolist()]
        seq_lens = _int_list(getattr(metadata, SEQ_LENS_ATTR, None))
        if seq_lens is None:
            seq_lens = [int(x) for x in metadata.seq_lens.tolist()]
        query_lens = [b - a for a, b in zip(starts, starts[1:])]
        prompts, _ = metadata_prompt_lens(metadata)
        if prompts is None and prompt_lens_provider is not None:
            prompts = _int_list(prompt_lens_provider(metadata))
        with _NvtxRange("trianglemix.plan"):
            plan = self._plan(query_lens, seq_lens, prompts)
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
        """The device's one workspace, grown (never shrunk) to the largest
        size a step has needed, so the router holds one buffer per device."""
        key = device.index or 0
        ws = self._workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._workspaces[key] = ws
        return ws

    def _launch(self, plan: TriangleBatchPlan, query, key_cache, value_cache, block_table,
                out, value_offset_pages: int = 0) -> int:
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
                                    stream=stream, value_offset_pages=value_offset_pages)
            return 1
        cu = plan.cu_seqlens_q
        seqs = [r.seq_len for r in reqs]
        prompts = [r.prompt_len for r in reqs]
        nbytes = _native.varlen_workspace_size(cu, seqs, prompts)
        _native.paged_attention_varlen(query, key_cache, value_cache, block_table, out, cu, seqs,
                                       prompts, scale,
                                       workspace=self._workspace(query.device, nbytes),
                                       stream=stream, value_offset_pages=value_offset_pages)
        return -(-plan.batch_size // 16)

    def attend(self, plan: TriangleBatchPlan, layer_name: str, query: torch.Tensor,
               key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
               out: torch.Tensor, *, causal: bool = True,
               unsupported_features: bool = False, value_offset_pages: int = 0) -> bool:
        """Run the kernel into ``out`` if the call qualifies; False: run the stock backend.

        With ``strict`` configured, a launch error raises instead of falling
        back (reference plugin.py:1406-1535).  ``value_offset_pages`` = 1 with
        one interleaved page view as both caches reads vLLM's
        ``[num_blocks, 2, ...]`` cache (``_native._value_ptr``).
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
            with _NvtxRange("trianglemix.attend"):
                launches = self._launch(plan, query, key_cache, value_cache, block_table, out,
                                        value_offset_pages)
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
# The doubled block table of an interleaved-cache step, kept on its metadata.
INTERLEAVED_TABLE_ATTR = "trianglemix_interleaved_block_table"


def interleaved_pages(kv_cache: torch.Tensor) -> torch.Tensor | None:
    """vLLM's ``[num_blocks, 2, block_size, kv_heads, head_size]`` cache (the
    Triton backend's) as ``2 * num_blocks`` pages: block b's K page is page
    2b and its V page 2b + 1.  None when the cache has another shape or is
    not contiguous."""
    if kv_cache.dim() != 5 or kv_cache.shape[1] != 2 or not kv_cache.is_contiguous():
        return None
    return kv_cache.view(kv_cache.shape[0] * 2, *kv_cache.shape[2:])


def interleaved_block_table(metadata: Any) -> torch.Tensor:
    """The step's block table with every entry doubled (block b -> K page 2b),
    computed once per metadata object and shared by the step's layers.  The
    cached copy is kept with the table it was made from, so a metadata copy
    that carries another block table (vLLM's ``update_block_table``) gets its
    own."""
    source = metadata.block_table
    cached = getattr(metadata, INTERLEAVED_TABLE_ATTR, None)
    if cached is None or cached[0] is not source:
        cached = (source, source * 2)
        setattr(metadata, INTERLEAVED_TABLE_ATTR, cached)
    return cached[1]


def _wrap_forward(router: TriangleMixRouter, original: Callable, interleaved: bool,
                  prompt_lens_provider: Callable[[Any], Sequence[int]] | None) -> Callable:
    """A backend ``forward`` that runs selected layers through ``router`` and
    everything else (and every call the kernel cannot take) through
    ``original``.  ``interleaved``: the cache is ``[num_blocks, 2, ...]``
    (vLLM's Triton backend), else ``[2, num_blocks, ...]`` (FlashAttention)."""

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        name = str(getattr(layer, "layer_name", ""))
        if (attn_metadata is None or output_scale is not None or output_block_scale is not None
                or not router.selects(name)):
            return original(self, layer, query, key, value, kv_cache, attn_metadata, output,
                            output_scale, output_block_scale)
        plan = router.plan_for_metadata(attn_metadata, prompt_lens_provider)
        reason = None
        if (int(getattr(self, "dcp_world_size", 1) or 1) > 1
                or int(getattr(self, "pcp_world_size", 1) or 1) > 1):
            # Context parallelism shards the KV cache across ranks, so this
            # rank's cache holds part of each sequence (reference
            # plugin.py:1254-1256 falls back the same way).
            reason = FallbackReason.CONTEXT_PARALLEL
        elif interleaved:
            pages = interleaved_pages(kv_cache)
            if pages is None:
                reason = FallbackReason.KV_CACHE_UNSUPPORTED
            else:
                key_cache = value_cache = pages
                table, offset = interleaved_block_table(attn_metadata), 1
        else:
            key_cache, value_cache = kv_cache.unbind(0)
            table, offset = attn_metadata.block_table, 0
        if reason is not None:
            router.stats.record_layer_fallback(plan_id=plan.plan_id,
                                               layer_index=extract_layer_index(name),
                                               reason=reason)
            return original(self, layer, query, key, value, kv_cache, attn_metadata, output,
                            output_scale, output_block_scale)
        rows = int(getattr(attn_metadata, "num_actual_tokens", query.shape[0]))
        q = query[:rows]
        out = output[:rows].view(rows, q.shape[1], -1)
        extras = (getattr(self, "sliding_window", None) not in (None, (-1, -1))
                  or getattr(self, "alibi_slopes", None) is not None
                  or bool(getattr(self, "logits_soft_cap", 0) or 0)
                  or getattr(self, "sinks", None) is not None)
        if router.attend(plan, name, q, key_cache, value_cache, table, out,
                         causal=bool(getattr(attn_metadata, "causal", True)),
                         unsupported_features=extras, value_offset_pages=offset):
            return output
        return original(self, layer, query, key, value, kv_cache, attn_metadata, output,
                        output_scale, output_block_scale)

    return forward


def _install_hook(router, impl_cls, interleaved, prompt_lens_provider) -> bool:
    original = getattr(impl_cls, _HOOK_ATTR, None) or impl_cls.forward
    setattr(impl_cls, _HOOK_ATTR, original)
    impl_cls.forward = _wrap_forward(router, original, interleaved, prompt_lens_provider)
    return True


def _uninstall_hook(impl_cls) -> bool:
    original = getattr(impl_cls, _HOOK_ATTR, None)
    if original is None:
        return False
    impl_cls.forward = original
    delattr(impl_cls, _HOOK_ATTR)
    return True


def install_vllm_flash_attention_hook(router: TriangleMixRouter, *, impl_cls: type | None = None,
                                      prompt_lens_provider: Callable[[Any], Sequence[int]]
                                      | None = None) -> bool:
    """Wrap FlashAttentionImpl.forward so selected layers take the TriangleMix kernel.

    ``impl_cls`` defaults to vLLM's ``FlashAttentionImpl`` (cache
    ``[2, num_blocks, block_size, kv_heads, head_size]``); returns False when
    vLLM is not importable.  Installing twice replaces the router.
    """
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl as impl_cls
        except Exception:  # vLLM absent or incompatible: nothing to hook
            return False
    return _install_hook(router, impl_cls, False, prompt_lens_provider)


def uninstall_vllm_flash_attention_hook(impl_cls: type | None = None) -> bool:
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl as impl_cls
        except Exception:
            return False
    return _uninstall_hook(impl_cls)


def install_vllm_triton_attention_hook(router: TriangleMixRouter, *, impl_cls: type | None = None,
                                       prompt_lens_provider: Callable[[Any], Sequence[int]]
                                       | None = None) -> bool:
    """Wrap TritonAttentionImpl.forward (vLLM's Triton backend) the same way.

    Its cache is ``[num_blocks, 2, block_size, kv_heads, head_size]``: a
    block's K and V pages are adjacent.  The kernel reads it in place as
    ``2 * num_blocks`` pages with the block table doubled and V one page past
    K (``interleaved_pages``, ``_native._value_ptr``).  Returns False when
    vLLM is not importable.
    """
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl as impl_cls
        except Exception:
            return False
    return _install_hook(router, impl_cls, True, prompt_lens_provider)


def uninstall_vllm_triton_attention_hook(impl_cls: type | None = None) -> bool:
    if impl_cls is None:
        try:
            from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl as impl_cls
        except Exception:
            return False
    return _uninstall_hook(impl_cls)


# ------------------------------------------------------------ step metadata
# The model runner's prompt lengths of the step being built (set around
# GPUModelRunner._build_attention_metadata, read by the metadata builder).
_STEP_PROMPTS: contextvars.ContextVar[tuple[int, ...] | None] = contextvars.ContextVar(
    "trianglemix_step_prompts", default=None)
_META_ATTR = "_trianglemix_original_build"
_RUNNER_ATTR = "_trianglemix_original_build_attention_metadata"


def install_vllm_metadata_patch(*, builder_cls: type | None = None,
                                runner_cls: type | None = None) -> bool:
    """Put host lengths and final prompt lengths on each step's attention metadata.

    ``runner_cls._build_attention_metadata`` (vLLM's GPUModelRunner) is
    wrapped to publish ``input_batch.num_prompt_tokens`` of the step's
    requests, the scheduler's final prompt lengths, while it builds the
    step's metadata; ``builder_cls.build`` (FlashAttentionMetadataBuilder) is
    wrapped to copy them, with the host copies of ``query_start_loc`` and
    ``seq_lens`` that the common metadata already holds, onto the metadata it
    returns.  The hook then plans a step without reading the device.  Returns
    False when vLLM is not importable.
    """
    if builder_cls is None or runner_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionMetadataBuilder
            from vllm.v1.worker.gpu_model_runner import GPUModelRunner
        except Exception:
            return False
        builder_cls = builder_cls or FlashAttentionMetadataBuilder
        runner_cls = runner_cls or GPUModelRunner
    build = getattr(builder_cls, _META_ATTR, None) or builder_cls.build
    prepare = getattr(runner_cls, _RUNNER_ATTR, None) or runner_cls._build_attention_metadata

    def build_with_lengths(self, common_prefix_len, common_attn_metadata, *args, **kwargs):
        meta = build(self, common_prefix_len, common_attn_metadata, *args, **kwargs)
        try:
            n = int(common_attn_metadata.num_reqs)
            starts = common_attn_metadata.query_start_loc_cpu[:n + 1].tolist()
            setattr(meta, QUERY_START_ATTR, starts)
            seqs = getattr(common_attn_metadata, "_seq_lens_cpu", None)
            if isinstance(seqs, torch.Tensor) and seqs.device.type == "cpu":
                setattr(meta, SEQ_LENS_ATTR, seqs[:n].tolist())
            prompts = _STEP_PROMPTS.get()
            if prompts is not None and len(prompts) >= n:
                setattr(meta, PROMPT_LENS_ATTR, list(prompts[:n]))
        except Exception:  # metadata of another shape: plan from the device instead
            runtime_stats().record_runtime_error(stage="metadata_lengths")
        return meta

    def build_attention_metadata(self, num_tokens, num_reqs, *args, **kwargs):
        prompts = None
        batch = getattr(self, "input_batch", None)
        counts = getattr(batch, "num_prompt_tokens", None)
        if counts is not None:
            prompts = tuple(int(x) for x in counts[:int(num_reqs)])
        token = _STEP_PROMPTS.set(prompts)
        try:
            return prepare(self, num_tokens, num_reqs, *args, **kwargs)
        finally:
            _STEP_PROMPTS.reset(token)

    setattr(builder_cls, _META_ATTR, build)
    builder_cls.build = build_with_lengths
    setattr(runner_cls, _RUNNER_ATTR, prepare)
    runner_cls._build_attention_metadata = build_attention_metadata
    return True


def uninstall_vllm_metadata_patch(*, builder_cls: type | None = None,
                                  runner_cls: type | None = None) -> bool:
    if builder_cls is None or runner_cls is None:
        try:
            from vllm.v1.attention.backends.flash_attn import FlashAttentionMetadataBuilder
            from vllm.v1.worker.gpu_model_runner import GPUModelRunner
        except Exception:
            return False
        builder_cls = builder_cls or FlashAttentionMetadataBuilder
        runner_cls = runner_cls or GPUModelRunner
    done = False
    for cls, attr, name in ((builder_cls, _META_ATTR, "build"),
                            (runner_cls, _RUNNER_ATTR, "_build_attention_metadata")):
        original = getattr(cls, attr, None)
        if original is not None:
            setattr(cls, name, original)
            delattr(cls, attr)
            done = True
    return done


# vLLM's V2 model runner (vllm/v1/worker/gpu, the default for Qwen3 in vLLM
# 0.22) builds a step's attention metadata in ModelState.prepare_attn from its
# InputBatch; the scheduler's prompt lengths are in the runner's
# req_states.prompt_len, indexed by the batch's idx_mapping_np.
_V2_RUNNER: contextvars.ContextVar[Any] = contextvars.ContextVar("trianglemix_v2_runner",
                                                                 default=None)
_V2_EXEC_ATTR = "_trianglemix_original_execute_model"
_V2_PREP_ATTR = "_trianglemix_original_prepare_attn"


def install_vllm_v2_runner_patch(*, runner_cls: type | None = None,
                                 state_cls: type | None = None) -> bool:
    """Publish the final prompt lengths of each V2-runner step to the metadata
    builder patch (``install_vllm_metadata_patch``).

    ``runner_cls.execute_model`` is wrapped to make the runner visible while
    it runs; ``state_cls.prepare_attn`` is wrapped to read the prompt length
    of each batch row and publish them while the metadata is built.  Returns
    False when vLLM's V2 runner is not importable.
    """
    if runner_cls is None or state_cls is None:
        try:
            from vllm.v1.worker.gpu.model_runner import GPUModelRunner as V2Runner
            from vllm.v1.worker.gpu.model_states.default import DefaultModelState
        except Exception:
            return False
        runner_cls = runner_cls or V2Runner
        state_cls = state_cls or DefaultModelState
    execute = getattr(runner_cls, _V2_EXEC_ATTR, None) or runner_cls.execute_model
    prepare = getattr(state_cls, _V2_PREP_ATTR, None) or state_cls.prepare_attn

    def execute_model(self, *args, **kwargs):
        token = _V2_RUNNER.set(self)
        try:
            return execute(self, *args, **kwargs)
        finally:
            _V2_RUNNER.reset(token)

    def prepare_attn(self, input_batch, *args, **kwargs):
        prompts = None
        runner = _V2_RUNNER.get()
        if runner is not None:
            try:
                rows = input_batch.idx_mapping_np[:int(input_batch.num_reqs)]
                prompts = tuple(int(x) for x in runner.req_states.prompt_len.np[rows])
            except Exception:  # another runner layout: the step falls back
                runtime_stats().record_runtime_error(stage="v2_prompt_lengths")
        token = _STEP_PROMPTS.set(prompts)
        try:
            return prepare(self, input_batch, *args, **kwargs)
        finally:
            _STEP_PROMPTS.reset(token)

    setattr(runner_cls, _V2_EXEC_ATTR, execute)
    runner_cls.execute_model = execute_model
    setattr(state_cls, _V2_PREP_ATTR, prepare)
    state_cls.prepare_attn = prepare_attn
    return True


def uninstall_vllm_v2_runner_patch(*, runner_cls: type | None = None,
                                   state_cls: type | None = None) -> bool:
    if runner_cls is None or state_cls is None:
        try:
            from vllm.v1.worker.gpu.model_runner import GPUModelRunner as V2Runner
            from vllm.v1.worker.gpu.model_states.default import DefaultModelState
        except Exception:
            return False
        runner_cls = runner_cls or V2Runner
        state_cls = state_cls or DefaultModelState
    done = False
    for cls, attr, name in ((runner_cls, _V2_EXEC_ATTR, "execute_model"),
                            (state_cls, _V2_PREP_ATTR, "prepare_attn")):
        original = getattr(cls, attr, None)
        if original is not None:
            setattr(cls, name, original)
            delattr(cls, attr)
            done = True
    return done


# ------------------------------------------------------------ vLLM plugin entry
_REGISTER_LOCK = threading.Lock()
_ROUTER: TriangleMixRouter | None = None
_INIT_ATTR = "_trianglemix_original_init"


def registered_router() -> TriangleMixRouter | None:
    """The router ``register`` installed in this process, if any."""
    return _ROUTER


def _strict_from_environment() -> bool:
    value = os.getenv("VLLM_ASCEND_TRIANGLE_MIX_STRICT")
    try:
        return coerce_bool(value, name="strict") if value is not None else False
    except ValueError:
        return False


def _configure_from_vllm(router: TriangleMixRouter, impl_cls: type) -> None:
    """Wrap ``impl_cls.__init__`` so that the first attention layer vLLM
    builds (while its configuration is current) sets the router's
    configuration from ``additional_config.trianglemix``."""
    original = getattr(impl_cls, _INIT_ATTR, None) or impl_cls.__init__
    state = {"done": False}

    def __init__(self, *args, **kwargs):
        original(self, *args, **kwargs)
        if state["done"]:
            return
        state["done"] = True
        try:
            from vllm.config import get_current_vllm_config

            config = resolve_plugin_config(get_current_vllm_config())
        except Exception:
            runtime_stats().record_runtime_error(stage="plugin_config")
            if router.config.strict or _strict_from_environment():
                raise
            logger.warning("TriangleMix configuration could not be read; the stock "
                           "attention path stays active", exc_info=True)
            return
        router.config = config
        router.stats.configure(config.stats_recent_capacity, config.stats_log_interval)

    setattr(impl_cls, _INIT_ATTR, original)
    impl_cls.__init__ = __init__


# vLLM attention backends the plugin hooks: (module, impl class, metadata
# builder class, cache layout interleaved).  FlashAttention is vLLM's CUDA
# default; the Triton backend runs where vLLM's FlashAttention extension is
# not built (as in this image).
_BACKENDS = (
    ("vllm.v1.attention.backends.flash_attn", "FlashAttentionImpl",
     "FlashAttentionMetadataBuilder", False),
    ("vllm.v1.attention.backends.triton_attn", "TritonAttentionImpl",
     "TritonAttentionMetadataBuilder", True),
)
_HOOKED: list[tuple[type, type]] = []  # (impl class, builder class) hooked by register


def register() -> None:
    """vLLM ``general_plugins`` entry point (declared in pyproject.toml).

    Installs the forward hook and the metadata patch on each of vLLM's
    FlashAttention and Triton backends that imports, once per process
    (reference plugin.py:1705-1741).  The configuration starts from the
    environment and is replaced by ``additional_config.trianglemix`` when vLLM
    builds its first hooked attention layer; the path is off unless enabled.
    A failure leaves vLLM's own attention in place, or raises with
    ``strict``.
    """
    import importlib

    global _ROUTER
    with _REGISTER_LOCK:
        if _ROUTER is not None:
            return
        hooked: list[tuple[type, type]] = []
        try:
            from vllm.v1.worker.gpu_model_runner import GPUModelRunner

            router = TriangleMixRouter(resolve_plugin_config(None))
            for module, impl_name, builder_name, interleaved in _BACKENDS:
                try:
                    mod = importlib.import_module(module)
                    impl_cls, builder_cls = getattr(mod, impl_name), getattr(mod, builder_name)
                except Exception:  # this vLLM build lacks the backend
                    continue
                _configure_from_vllm(router, impl_cls)
                _install_hook(router, impl_cls, interleaved, None)
                if not install_vllm_metadata_patch(builder_cls=builder_cls,
                                                   runner_cls=GPUModelRunner):
                    raise RuntimeError(f"{builder_name} could not be patched")
                hooked.append((impl_cls, builder_cls))
            if not hooked:
                raise RuntimeError("no vLLM attention backend could be hooked")
            install_vllm_v2_runner_patch()
        except Exception:
            for impl_cls, builder_cls in hooked:
                _unhook(impl_cls, builder_cls)
            runtime_stats().record_runtime_error(stage="plugin_register")
            if _strict_from_environment():
                raise
            logger.warning("TriangleMix plugin could not hook vLLM; the stock attention "
                           "path stays active", exc_info=True)
            return
        _HOOKED[:] = hooked
        _ROUTER = router


def _unhook(impl_cls: type, builder_cls: type) -> None:
    from vllm.v1.worker.gpu_model_runner import GPUModelRunner

    _uninstall_hook(impl_cls)
    uninstall_vllm_metadata_patch(builder_cls=builder_cls, runner_cls=GPUModelRunner)
    original = getattr(impl_cls, _INIT_ATTR, None)
    if original is not None:
        impl_cls.__init__ = original
        delattr(impl_cls, _INIT_ATTR)


def unregister() -> bool:
    """Undo ``register`` in this process (vLLM's own attention path returns)."""
    global _ROUTER
    with _REGISTER_LOCK:
        if _ROUTER is None:
            return False
        for impl_cls, builder_cls in _HOOKED:
            _unhook(impl_cls, builder_cls)
        _HOOKED.clear()
        uninstall_vllm_v2_runner_patch()
        _ROUTER = None
        return True
