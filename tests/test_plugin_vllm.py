"""The vLLM integration against vLLM 0.22 itself, on CPU.

``register`` (the ``vllm.general_plugins`` entry point, reference
package/setup.py:292-294 and plugin.py:1705-1741) must wrap vLLM's real
FlashAttentionImpl, FlashAttentionMetadataBuilder and GPUModelRunner, and
undo it.  The metadata patch must carry the step's host lengths and the
scheduler's final prompt lengths to the planner, so that an intermediate
chunk of a chunked prefill is planned on the whole prompt (reference
package/tests/test_planning_stats.py:122-151) and a step without prompt
lengths falls back (reference plugin.py:523-570).
"""

from __future__ import annotations

import inspect
import sys
import types
from pathlib import Path

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package

tm = load_package()
FR = tm.planning.FallbackReason
ROOT = Path(__file__).resolve().parents[1]

vllm_fa = pytest.importorskip("vllm.v1.attention.backends.flash_attn")
vllm_runner = pytest.importorskip("vllm.v1.worker.gpu_model_runner")


def router(**cfg):
    kernel = tm.TriangleMixConfig(enabled=True, layer_indices=frozenset({1, 3, 5}))
    return tm.plugin.TriangleMixRouter(tm.config.PluginConfig(kernel=kernel, **cfg),
                                       stats=tm.stats.TriangleMixRuntimeStats())


def test_pyproject_declares_the_vllm_entry_point():
    import tomllib

    meta = tomllib.loads((ROOT / "pyproject.toml").read_text())
    target = meta["project"]["entry-points"]["vllm.general_plugins"]["trianglemix"]
    module, func = target.split(":")
    assert module == "trianglemix_b200.plugin" and func == "register"
    assert callable(getattr(tm.plugin, func))
    assert meta["tool"]["setuptools"]["package-dir"]["trianglemix_b200"] == \
        "sparse-attention-op-for-ascend-npu-_b200"


def test_register_wraps_and_unregister_restores_vllm():
    impl, builder, runner = (vllm_fa.FlashAttentionImpl, vllm_fa.FlashAttentionMetadataBuilder,
                             vllm_runner.GPUModelRunner)
    originals = (impl.forward, impl.__init__, builder.build, runner._build_attention_metadata)
    forward_params = list(inspect.signature(impl.forward).parameters)
    tm.plugin.register()
    try:
        assert tm.plugin.registered_router() is not None
        assert impl.forward is not originals[0] and impl._trianglemix_original_forward is originals[0]
        assert impl.__init__ is not originals[1]
        assert builder.build is not originals[2]
        assert runner._build_attention_metadata is not originals[3]
        # The hook reads these FlashAttentionMetadata fields.
        fields = {f.name for f in __import__("dataclasses").fields(vllm_fa.FlashAttentionMetadata)}
        assert {"query_start_loc", "seq_lens", "block_table", "causal",
                "num_actual_tokens"} <= fields
        # The wrapper takes forward's arguments (positional names match).
        wrapped = list(inspect.signature(impl.forward).parameters)
        assert wrapped == forward_params
        # Registering twice keeps one set of wrappers.
        tm.plugin.register()
        assert impl._trianglemix_original_forward is originals[0]
        # Off by default: no layer is selected.
        assert not tm.plugin.registered_router().selects("model.layers.5.self_attn.attn")
    finally:
        assert tm.plugin.unregister()
    assert (impl.forward, impl.__init__, builder.build,
            runner._build_attention_metadata) == originals


class FakeBuilder:
    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        return types.SimpleNamespace(query_start_loc=None, seq_lens=None)


class FakeRunner:
    """Calls the builder inside _build_attention_metadata, as vLLM's runner does."""

    def __init__(self, prompts, common):
        self.input_batch = types.SimpleNamespace(num_prompt_tokens=np.array(prompts + [0, 0]))
        self.common = common

    def _build_attention_metadata(self, num_tokens, num_reqs, max_query_len, **kwargs):
        return FakeBuilder().build(0, self.common)


def test_metadata_patch_carries_host_and_prompt_lengths():
    common = types.SimpleNamespace(num_reqs=2, query_start_loc_cpu=torch.tensor([0, 2048, 2176]),
                                   _seq_lens_cpu=torch.tensor([4096, 8320, 0]))
    assert tm.plugin.install_vllm_metadata_patch(builder_cls=FakeBuilder, runner_cls=FakeRunner)
    try:
        meta = FakeRunner([8320, 8320], common)._build_attention_metadata(2176, 2, 2048)
        assert meta.trianglemix_query_start_loc == [0, 2048, 2176]
        assert meta.trianglemix_seq_lens == [4096, 8320]
        assert meta.trianglemix_prompt_lens == [8320, 8320]
        # Outside the runner the builder attaches no prompt lengths.
        plain = FakeBuilder().build(0, common)
        assert not hasattr(plain, "trianglemix_prompt_lens")
    finally:
        assert tm.plugin.uninstall_vllm_metadata_patch(builder_cls=FakeBuilder,
                                                       runner_cls=FakeRunner)
    assert not hasattr(FakeBuilder, "_trianglemix_original_build")


def meta(starts, seqs, prompts=None):
    m = types.SimpleNamespace(query_start_loc=torch.tensor(starts), seq_lens=torch.tensor(seqs))
    m.trianglemix_query_start_loc = list(starts)
    m.trianglemix_seq_lens = list(seqs)
    if prompts is not None:
        m.trianglemix_prompt_lens = list(prompts)
    return m


def test_chunked_prefill_is_planned_on_the_final_prompt_through_the_hook():
    r = router()
    first = r.plan_for_metadata(meta([0, 2048], [2048], [8320]))
    middle = r.plan_for_metadata(meta([0, 2048], [4096], [8320]))
    tail = r.plan_for_metadata(meta([0, 128], [8320], [8320]))
    # The reference's thresholds (TriangleMixConfig defaults): the first chunk
    # saves too few pairs, the middle chunk is direct, the final 128-row
    # chunk is all dense tail (the reference test's three outcomes).
    assert not first.direct and first.primary_reason is FR.BELOW_SPLIT_MIN_SAVED_QK
    assert middle.direct
    assert not tail.direct and tail.primary_reason is FR.NO_SPARSE_MIDDLE
    # An intermediate chunk has no dense tail of its own: its plan ends its
    # sparse rows at the prompt's last 128 rows, not at the chunk's end.
    assert middle.requests[0].prompt_len == 8320
    # Without prompt lengths the step falls back (it is not planned as if the
    # prompt ended at the chunk's end).
    missing = r.plan_for_metadata(meta([0, 2048], [4096]))
    assert not missing.direct and missing.primary_reason is FR.MISSING_METADATA
    # A provider callback still supplies them.
    provided = r.plan_for_metadata(meta([0, 2048], [4096]), lambda m: [8320])
    assert provided.direct


def test_host_lengths_avoid_device_reads():
    r = router()
    m = meta([0, 4096], [4096], [4096])
    m.query_start_loc = m.seq_lens = None  # would fail if the planner read them
    assert r.plan_for_metadata(m).direct


class FakeImpl:
    def __init__(self, dcp=1):
        self.calls = 0
        self.dcp_world_size = dcp

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        self.calls += 1
        return output


def test_context_parallel_falls_back():
    r = router()
    assert tm.plugin.install_vllm_flash_attention_hook(r, impl_cls=FakeImpl)
    try:
        impl = FakeImpl(dcp=2)
        m = meta([0, 4096], [4096], [4096])
        m.num_actual_tokens, m.causal = 4096, True
        m.block_table = torch.zeros(1, 32, dtype=torch.int32)
        q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16)
        kv = torch.zeros(2, 64, 128, 8, 128, dtype=torch.bfloat16)
        out = torch.zeros(4096, 32 * 128, dtype=torch.bfloat16)
        layer = types.SimpleNamespace(layer_name="model.layers.3.self_attn.attn")
        impl.forward(layer, q, None, None, kv, m, out)
        assert impl.calls == 1
        assert r.stats.snapshot()["counters"]["layer_fia_reason:context_parallel"] == 1
    finally:
        assert tm.plugin.uninstall_vllm_flash_attention_hook(impl_cls=FakeImpl)


def test_router_keeps_one_workspace_per_device():
    r = router()
    dev = torch.device("cpu")
    for n in (4096, 1 << 20, 2048, 3 << 20, 512):
        ws = r._workspace(dev, n)
        assert ws.numel() >= n
    assert len(r._workspaces) == 1
    assert r._workspaces[0].numel() == 3 << 20


vllm_triton = pytest.importorskip("vllm.v1.attention.backends.triton_attn")


def test_register_hooks_the_triton_backend_too():
    impl, builder = vllm_triton.TritonAttentionImpl, vllm_triton.TritonAttentionMetadataBuilder
    originals = (impl.forward, impl.__init__, builder.build)
    forward_params = list(inspect.signature(impl.forward).parameters)
    tm.plugin.register()
    try:
        assert impl.forward is not originals[0] and impl._trianglemix_original_forward is originals[0]
        assert impl.__init__ is not originals[1] and builder.build is not originals[2]
        assert list(inspect.signature(impl.forward).parameters) == forward_params
        # The Triton backend's cache shape, which the hook reads in place.
        assert vllm_triton.TritonAttentionBackend.get_kv_cache_shape(10, 128, 8, 128) == \
            (10, 2, 128, 8, 128)
        fields = {f.name for f in __import__("dataclasses").fields(vllm_triton.TritonAttentionMetadata)}
        assert {"query_start_loc", "seq_lens", "block_table", "num_actual_tokens"} <= fields
    finally:
        assert tm.plugin.unregister()
    assert (impl.forward, impl.__init__, builder.build) == originals


def test_interleaved_pages_view_and_doubled_table():
    kv = torch.arange(3 * 2 * 4 * 2 * 3, dtype=torch.float32).view(3, 2, 4, 2, 3)
    pages = tm.plugin.interleaved_pages(kv)
    assert pages.shape == (6, 4, 2, 3) and pages.data_ptr() == kv.data_ptr()
    for b in range(3):
        assert torch.equal(pages[2 * b], kv[b, 0]) and torch.equal(pages[2 * b + 1], kv[b, 1])
    assert tm.plugin.interleaved_pages(kv.transpose(0, 1)) is None
    assert tm.plugin.interleaved_pages(torch.zeros(2, 3, 4, 2, 3)) is None
    m = types.SimpleNamespace(block_table=torch.tensor([[4, 0, 7]], dtype=torch.int32))
    table = tm.plugin.interleaved_block_table(m)
    assert table.dtype == torch.int32 and table.tolist() == [[8, 0, 14]]
    assert tm.plugin.interleaved_block_table(m) is table  # once per step's metadata
    # A shallow copy with another block table (vLLM's update_block_table).
    import copy
    m2 = copy.copy(m)
    m2.block_table = torch.tensor([[1, 2, 3]], dtype=torch.int32)
    assert tm.plugin.interleaved_block_table(m2).tolist() == [[2, 4, 6]]
    assert tm.plugin.interleaved_block_table(m) is table


class CaptureRouter:
    """Router stand-in that records what the hook hands to ``attend``."""

    def __init__(self):
        self.seen = None
        self.stats = tm.stats.TriangleMixRuntimeStats()

    def selects(self, name):
        return True

    def plan_for_metadata(self, metadata, provider=None):
        return types.SimpleNamespace(plan_id=1)

    def attend(self, plan, name, q, key_cache, value_cache, table, out, **kw):
        self.seen = (key_cache, value_cache, table, kw)
        return True


def test_triton_hook_passes_the_interleaved_cache():
    r = CaptureRouter()
    assert tm.plugin.install_vllm_triton_attention_hook(r, impl_cls=FakeImpl)
    try:
        impl = FakeImpl()
        m = types.SimpleNamespace(num_actual_tokens=256,
                                  block_table=torch.tensor([[3, 1]], dtype=torch.int32))
        q = torch.zeros(256, 32, 128, dtype=torch.bfloat16)
        kv = torch.zeros(4, 2, 128, 8, 128, dtype=torch.bfloat16)
        out = torch.zeros(256, 32 * 128, dtype=torch.bfloat16)
        layer = types.SimpleNamespace(layer_name="model.layers.3.self_attn.attn")
        assert impl.forward(layer, q, None, None, kv, m, out) is out
        assert impl.calls == 0  # the kernel path took the call
        key_cache, value_cache, table, kw = r.seen
        assert key_cache.shape == (8, 128, 8, 128) and value_cache is key_cache
        assert key_cache.data_ptr() == kv.data_ptr()
        assert table.tolist() == [[6, 2]] and kw["value_offset_pages"] == 1
        # A cache of another layout goes to the stock path with a reason.
        impl.forward(layer, q, None, None, kv.transpose(0, 1).contiguous().transpose(0, 1), m, out)
        assert impl.calls == 1
        assert r.stats.snapshot()["counters"]["layer_fia_reason:kv_cache_unsupported"] == 1
    finally:
        assert tm.plugin.uninstall_vllm_triton_attention_hook(impl_cls=FakeImpl)


class FakeV2State:
    """Builds the step's metadata in prepare_attn, as vLLM's V2 ModelState does."""

    common = None

    def prepare_attn(self, input_batch, cudagraph_mode, block_tables, slot_mappings,
                     attn_groups, kv_cache_config, for_capture=False):
        return FakeBuilder().build(common_prefix_len=0, common_attn_metadata=self.common)


class FakeV2Runner:
    def __init__(self, prompt_lens, common):
        self.req_states = types.SimpleNamespace(
            prompt_len=types.SimpleNamespace(np=np.array(prompt_lens, dtype=np.int32)))
        self.model_state = FakeV2State()
        self.model_state.common = common

    def execute_model(self, input_batch):
        return self.model_state.prepare_attn(input_batch, None, (), None, [], None)


def test_v2_runner_patch_carries_prompt_lengths_in_batch_order():
    common = types.SimpleNamespace(num_reqs=2, query_start_loc_cpu=torch.tensor([0, 2048, 2176]),
                                   _seq_lens_cpu=torch.tensor([4096, 8320]))
    assert tm.plugin.install_vllm_metadata_patch(builder_cls=FakeBuilder, runner_cls=FakeRunner)
    assert tm.plugin.install_vllm_v2_runner_patch(runner_cls=FakeV2Runner, state_cls=FakeV2State)
    try:
        runner = FakeV2Runner([9000, 8320, 4096], common)
        # Batch rows 0 and 1 are request states 2 and 0.
        batch = types.SimpleNamespace(num_reqs=2, idx_mapping_np=np.array([2, 0]))
        meta = runner.execute_model(batch)
        assert meta.trianglemix_prompt_lens == [4096, 9000]
        # prepare_attn outside execute_model (a capture or dummy run): none.
        plain = runner.model_state.prepare_attn(batch, None, (), None, [], None)
        assert not hasattr(plain, "trianglemix_prompt_lens")
    finally:
        assert tm.plugin.uninstall_vllm_v2_runner_patch(runner_cls=FakeV2Runner,
                                                        state_cls=FakeV2State)
        assert tm.plugin.uninstall_vllm_metadata_patch(builder_cls=FakeBuilder,
                                                       runner_cls=FakeRunner)


def test_register_patches_vllm_v2_runner():
    v2_runner = pytest.importorskip("vllm.v1.worker.gpu.model_runner")
    v2_state = pytest.importorskip("vllm.v1.worker.gpu.model_states.default")
    runner, state = v2_runner.GPUModelRunner, v2_state.DefaultModelState
    originals = (runner.execute_model, state.prepare_attn)
    assert list(inspect.signature(state.prepare_attn).parameters)[:2] == ["self", "input_batch"]
    tm.plugin.register()
    try:
        assert runner.execute_model is not originals[0]
        assert state.prepare_attn is not originals[1]
    finally:
        assert tm.plugin.unregister()
    assert (runner.execute_model, state.prepare_attn) == originals
