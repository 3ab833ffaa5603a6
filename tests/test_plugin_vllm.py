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
