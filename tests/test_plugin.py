"""Serving integration on CPU: configuration, per-step plans, counters, routing.

Cases follow the reference plugin's own tests
(package/tests/test_planning_stats.py and test_plugin.py in the reference
project): the same configuration precedence, the same crossover boundaries
(2260 / 2261 tokens), chunked prefills planned on the final prompt length,
decode and mixed batches falling back, plans counted once across layers.
Where this build differs on purpose, the test says so: a packed batch of
eligible prefills is direct here (one varlen launch).  The router's launch
itself needs a GPU (tests/test_gpu_plugin.py); here its decisions run against
CPU tensors, which the router must reject before any launch.
"""

from __future__ import annotations

import os
import types
from unittest.mock import patch

import pytest
import torch

from __graft_entry__ import load_package

tm = load_package()
FR = tm.planning.FallbackReason


def kcfg(**overrides):
    values = dict(enabled=True, layer_indices=frozenset({1, 3, 5}))
    values.update(overrides)
    return tm.TriangleMixConfig(**values)


def plan(*, state="PrefillNoCache", ends, seqs, prompts, decodes=0, prefills=None, config=None):
    return tm.planning.build_batch_plan(
        state_name=state, cumulative_query_ends=ends, seq_lens=seqs, prompt_lens=prompts,
        num_decodes=decodes, num_prefills=len(seqs) if prefills is None else prefills,
        config=config or kcfg())


# ------------------------------------------------------------------ config
def test_additional_config_section_and_string_booleans():
    holder = types.SimpleNamespace(additional_config={
        "trianglemix": {"enabled": "false", "strict": "off", "layers": "1,3-4"}})
    resolved = tm.config.resolve_plugin_config(holder)
    assert not resolved.kernel.enabled and not resolved.strict
    assert resolved.kernel.layer_indices == frozenset({1, 3, 4})


def test_invalid_boolean_is_rejected():
    holder = types.SimpleNamespace(additional_config={"trianglemix": {"enabled": "sometimes"}})
    with pytest.raises(ValueError, match="must be a boolean"):
        tm.config.resolve_plugin_config(holder)


def test_environment_is_the_fallback_and_section_wins():
    env = {"VLLM_ASCEND_ENABLE_TRIANGLE_MIX": "yes", "VLLM_ASCEND_TRIANGLE_MIX_LAYERS": "2-3",
           "VLLM_ASCEND_TRIANGLE_MIX_DIRECT_MIN_SAVED_QK": "5"}
    with patch.dict(os.environ, env, clear=True):
        resolved = tm.config.resolve_plugin_config(None)
        assert resolved.enabled and resolved.kernel.layer_indices == frozenset({2, 3})
        assert resolved.kernel.direct_min_saved_qk == 5
        holder = types.SimpleNamespace(additional_config={"layers": [7]})
        assert tm.config.resolve_plugin_config(holder).kernel.layer_indices == frozenset({7})


def test_threshold_profiles():
    # Default: the thresholds measured on B200 (no saved-pairs minimum).
    with patch.dict(os.environ, {}, clear=True):
        b200 = tm.config.resolve_plugin_config(None).kernel
        assert (b200.direct_min_saved_qk, b200.direct_split_min_saved_qk) == (0, 0)
        assert b200.direct_min_sparse_rows == 128 and b200.direct_split_min_sparse_rows == 128
        # "910b" restores the reference's values.
        ref = tm.config.resolve_plugin_config(types.SimpleNamespace(
            additional_config={"trianglemix": {"threshold_profile": "910B"}})).kernel
        assert (ref.direct_min_saved_qk, ref.direct_split_min_saved_qk) == (913_152, 1_299_264)
        assert ref.direct_split_min_sparse_rows == 192
        # An explicit threshold key wins over the profile.
        mixed = tm.config.resolve_plugin_config(types.SimpleNamespace(
            additional_config={"trianglemix": {"min_saved_qk": 7}})).kernel
        assert mixed.direct_min_saved_qk == 7 and mixed.direct_split_min_saved_qk == 0
    with patch.dict(os.environ, {"VLLM_ASCEND_TRIANGLE_MIX_THRESHOLD_PROFILE": "910b"},
                    clear=True):
        assert tm.config.resolve_plugin_config(None).kernel.direct_min_saved_qk == 913_152
    with pytest.raises(ValueError, match="threshold_profile"):
        tm.config.resolve_plugin_config(types.SimpleNamespace(
            additional_config={"threshold_profile": "h100"}))


def test_b200_thresholds_route_early_chunks_direct():
    # The second 512-token chunk of a long prompt (503 sparse rows, 126,756
    # saved pairs) falls back under the reference's 910B gates but measured
    # 2.4x faster through this library on B200 than the dense baseline.
    with patch.dict(os.environ, {"VLLM_ASCEND_ENABLE_TRIANGLE_MIX": "1",
                                 "VLLM_ASCEND_TRIANGLE_MIX_LAYERS": "1"}, clear=True):
        b200 = tm.config.resolve_plugin_config(None).kernel
    args = dict(ends=[512], seqs=[1024], prompts=[8192], state="ChunkedPrefill")
    assert plan(**args, config=b200).direct
    reference = plan(**args)
    assert not reference.direct


def test_negative_stats_capacity_is_rejected():
    holder = types.SimpleNamespace(additional_config={"stats_recent_capacity": -1})
    with pytest.raises(ValueError, match="non-negative"):
        tm.config.resolve_plugin_config(holder)


# ------------------------------------------------------------------ planning
def test_full_prompt_split_crossover_boundary():
    before = plan(ends=[2260], seqs=[2260], prompts=[2260])
    at = plan(ends=[2261], seqs=[2261], prompts=[2261])
    assert not before.direct and before.primary_reason is FR.BELOW_SPLIT_MIN_SAVED_QK
    assert at.direct and at.requests[0].saved_qk == 1_300_078


def test_chunked_prefill_uses_final_prompt_length():
    first = plan(state="ChunkedPrefill", ends=[2048], seqs=[2048], prompts=[8320])
    middle = plan(state="ChunkedPrefill", ends=[2048], seqs=[4096], prompts=[8320])
    tail = plan(state="ChunkedPrefill", ends=[128], seqs=[8320], prompts=[8320])
    assert first.primary_reason is FR.BELOW_SPLIT_MIN_SAVED_QK
    assert middle.direct and (middle.requests[0].q_begin, middle.requests[0].q_end) == (2048, 4096)
    assert tail.primary_reason is FR.NO_SPARSE_MIDDLE


def test_decode_and_mixed_batches_fall_back():
    decode = plan(state="DecodeOnly", ends=[1], seqs=[4096], prompts=[4096], decodes=1,
                  prefills=0)
    mixed = plan(state="ChunkedPrefill", ends=[1, 2049], seqs=[4096, 4096],
                 prompts=[4096, 8320], decodes=1, prefills=1)
    assert decode.primary_reason is FR.STATE_UNSUPPORTED
    assert mixed.primary_reason is FR.MIXED_DECODE


def test_packed_batch_of_eligible_prefills_is_direct():
    """Differs from the reference on purpose: batch > 1 runs as one varlen launch."""
    p = plan(ends=[2048, 3072], seqs=[4096, 7168], prompts=[8320, 8192])
    assert [r.query_len for r in p.requests] == [2048, 1024]
    assert p.direct and p.cu_seqlens_q == [0, 2048, 3072]
    partial = plan(ends=[2048, 2148], seqs=[4096, 100], prompts=[8320, 100])
    assert not partial.direct and partial.primary_reason is FR.NO_SPARSE_MIDDLE


def test_missing_metadata_and_geometry():
    assert plan(ends=[4096], seqs=[4096], prompts=None).primary_reason is FR.MISSING_METADATA
    odd = plan(ends=[4096], seqs=[4096], prompts=[4096], config=kcfg(local_window=1024))
    assert odd.primary_reason is FR.GEOMETRY_UNSUPPORTED
    empty = plan(ends=[], seqs=[], prompts=[])
    assert empty.batch_size == 0 and empty.primary_reason is FR.MISSING_METADATA


def test_step_state_from_lengths():
    st = tm.plugin.step_state
    assert st([1, 1], [10, 20]) == ("DecodeOnly", 2)
    assert st([10, 20], [10, 20]) == ("PrefillNoCache", 0)
    assert st([10, 1], [30, 20]) == ("ChunkedPrefill", 1)


# ------------------------------------------------------------------ stats
def test_plan_counted_once_and_layer_counters():
    stats = tm.stats.TriangleMixRuntimeStats()
    stats.configure(4)
    p = plan(ends=[4096], seqs=[4096], prompts=[4096])
    stats.record_planner_decision(p)
    stats.record_planner_decision(p)
    stats.record_layer_dispatch(plan_id=p.plan_id, layer_index=7, saved_qk=2_000_000,
                                host_enqueue_ns=31_000)
    stats.record_layer_dispatch(plan_id=p.plan_id, layer_index=7, saved_qk=2_000_000,
                                host_enqueue_ns=41_000)
    stats.record_layer_fallback(plan_id=p.plan_id, layer_index=9, reason=FR.GRAPH_CAPTURE)
    snap = stats.snapshot()
    c = snap["counters"]
    assert c["request_total"] == 1 and c["request_planner_eligible"] == 1
    assert c["single_launch"] == 2 and c["layer_fia_reason:graph_capture"] == 1
    assert snap["layers"] == {"direct": {"7": 2}, "fia": {"9": 1}}
    assert snap["performance"]["host_enqueue_us_per_launch"] == 36.0
    assert snap["performance"]["host_enqueue_us_max"] == 41.0
    ex = snap["recent"][0]["execution"]
    assert ex["observed_route"] == "mixed" and ex["fallback_reasons"] == {"graph_capture": 1}
    stats.snapshot(reset=True)
    assert stats.snapshot()["counters"] == {}


def test_recent_capacity_and_log_interval():
    stats = tm.stats.TriangleMixRuntimeStats()
    stats.configure(2, log_interval=3)
    logs = []
    for _ in range(5):
        stats.record_planner_decision(plan(ends=[4096], seqs=[4096], prompts=[4096]))
        entry = stats.structured_log_if_due()
        if entry is not None:
            logs.append(entry["counters"]["request_total"])
    assert logs == [3]
    assert len(stats.snapshot()["recent"]) == 2


# ------------------------------------------------------------------ router / hook
def router(strict=False):
    cfg = tm.config.PluginConfig(kernel=kcfg(), strict=strict)
    return tm.plugin.TriangleMixRouter(cfg, stats=tm.stats.TriangleMixRuntimeStats())


def test_router_rejects_cpu_tensors_before_any_launch():
    r = router()
    p = r.plan_step(query_lens=[4096], seq_lens=[4096])
    q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16)
    kc = torch.zeros(64, 128, 8, 128, dtype=torch.bfloat16)
    table = torch.zeros(1, 32, dtype=torch.int32)
    assert not r.attend(p, "model.layers.1.self_attn", q, kc, kc, table, torch.empty_like(q))
    assert r.stats.snapshot()["counters"]["layer_fia_reason:query_unsupported"] == 1
    # Non-causal and unsupported features are reported as such.
    assert r.dispatch_reason(p, q, kc, kc, table, q, causal=False) is FR.NON_CAUSAL
    assert r.dispatch_reason(p, q, kc, kc, table, q, unsupported_features=True) \
        is FR.MODEL_UNSUPPORTED
    ineligible = r.plan_step(query_lens=[100], seq_lens=[100])
    assert r.dispatch_reason(ineligible, q, kc, kc, table, q) is FR.NO_SPARSE_MIDDLE


class FakeImpl:
    """Stands in for vLLM's FlashAttentionImpl (same forward signature)."""

    def __init__(self):
        self.calls = 0

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        self.calls += 1
        return output


def test_hook_routes_only_selected_layers_and_falls_back():
    r = router()
    assert tm.plugin.install_vllm_flash_attention_hook(r, impl_cls=FakeImpl)
    try:
        impl = FakeImpl()
        meta = types.SimpleNamespace(query_start_loc=torch.tensor([0, 4096]),
                                     seq_lens=torch.tensor([4096]), num_actual_tokens=4096,
                                     block_table=torch.zeros(1, 32, dtype=torch.int32),
                                     causal=True)
        q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16)
        kv = torch.zeros(2, 64, 128, 8, 128, dtype=torch.bfloat16)
        out = torch.zeros(4096, 32 * 128, dtype=torch.bfloat16)
        unselected = types.SimpleNamespace(layer_name="model.layers.2.self_attn.attn")
        selected = types.SimpleNamespace(layer_name="model.layers.3.self_attn.attn")
        impl.forward(unselected, q, None, None, kv, meta, out)
        assert impl.calls == 1 and r.stats.snapshot()["counters"] == {}
        impl.forward(selected, q, None, None, kv, meta, out)   # CPU tensors: stock path
        impl.forward(selected, q, None, None, kv, meta, out)   # same step: plan reused
        snap = r.stats.snapshot()
        assert impl.calls == 3
        assert snap["counters"]["request_total"] == 1
        assert snap["layers"]["fia"] == {"3": 2}
        assert impl.forward(selected, q, None, None, kv, None, out) is out  # profiling run
    finally:
        assert tm.plugin.uninstall_vllm_flash_attention_hook(impl_cls=FakeImpl)
    assert not hasattr(FakeImpl, "_trianglemix_original_forward")


def test_nvtx_ranges_are_balanced_and_never_raise(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    with tm.plugin._NvtxRange("trianglemix.attend"):
        pass
    assert calls == [("push", "trianglemix.attend"), ("pop",)]

    def broken(name):
        raise RuntimeError("no NVTX")

    monkeypatch.setattr(torch.cuda.nvtx, "range_push", broken)
    calls.clear()
    with tm.plugin._NvtxRange("trianglemix.plan"):
        pass
    assert calls == []  # nothing pushed, nothing popped
