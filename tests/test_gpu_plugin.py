"""The serving router and the vLLM-hook path on the GPU, against the oracle.

The router launches through the C ABI (batch-one, head shard, varlen) and the
hook wraps a FlashAttentionImpl-shaped class: kv_cache [2, pages, 128, heads,
128] and output [tokens, heads * 128], as vLLM's CUDA backend passes them.
"""

from __future__ import annotations

import types

import pytest
import torch

from __graft_entry__ import load_package
from gpu_helpers import assert_close
from inputs import SCALE, baseline_inputs, varlen_inputs
from oracle.triangle_oracle import oracle_attention

pytestmark = pytest.mark.gpu
tm = load_package()


def router():
    kcfg = tm.TriangleMixConfig(enabled=True, layer_indices=frozenset({0}),
                                direct_min_sparse_rows=0, direct_min_saved_qk=0,
                                direct_split_min_sparse_rows=0, direct_split_min_saved_qk=0)
    return tm.plugin.TriangleMixRouter(tm.config.PluginConfig(kernel=kcfg, strict=True),
                                       stats=tm.stats.TriangleMixRuntimeStats())


def test_router_batch_one_and_head_shard(cuda_device):
    r = router()
    q, k, v, table = baseline_inputs(1500, 1500, seed=31)
    p = r.plan_step(query_lens=[1500], seq_lens=[1500])
    assert p.direct
    ref = oracle_attention(q, k, v, table, 0, 1500, 1500, SCALE).to(torch.bfloat16)
    qd, kd, vd, td = (t.to(cuda_device) for t in (q, k, v, table))
    out = torch.empty_like(qd)
    assert r.attend(p, "model.layers.0.attn", qd, kd, vd, td, out)
    torch.cuda.synchronize()
    assert_close(out.cpu(), ref, "router batch-one")
    # A tensor-parallel shard: KV heads 2-3 and their query heads 8-15.
    qs, ks, vs = qd[:, 8:16].contiguous(), kd[:, :, 2:4].contiguous(), vd[:, :, 2:4].contiguous()
    outs = torch.empty_like(qs)
    assert r.attend(p, "model.layers.0.attn", qs, ks, vs, td, outs)
    torch.cuda.synchronize()
    assert_close(outs.cpu(), ref[:, 8:16], "router head shard")
    assert tm._native.device_status(cuda_device.index or 0) == 0
    assert r.stats.snapshot()["counters"]["layer_direct"] == 2


def test_hook_varlen_batch_matches_oracle(cuda_device):
    specs = [(900, 900, 900), (640, 1200, 1200), (1100, 1100, 1100)]
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=32)
    r = router()

    class Impl:
        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            raise AssertionError("the stock path must not run for this batch")

    assert tm.plugin.install_vllm_flash_attention_hook(r, impl_cls=Impl)
    try:
        kv = torch.stack([k, v]).to(cuda_device)
        meta = types.SimpleNamespace(
            query_start_loc=torch.tensor(cu, dtype=torch.int32, device=cuda_device),
            seq_lens=torch.tensor([s for _, s, _ in specs], dtype=torch.int32, device=cuda_device),
            num_actual_tokens=cu[-1], block_table=tables.to(cuda_device), causal=True,
            # the scheduler's final prompt lengths, as the metadata patch attaches them
            trianglemix_prompt_lens=[p for _, _, p in specs])
        out = torch.zeros(cu[-1], 32 * 128, dtype=torch.bfloat16, device=cuda_device)
        layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
        Impl().forward(layer, q.to(cuda_device), None, None, kv, meta, out)
        torch.cuda.synchronize()
    finally:
        tm.plugin.uninstall_vllm_flash_attention_hook(impl_cls=Impl)
    got = out.view(cu[-1], 32, 128).cpu()
    for i, (rows, seq, prompt) in enumerate(specs):
        ref = oracle_attention(q[cu[i]:cu[i + 1]], k, v, per_request[i], seq - rows, seq, prompt,
                               SCALE)
        assert_close(got[cu[i]:cu[i + 1]], ref.to(torch.bfloat16), f"hook request {i}")
    snap = r.stats.snapshot()
    assert snap["counters"]["layer_direct"] == 1 and snap["counters"]["request_total"] == 3


@pytest.mark.parametrize("specs", [[(1500, 1500, 1500)],
                                   [(900, 900, 900), (640, 1200, 1200), (1100, 1100, 1100)]],
                         ids=["batch_one", "varlen"])
def test_triton_hook_interleaved_cache_matches_oracle(cuda_device, specs):
    """vLLM's Triton backend cache, [num_blocks, 2, 128, heads, 128]: the hook
    reads a block's K and V pages in place (doubled block table, V one page
    past K) and must match the oracle on the same K and V."""
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=33)
    r = router()

    class Impl:
        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            raise AssertionError("the stock path must not run for this batch")

    assert tm.plugin.install_vllm_triton_attention_hook(r, impl_cls=Impl)
    try:
        kv = torch.stack([k, v], dim=1).to(cuda_device)  # [blocks, 2, 128, 8, 128]
        meta = types.SimpleNamespace(
            query_start_loc=torch.tensor(cu, dtype=torch.int32, device=cuda_device),
            seq_lens=torch.tensor([s for _, s, _ in specs], dtype=torch.int32, device=cuda_device),
            num_actual_tokens=cu[-1], block_table=tables.to(cuda_device),
            trianglemix_prompt_lens=[p for _, _, p in specs])
        out = torch.zeros(cu[-1], 32 * 128, dtype=torch.bfloat16, device=cuda_device)
        layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
        Impl().forward(layer, q.to(cuda_device), None, None, kv, meta, out)
        torch.cuda.synchronize()
    finally:
        tm.plugin.uninstall_vllm_triton_attention_hook(impl_cls=Impl)
    assert tm._native.device_status(cuda_device.index or 0) == 0
    got = out.view(cu[-1], 32, 128).cpu()
    for i, (rows, seq, prompt) in enumerate(specs):
        ref = oracle_attention(q[cu[i]:cu[i + 1]], k, v, per_request[i], seq - rows, seq, prompt,
                               SCALE)
        assert_close(got[cu[i]:cu[i + 1]], ref.to(torch.bfloat16), f"triton hook request {i}")
    assert r.stats.snapshot()["counters"]["layer_direct"] == 1
