"""The torch operator boundary: schemas, fail-closed checks, out semantics.

Mirrors the reference adapter contracts (operator/torch_adapter/
triangle_paged_attention_torch.cpp:29-97, tests test_adapter_out_contract.py)
on the CUDA dispatch key.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close
from inputs import SCALE, baseline_inputs
from oracle.triangle_oracle import oracle_attention

pytestmark = pytest.mark.gpu


def _inputs(dev, seq=1300, prompt=1300):
    q, k, v, table = baseline_inputs(seq, seq, seed=41)
    return (q, k, v, table), tuple(t.to(dev) for t in (q, k, v, table))


def test_out_variant_writes_caller_buffer(adapter, cuda_device):
    (q, k, v, table), (qd, kd, vd, td) = _inputs(cuda_device)
    out = torch.full_like(qd, float("nan"))
    ptr = out.data_ptr()
    res = torch.ops.trianglemix.triangle_paged_sparse_attention.out(
        qd, kd, vd, td, 0, 1300, 1300, SCALE, out=out)
    torch.cuda.synchronize()
    assert res.data_ptr() == ptr
    assert_close(out.cpu(), oracle_attention(q, k, v, table, 0, 1300, 1300, SCALE), "out variant")


def test_c_ascend_alias_is_the_out_operator(adapter, cuda_device):
    """torch.ops._C_ascend.npu_triangle_paged_sparse_attention, the name of the
    reference's in-tree registration (README.md:34-36 of the reference), writes
    the caller's buffer and applies the same gates."""
    (q, k, v, table), (qd, kd, vd, td) = _inputs(cuda_device)
    out = torch.full_like(qd, float("nan"))
    ptr = out.data_ptr()
    res = torch.ops._C_ascend.npu_triangle_paged_sparse_attention(
        qd, kd, vd, td, 0, 1300, 1300, SCALE, out=out)
    torch.cuda.synchronize()
    assert res.data_ptr() == ptr
    assert_close(out.cpu(), oracle_attention(q, k, v, table, 0, 1300, 1300, SCALE), "_C_ascend")
    with pytest.raises(RuntimeError, match="query must be BF16"):
        torch.ops._C_ascend.npu_triangle_paged_sparse_attention(
            qd.float(), kd, vd, td, 0, 1300, 1300, SCALE, out=out)


def test_functional_variant_and_workspace_size(adapter, cuda_device):
    (q, k, v, table), (qd, kd, vd, td) = _inputs(cuda_device)
    out = torch.ops.trianglemix_reference.triangle_paged_sparse_attention(qd, kd, vd, td, 0, 1300,
                                                                          1300, SCALE)
    torch.cuda.synchronize()
    assert_close(out.cpu(), oracle_attention(q, k, v, table, 0, 1300, 1300, SCALE), "functional")
    ws = torch.ops.trianglemix_reference.triangle_paged_sparse_attention_workspace_size(
        qd, kd, vd, td, 0, 1300, 1300, SCALE)
    assert ws == adapter._native.workspace_size(1300, 0, 1300, 1300)


def test_direct_path_api(adapter, cuda_device):
    """kernel.triangle_direct_paged_attention (reference kernel.py:445-489)."""
    (q, k, v, table), (qd, kd, vd, td) = _inputs(cuda_device, 2048, 4096)
    cfg = adapter.TriangleMixConfig(enabled=True, layer_indices=frozenset({5}))
    out = torch.empty_like(qd)
    adapter.triangle_direct_paged_attention(query=qd, key_cache=kd, value_cache=vd, block_table=td,
                                            seq_len=2048, prompt_len=4096, output=out,
                                            softmax_scale=SCALE, config=cfg)
    torch.cuda.synchronize()
    assert_close(out.cpu(), oracle_attention(q, k, v, table, 0, 2048, 4096, SCALE), "direct path")


@pytest.mark.parametrize("mutate,message", [
    (lambda t: (t[0].float(),) + t[1:], "query must be BF16"),
    (lambda t: (t[0][:, :16].contiguous(),) + t[1:], "query must be [Tq, 32, 128]"),
    (lambda t: (t[0], t[1][:, :, :4].contiguous(), t[2], t[3]), "key_cache must be [pages, 128, 8, 128]"),
    (lambda t: (t[0], t[1], t[2][:-1].contiguous(), t[3]), "value_cache shape must equal key_cache shape"),
    (lambda t: t[:3] + (t[3].long(),), "block_table must be INT32"),
    (lambda t: t[:3] + (t[3].view(-1),), "block_table must be [1, max_pages]"),
    (lambda t: (t[0].cpu(),) + t[1:], "query must be a CUDA tensor"),
    (lambda t: (t[0].transpose(0, 1).contiguous().transpose(0, 1),) + t[1:], "all inputs must be contiguous"),
])
def test_fail_closed_input_gates(adapter, cuda_device, mutate, message):
    _, inputs = _inputs(cuda_device)
    qd, kd, vd, td = mutate(inputs)
    with pytest.raises(RuntimeError, match=message.replace("[", r"\[").replace("]", r"\]")):
        torch.ops.trianglemix_reference.triangle_paged_sparse_attention(qd, kd, vd, td, 0, 1300, 1300,
                                                                        SCALE)


@pytest.mark.parametrize("qs,seq,prompt,scale,message", [
    (1, 1300, 1300, SCALE, "query_start \\+ Tq == seq_len"),
    (0, 1300, 1299, SCALE, "invalid query_start/seq_len/prompt_len/scale"),
    (0, 1300, 1300, 0.0, "invalid query_start/seq_len/prompt_len/scale"),
    (0, 1300, 1300, float("inf"), "invalid query_start/seq_len/prompt_len/scale"),
])
def test_fail_closed_attribute_gates(adapter, cuda_device, qs, seq, prompt, scale, message):
    _, (qd, kd, vd, td) = _inputs(cuda_device)
    with pytest.raises(RuntimeError, match=message):
        torch.ops.trianglemix_reference.triangle_paged_sparse_attention(qd, kd, vd, td, qs, seq, prompt,
                                                                        scale)


def test_short_block_table_rejected(adapter, cuda_device):
    _, (qd, kd, vd, td) = _inputs(cuda_device)
    with pytest.raises(RuntimeError, match="block_table lacks logical pages"):
        torch.ops.trianglemix_reference.triangle_paged_sparse_attention(
            qd, kd, vd, td[:, :5].contiguous(), 0, 1300, 1300, SCALE)


def test_out_checks(adapter, cuda_device):
    _, (qd, kd, vd, td) = _inputs(cuda_device)
    op = torch.ops.trianglemix.triangle_paged_sparse_attention.out
    with pytest.raises(RuntimeError, match="out must be BF16"):
        op(qd, kd, vd, td, 0, 1300, 1300, SCALE, out=torch.empty_like(qd, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="out shape must exactly match query"):
        op(qd, kd, vd, td, 0, 1300, 1300, SCALE, out=torch.empty_like(qd)[:-1])
    with pytest.raises(RuntimeError, match="out must be contiguous"):
        op(qd, kd, vd, td, 0, 1300, 1300, SCALE,
           out=torch.empty(32, 1300, 128, dtype=torch.bfloat16, device=cuda_device).transpose(0, 1))
    with pytest.raises(RuntimeError):
        op(qd, kd, vd, td, 0, 1300, 1300, SCALE, out=qd)  # aliases the query
    with pytest.raises(RuntimeError, match="out must be a CUDA tensor"):
        op(qd, kd, vd, td, 0, 1300, 1300, SCALE, out=torch.empty_like(qd, device="cpu"))
