"""The all-dense control (tpsa_paged_attention_dense) against a plain
PyTorch fp32 causal attention over the same paged context.

The control is the kernel with no sparse rows: row query_start + i of the
chunk reads keys [0, query_start + i].  It is the dense comparator of the
chunked-prefill crossover, so its numerics are held to the same tolerance as
the sparse path (max-abs 2e-2, mean-abs 2e-3 on bf16 output).
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close, workspace_for
from inputs import PAGE, SCALE, baseline_inputs

pytestmark = pytest.mark.gpu


def torch_causal_fp32(q, k, v, table, q0, seq):
    """fp32 causal GQA attention of the chunk over the gathered context."""
    pages = table[0, :(seq + PAGE - 1) // PAGE].long()
    kc = k.index_select(0, pages).reshape(-1, k.shape[2], k.shape[3])[:seq].float()
    vc = v.index_select(0, pages).reshape(-1, v.shape[2], v.shape[3])[:seq].float()
    tq, hq, _ = q.shape
    group = hq // k.shape[2]
    rows = torch.arange(q0, q0 + tq, device=q.device)[:, None]
    keys = torch.arange(seq, device=q.device)[None, :]
    visible = keys <= rows
    out = torch.empty(tq, hq, q.shape[2], dtype=torch.float32, device=q.device)
    for h in range(hq):
        s = (q[:, h].float() @ kc[:, h // group].T) * SCALE
        s = s.masked_fill(~visible, float("-inf"))
        out[:, h] = torch.softmax(s, dim=-1) @ vc[:, h // group]
    return out


@pytest.mark.parametrize("tq,seq", [(1024, 1024), (512, 3000), (2048, 8320), (512, 8192),
                                    (8192, 8192)])
def test_dense_control_matches_torch_fp32(tm, cuda_device, tq, seq):
    dev = cuda_device
    q0 = seq - tq
    q, k, v, table = (t.to(dev) for t in baseline_inputs(tq, seq, seed=31))
    out = torch.full_like(q, float("nan"))
    tm._native.paged_attention_dense(q, k, v, table, out, q0, seq, SCALE)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    ref = torch_causal_fp32(q, k, v, table, q0, seq)
    assert_close(out.cpu(), ref.cpu(), f"dense control tq={tq} seq={seq}")


def test_dense_control_differs_from_trianglemix_only_on_sparse_rows(tm, cuda_device):
    """Rows outside the sparse middle (the dense prefix q < 521 and the last
    128 prompt rows) have the same key set in both modes.  The dense prefix
    runs the same tiles in the same order, so it is bit-identical; the
    TriangleMix plan splits the last two blocks into split-KV pieces, so the
    tail agrees within the tolerance.  Sparse rows differ."""
    dev = cuda_device
    tq = seq = 2048
    q, k, v, table = (t.to(dev) for t in baseline_inputs(tq, seq, seed=32))
    dense, sparse = torch.empty_like(q), torch.empty_like(q)
    tm._native.paged_attention_dense(q, k, v, table, dense, 0, seq, SCALE)
    tm._native.paged_attention(q, k, v, table, sparse, 0, seq, seq, SCALE,
                               workspace=workspace_for(tm, tq, 0, seq, seq, 8, dev))
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    assert torch.equal(dense[:521], sparse[:521])
    assert_close(dense[seq - 128:].cpu(), sparse[seq - 128:].float().cpu(), "dense tail rows")
    assert not torch.equal(dense[600:seq - 128], sparse[600:seq - 128])
