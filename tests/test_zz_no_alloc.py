"""The entry point that allocates nothing (tpsa_paged_attention_static_scratch).

It runs through the C ABI, twice in a row, on two different split-KV shapes,
so the second call finds the first call's contents in the shared static
scratch. Each output is compared with tpsa_paged_attention on the same
inputs, using a caller workspace, within the parity tolerance. This file
is collected last so that the shared scratch has seen every earlier test's
launches, and it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close, workspace_for
from inputs import SCALE, baseline_inputs

pytestmark = pytest.mark.gpu

# (query_tokens, seq_len): the last 4096-token chunk of an 8192-token prompt
# and the last 2048-token chunk of an 8320-token prompt; both split their
# dense-tail blocks, so the scratch holds partial slots as well as control
# words.
CASES = ((4096, 8192, 11), (2048, 8320, 12))


def _run(tm, dev, q, k, v, table, q0, seq, *, static):
    qd, kd, vd, td = (t.to(dev) for t in (q, k, v, table))
    out = torch.full_like(qd, float("nan"))
    if static:
        # Nothing is allocated through torch's allocator by the call.
        torch.cuda.synchronize(dev)
        before = torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)
        tm._native.paged_attention_static_scratch(qd, kd, vd, td, out, q0, seq, seq, SCALE)
        torch.cuda.synchronize(dev)
        assert (torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)) == before
    else:
        ws = workspace_for(tm, q.shape[0], q0, seq, seq, 8, dev)
        tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, workspace=ws)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    return out.cpu()


def test_static_scratch_matches_workspace_entry_point_twice(tm, cuda_device):
    inputs, expected = [], []
    for tq, seq, seed in CASES:
        q0 = seq - tq
        plan = tm._native.make_plan(tq, q0, seq, seq, 8, 0, SCALE)
        assert plan.workspace_bytes > 2048, "case must use split-KV partial slots"
        x = baseline_inputs(tq, seq, seed)
        inputs.append((x, q0, seq))
        expected.append(_run(tm, cuda_device, *x, q0, seq, static=False))
    # Two calls in a row through the entry point that allocates nothing.
    got = [_run(tm, cuda_device, *x, q0, seq, static=True) for x, q0, seq in inputs]
    for (tq, seq, _), g, e in zip(CASES, got, expected):
        assert_close(g, e, f"static scratch tq={tq} seq={seq}")
