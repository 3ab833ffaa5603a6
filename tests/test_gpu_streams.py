"""Control words across streams and CUDA graph capture.

A launch's scheduler and split counters live in a library-owned control
block of the launching stream; the last CTA of each launch zeroes the block
on its way out, so no memset precedes the kernel.  A launch captured into a
CUDA graph keeps its counters in its workspace instead (cleared by a memset
node of the graph), because a graph may be replayed on any stream.

These tests run launches on two streams back to back with no
synchronisation between them, and one captured launch replayed twice, and
compare every output with a launch of the same inputs on the default stream.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import run_cabi, workspace_for
from inputs import SCALE, baseline_inputs

pytestmark = pytest.mark.gpu

# (query tokens, seq_len, seed); the 16384-token context splits its
# dense-tail blocks, so its launches also use the split counters.
CASES = ((2048, 4096, 21), (4096, 16384, 22))


def _device_inputs(dev, tq, seq, seed):
    q, k, v, table = baseline_inputs(tq, seq, seed)
    return (q, k, v, table), tuple(x.to(dev) for x in (q, k, v, table))


def test_two_streams_back_to_back(tm, cuda_device):
    dev = cuda_device
    cases = []
    for tq, seq, seed in CASES:
        host, dev_in = _device_inputs(dev, tq, seq, seed)
        q0 = seq - tq
        expected = run_cabi(tm, *host, q0, seq, seq, dev)
        cases.append((dev_in, q0, seq, expected))
    streams = [torch.cuda.Stream(dev) for _ in cases]
    reps = 3
    outs = [[torch.full_like(c[0][0], float("nan")) for _ in range(reps)] for c in cases]
    spaces = [workspace_for(tm, c[0][0].shape[0], c[1], c[2], c[2], 8, dev) for c in cases]
    torch.cuda.synchronize(dev)
    for r in range(reps):
        for i, ((qd, kd, vd, td), q0, seq, _) in enumerate(cases):
            tm._native.paged_attention(qd, kd, vd, td, outs[i][r], q0, seq, seq, SCALE,
                                       workspace=spaces[i], stream=streams[i].cuda_stream)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    for i, c in enumerate(cases):
        for r in range(reps):
            assert torch.equal(outs[i][r].cpu(), c[3]), f"stream {i} launch {r}"


def test_captured_launch_replays(tm, cuda_device):
    dev = cuda_device
    tq, seq, seed = CASES[1]
    q0 = seq - tq
    host, (qd, kd, vd, td) = _device_inputs(dev, tq, seq, seed)
    expected = run_cabi(tm, *host, q0, seq, seq, dev)
    out = torch.empty_like(qd)
    ws = workspace_for(tm, tq, q0, seq, seq, 8, dev)
    side = torch.cuda.Stream(dev)
    # One eager launch on the side stream first: its control block is then in
    # use when the capture runs, and the captured launch must not take it.
    tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, workspace=ws,
                               stream=side.cuda_stream)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, workspace=ws,
                                   stream=side.cuda_stream)
    for _ in range(2):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize(dev)
        assert torch.equal(out.cpu(), expected)
        # An eager launch on the capture stream between replays.
        tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, workspace=ws,
                                   stream=side.cuda_stream)
        torch.cuda.synchronize(dev)
        assert torch.equal(out.cpu(), expected)
    assert tm._native.device_status(dev.index or 0) == 0
