"""A bounded wait of the kernel made to run out, on the GPU.

The test hook tpsa_debug_wait_probe puts the next launch in probe mode: in
every CTA the scheduler waits on a barrier that nothing arrives on, with a
200 us limit, before it claims any work.  The wait runs out, which sets the
CTA's abort flag and TPSA_DEVICE_WAIT_TIMEOUT; the producers, the MMA warp
and the softmax warps, all waiting for their first item record, leave
through their abort paths; TMEM is released at the common exit.  Nothing is
loaded, computed or stored, so the output keeps its fill.  The checks: the
status bit is set, reading the status clears it, and the next ordinary
launch in the same process matches the oracle.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close, run_cabi, workspace_for
from inputs import SCALE, baseline_inputs
from oracle.triangle_oracle import oracle_attention

pytestmark = pytest.mark.gpu

TPSA_DEVICE_WAIT_TIMEOUT = 0x1
PROBE_LIMIT_NS = 200_000


def test_probe_wait_runs_out_and_next_launch_is_correct(tm, cuda_device):
    tq = seq = 1024
    q, k, v, table = baseline_inputs(tq, seq, seed=21)
    dev = cuda_device
    assert tm._native.device_status(dev.index or 0) == 0
    qd, kd, vd, td = (t.to(dev) for t in (q, k, v, table))
    out = torch.full_like(qd, float("nan"))
    ws = workspace_for(tm, tq, 0, seq, seq, 8, dev)
    tm._native.debug_wait_probe(PROBE_LIMIT_NS)
    tm._native.paged_attention(qd, kd, vd, td, out, 0, seq, seq, SCALE, workspace=ws)
    torch.cuda.synchronize(dev)
    status = tm._native.device_status(dev.index or 0)
    assert status & TPSA_DEVICE_WAIT_TIMEOUT, f"status {status:#x}: the probe wait did not run out"
    assert status == TPSA_DEVICE_WAIT_TIMEOUT, f"unexpected status bits {status:#x}"
    # Reading the word cleared it.
    assert tm._native.device_status(dev.index or 0) == 0
    # No output store ran.
    assert torch.isnan(out.float()).all(), "probe launch wrote output rows"
    # The context is usable and the next launch (probe disarmed) is correct.
    got = run_cabi(tm, q, k, v, table, 0, seq, seq, dev)
    ref = oracle_attention(q, k, v, table, 0, seq, seq, SCALE)
    assert_close(got, ref, "launch after the probe")


def test_probe_is_one_shot_and_thread_local(tm, cuda_device):
    """Arming affects only the next launch of the arming thread; 0 disarms."""
    import threading

    tq = seq = 512
    q, k, v, table = baseline_inputs(tq, seq, seed=22)
    dev = cuda_device
    tm._native.debug_wait_probe(PROBE_LIMIT_NS)
    tm._native.debug_wait_probe(0)  # disarmed again
    first = run_cabi(tm, q, k, v, table, 0, seq, seq, dev)  # asserts status 0
    tm._native.debug_wait_probe(PROBE_LIMIT_NS)
    other = {}

    def run_elsewhere():
        other["out"] = run_cabi(tm, q, k, v, table, 0, seq, seq, dev)

    th = threading.Thread(target=run_elsewhere)
    th.start()
    th.join()
    assert torch.equal(other["out"], first), "another thread's launch saw the probe"
    tm._native.debug_wait_probe(0)
    assert torch.equal(run_cabi(tm, q, k, v, table, 0, seq, seq, dev), first)
