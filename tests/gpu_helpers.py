"""Helpers for the GPU parity tests: launch through the C ABI and compare."""

from __future__ import annotations

import torch

from inputs import SCALE

MAX_ABS = 2e-2   # BASELINE tolerance on bf16 output vs the fp32 oracle
MEAN_ABS = 2e-3


def workspace_for(tm, query_tokens, query_start, seq_len, prompt_len, kv_heads, device):
    plan = tm._native.make_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, 0, SCALE)
    if plan.workspace_bytes == 0:
        return None
    return torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=device)


def run_cabi(tm, q, k, v, table, query_start, seq_len, prompt_len, device, *, scale=SCALE,
             kv_heads=None, visited=False):
    """Run the kernel through libtpsa's C ABI; returns (out_cpu, bitmap, tiles)."""
    qd, kd, vd, td = (t.to(device) for t in (q, k, v, table))
    out = torch.empty_like(qd)
    kvh = kv_heads or k.shape[2]
    ws = workspace_for(tm, q.shape[0], query_start, seq_len, prompt_len, kvh, device)
    bitmap = tiles = None
    if visited:
        words = (seq_len + 31) // 32
        bitmap = torch.zeros(q.shape[0] * q.shape[1] * words, dtype=torch.int32, device=device)
        tiles = torch.zeros(2, dtype=torch.int64, device=device)
    tm._native.paged_attention(qd, kd, vd, td, out, query_start, seq_len, prompt_len, scale,
                               kv_heads=kv_heads, workspace=ws, visited=bitmap, tile_counter=tiles)
    torch.cuda.synchronize(device)
    status = tm._native.device_status(device.index or 0)
    assert status == 0, f"device status word {status:#x}"
    if visited:
        return out.cpu(), bitmap.cpu(), tiles.cpu()
    return out.cpu()


def assert_close(actual, expected, what=""):
    a = actual.float()
    e = expected.float()
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    d = (a - e).abs()
    mx, mean = float(d.max()), float(d.mean())
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"{what}: max_abs {mx:.4g} mean_abs {mean:.4g}"
    return mx, mean
