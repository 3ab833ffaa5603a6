"""Parity on the exact inputs of every configuration bench.py times.

Each case runs bench.py's own input recipe (``bench.make_inputs`` /
``bench.make_batch_inputs``) through the C ABI at full size and compares a
seeded sample of query rows with the oracle's per-row evaluation
(``oracle_attention_rowwise``, the method of the reference oracle
operator/tests/triangle_v2_reference.py:490-587).  The sample covers the
dense prefix, the sparse band, every block boundary kind and every row of
the dense tail blocks, whose split-KV pieces are merged in the kernel, so a
wrong piece or merge shows in the sampled tail rows.  Tolerance as
everywhere: max-abs 2e-2, mean-abs 2e-3 (reference npu_v2_correctness.py
uses 5e-2 / 5e-3).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from gpu_helpers import assert_close, workspace_for
from inputs import SCALE
from oracle.triangle_oracle import oracle_attention_rowwise, prepare_logical_kv, visited_bitmap

pytestmark = pytest.mark.gpu

SPARSE_BEGIN = 521
TAIL = 128


def sample_rows(tq: int, query_start: int, prompt: int, n: int = 256, seed: int = 0) -> list[int]:
    """Rows of the chunk to check: every dense-tail row, the rows at each
    block edge near the sparse boundaries, and a seeded uniform sample."""
    rng = np.random.default_rng(seed)
    rows = set()
    tail0 = max(0, prompt - TAIL - query_start)
    rows.update(range(min(tail0, tq), tq))  # the whole dense tail (all split pieces)
    for q in (SPARSE_BEGIN - 1, SPARSE_BEGIN, SPARSE_BEGIN + 63, prompt - TAIL - 1):
        r = q - query_start
        if 0 <= r < tq:
            rows.add(r)
    rows.update((0, tq - 1))
    rows.update(int(r) for r in rng.integers(0, tq, size=n))
    return sorted(rows)


def check_rows(out, q, k, v, table, query_start, seq, prompt, rows, what):
    lkv = prepare_logical_kv(k, v, table, seq)
    ref = oracle_attention_rowwise(q, k, v, table, query_start, seq, prompt, SCALE, rows=rows,
                                   logical_kv=lkv)
    idx = torch.tensor(rows, dtype=torch.int64)
    return assert_close(out.index_select(0, idx), ref.index_select(0, idx), what)


def run_layer(tm, dev, q, k, v, table, query_start, seq, prompt):
    qd, kd, vd, td = (t.to(dev) for t in (q, k, v, table))
    out = torch.empty_like(qd)
    ws = workspace_for(tm, q.shape[0], query_start, seq, prompt, 8, dev)
    tm._native.paged_attention(qd, kd, vd, td, out, query_start, seq, prompt, SCALE, workspace=ws)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    return out.cpu()


@pytest.mark.parametrize("seq,tq", [(8192, 8192), (32768, 8192), (65536, 8192), (131072, 8192)],
                         ids=["prefill_8k", "32k_q8k", "64k_q8k", "128k_q8k"])
def test_bench_layer_matches_oracle(tm, cuda_device, seq, tq):
    """bench.py's timed layer (seed 0, random table over 2x the pages)."""
    q, k, v, table = bench.make_inputs(tq, seq, 0)
    q0 = seq - tq
    plan = tm._native.make_plan(tq, q0, seq, seq, 8, 0, SCALE)
    if seq >= 32768:
        # the plans the bench times at long contexts cut the tail into pieces
        assert plan.workspace_bytes > 0, "expected split dense-tail items"
    out = run_layer(tm, cuda_device, q, k, v, table, q0, seq, seq)
    assert torch.isfinite(out.float()).all()
    rows = sample_rows(tq, q0, seq)
    check_rows(out, q, k, v, table, q0, seq, seq, rows, f"bench layer {seq}/{tq}")


@pytest.mark.parametrize("seq,world,rank", [(8192, 8, 0), (8192, 4, 1), (32768, 8, 7),
                                             (32768, 2, 1)],
                         ids=["8k_1head", "8k_2heads", "32k_1head", "32k_4heads"])
def test_bench_head_slice_matches_oracle(tm, cuda_device, seq, world, rank):
    """One rank's KV-head slice of the bench layer (bench.py at --gpus N):
    the launches with few items per CTA, whose split pieces merge
    cooperatively (each piece a slice of the rows), checked on the sampled
    rows, the whole dense tail included."""
    tq = 8192
    q0 = seq - tq
    heads = 8 // world
    q, k, v, table = bench.make_inputs(tq, seq, 0, rank, world)
    plan = tm._native.make_plan(tq, q0, seq, seq, heads, 0, SCALE)
    assert plan.workspace_bytes > 2048, "expected split dense-tail items"
    dev = cuda_device
    qd, kd, vd, td = (t.to(dev) for t in (q, k, v, table))
    out = torch.empty_like(qd)
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=dev)
    tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, kv_heads=heads,
                               workspace=ws)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    out = out.cpu()
    assert torch.isfinite(out.float()).all()
    rows = sample_rows(tq, q0, seq)
    check_rows(out, q, k, v, table, q0, seq, seq, rows, f"head slice {seq} rank {rank}/{world}")


def test_bench_32k_visited_set_bit_exact(tm, cuda_device):
    """Visited keys of the 32K / 8K-chunk plan (split tail) equal the key sets."""
    seq, tq = 32768, 8192
    q0 = seq - tq
    q, k, v, table = bench.make_inputs(tq, seq, 0)
    dev = cuda_device
    qd, kd, vd, td = (t.to(dev) for t in (q, k, v, table))
    out = torch.empty_like(qd)
    words = (seq + 31) // 32
    bitmap = torch.zeros(tq * 32 * words, dtype=torch.int32, device=dev)
    tiles = torch.zeros(2, dtype=torch.int64, device=dev)
    ws = workspace_for(tm, tq, q0, seq, seq, 8, dev)
    tm._native.paged_attention(qd, kd, vd, td, out, q0, seq, seq, SCALE, workspace=ws,
                               visited=bitmap, tile_counter=tiles)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    want = torch.from_numpy(visited_bitmap(tq, 1, q0, seq, seq).view(np.int32)).to(dev)
    got = bitmap.view(tq, 32, words)
    bad = (got != want[:, None, :]).any(dim=2).any(dim=1)
    assert int(bad.sum()) == 0, f"{int(bad.sum())} rows differ, first {bad.nonzero()[:4].tolist()}"
    plan = tm._native.make_plan(tq, q0, seq, seq, 8, 0, SCALE)
    n_tiles = n_keys = 0
    for i in range(plan.total_items):
        it = tm._native.plan_item(plan, i)
        for t in range(it.tile_begin, it.tile_end):
            _, w, _, _ = tm._native.plan_tile(plan, it.block, t)
            n_tiles += 1
            n_keys += w
    assert int(tiles[0]) == n_tiles and int(tiles[1]) == n_keys


@pytest.mark.parametrize("batch", [4, 16])
def test_bench_batch_matches_oracle_per_request(tm, cuda_device, batch):
    """bench.py --batch B (config 4): the packed varlen launch, per request."""
    lens, cu, q, k, v, tables = bench.make_batch_inputs(batch)
    dev = cuda_device
    out = torch.full_like(q, float("nan"), device=dev)
    tm._native.paged_attention_varlen(q.to(dev), k.to(dev), v.to(dev), tables.to(dev), out, cu,
                                      lens, lens, SCALE)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    out = out.cpu()
    assert torch.isfinite(out.float()).all()
    for i, n in enumerate(lens):
        pages = (n + 127) // 128
        table = tables[i:i + 1, :pages].contiguous()
        rows = sample_rows(n, 0, n, n=64, seed=i)
        check_rows(out[cu[i]:cu[i + 1]], q[cu[i]:cu[i + 1]], k, v, table, 0, n, n, rows,
                   f"batch {batch} request {i} (len {n})")
