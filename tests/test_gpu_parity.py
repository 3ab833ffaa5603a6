"""Parity of the sm_100a kernel (through the C ABI) with the CPU oracle.

Tolerance (BASELINE): bf16 output within max-abs 2e-2 and mean-abs 2e-3 of
the fp32 oracle; the visited key set must match bit-exactly.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_helpers import MAX_ABS, MEAN_ABS, assert_close, run_cabi, workspace_for
from inputs import SCALE, baseline_inputs, inputs_digest, reference_case_inputs
from oracle.triangle_oracle import count_pairs, oracle_attention, visited_bitmap

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_cases.json").read_text())
OUTS = np.load(GOLDEN / "reference_cases.npz")


@pytest.mark.parametrize("case", META["cases"], ids=[c["name"] for c in META["cases"]])
def test_reference_correctness_matrix(tm, cuda_device, case):
    """The reference's 18 NPU correctness cases (npu_v2_correctness.py:51-216)."""
    q, k, v, table = reference_case_inputs(case["query_start"], case["query_tokens"],
                                           case["seq_len"], case["seed"])
    assert inputs_digest(q, k, v, table) == case["digest"]
    out = run_cabi(tm, q, k, v, table, case["query_start"], case["seq_len"], case["prompt_len"],
                   cuda_device)
    golden = torch.from_numpy(OUTS[case["name"]])
    assert_close(out[case["rows"]], golden, f"{case['name']} vs reference fixture")
    ref = oracle_attention(q, k, v, table, case["query_start"], case["seq_len"], case["prompt_len"], SCALE)
    assert_close(out, ref, f"{case['name']} vs oracle")


def test_shared_softmax_sentinel(tm, cuda_device):
    """Sink and window share one softmax: ~1.138, never the two-softmax 11."""
    s = META["sentinels"]["shared_softmax"]
    table = torch.tensor([s["table"]], dtype=torch.int32)
    k = torch.zeros(s["pages"], 128, 8, 128, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    flat = []
    for tok in range(522):
        page, off = divmod(tok, 128)
        flat.append((s["table"][page], off))
    for tok, (p, o) in enumerate(flat):
        v[p, o] = 10.0 if tok < 8 else (1000.0 if tok == 8 else 1.0)
    q = torch.zeros(1, 32, 128, dtype=torch.bfloat16)
    out = run_cabi(tm, q, k, v, table, 521, 522, 2048, cuda_device).float()
    assert abs(float(out[0, 0, 0]) - s["joint_expected"]) <= 0.04
    assert abs(float(out[0, 0, 0]) - s["value"]) <= 0.04
    assert abs(float(out[0, 0, 0]) - s["forbidden"]) >= 1.0
    assert float((out - out[0, 0, 0]).abs().max()) <= 0.04


def test_gqa_sentinel(tm, cuda_device):
    """Query head h reads kv head h // 4 (reference npu_v2_correctness.py:476-523)."""
    gen = torch.Generator().manual_seed(2202)
    perm = torch.randperm(4, generator=gen)
    table = perm[:1].to(torch.int32).view(1, 1)
    k = torch.zeros(4, 128, 8, 128, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    for h in range(8):
        v[int(table[0, 0]), 0, h] = float(h + 1)
    q = torch.zeros(1, 32, 128, dtype=torch.bfloat16)
    out = run_cabi(tm, q, k, v, table, 0, 1, 1024, cuda_device).float()
    expected = torch.tensor([float(h // 4 + 1) for h in range(32)])
    assert float((out[0, :, 0] - expected).abs().max()) <= 0.01


@pytest.mark.parametrize("seq", [4096])
def test_config0_one_chunk(tm, cuda_device, seq):
    """N=4096 one chunk, N(0,1) bf16, seed 0, 32 of 64 pages."""
    q, k, v, table = baseline_inputs(seq, seq, seed=0)
    out = run_cabi(tm, q, k, v, table, 0, seq, seq, cuda_device)
    ref = oracle_attention(q, k, v, table, 0, seq, seq, SCALE)
    assert_close(out, ref, "config 0")


@pytest.mark.parametrize("prompt,chunk", [(2869, 512), (8320, 2048)])
def test_chunked_prefill(tm, cuda_device, prompt, chunk):
    """every chunk attends all cached KV; prompt_len is final."""
    q_all, k, v, table = baseline_inputs(prompt, prompt, seed=1)
    for start in range(0, prompt, chunk):
        end = min(prompt, start + chunk)
        q = q_all[start:end].contiguous()
        out = run_cabi(tm, q, k, v, table, start, end, prompt, cuda_device)
        ref = oracle_attention(q, k, v, table, start, end, prompt, SCALE)
        assert_close(out, ref, f"chunk [{start},{end}) of {prompt}")


@pytest.mark.parametrize("seq", [16384])
def test_long_context_split_tail(tm, cuda_device, seq):
    """BASELINE config 3 shape: 8192 query rows at N=16K; tail blocks are split."""
    tq = 8192
    plan = tm._native.make_plan(tq, seq - tq, seq, seq, 8, 0, SCALE)
    assert plan.workspace_bytes > 0, "expected split dense-tail items"
    q, k, v, table = baseline_inputs(tq, seq, seed=3)
    out = run_cabi(tm, q, k, v, table, seq - tq, seq, seq, cuda_device)
    ref = oracle_attention(q, k, v, table, seq - tq, seq, seq, SCALE)
    assert_close(out, ref, "N=16K")


@pytest.mark.parametrize("query_start,tq,seq,prompt", [
    (0, 1100, 1100, 1100),      # prefix + sparse + tail
    (250, 5, 255, 2048),        # ragged dense prefix
    (519, 4, 523, 2048),        # sparse_begin crossing
    (700, 33, 733, 2048),       # ragged sparse
    (0, 2048, 2048, 2048),
    (1536, 512, 2048, 8320),    # intermediate chunk, no tail
    (3000, 1096, 4096, 4096),   # unaligned chunk start reaching the tail
    (1088, 92, 1180, 4000),     # composite tile whose band edge passes seq_len
])
def test_visited_key_set_bit_exact(tm, cuda_device, query_start, tq, seq, prompt):
    """Keys entering each (row, head) softmax equal the reference key set exactly."""
    q, k, v, table = baseline_inputs(tq, seq, seed=5)
    out, bitmap, tiles = run_cabi(tm, q, k, v, table, query_start, seq, prompt, cuda_device,
                                  visited=True)
    got = bitmap.numpy().view(np.uint32).reshape(tq * 32, -1)
    want = visited_bitmap(tq, 32, query_start, seq, prompt)
    mismatch = np.nonzero((got != want).any(axis=1))[0]
    assert mismatch.size == 0, f"{mismatch.size} rows differ, first row {mismatch[:4]}"
    # Loaded tiles equal the plan; keys loaded per row stay within 64-key rounding.
    plan = tm._native.make_plan(tq, query_start, seq, prompt, 8, 0, SCALE)
    n_tiles = n_keys = 0
    for i in range(plan.total_items):
        it = tm._native.plan_item(plan, i)
        for t in range(it.tile_begin, it.tile_end):
            _, w, _, _ = tm._native.plan_tile(plan, it.block, t)
            n_tiles += 1
            n_keys += w
    assert int(tiles[0]) == n_tiles and int(tiles[1]) == n_keys
    assert count_pairs(query_start, tq, seq, prompt) == int(np.unpackbits(
        want[::32].view(np.uint8)).sum())
    ref = oracle_attention(q, k, v, table, query_start, seq, prompt, SCALE)
    assert_close(out, ref, "visit-mode output")


@pytest.mark.parametrize("query_start,tq,seq,prompt", [
    (0, 1100, 1100, 1100),      # one chunk: the last page is written up to key 1099
    (1088, 92, 1180, 4000),     # intermediate chunk: the last sparse block's
                                # composite tile reads its band edge [1152, 1216)
])
def test_unwritten_cache_slots_never_reach_the_output(tm, cuda_device, query_start, tq, seq,
                                                      prompt):
    """Cache slots at or beyond seq_len hold whatever the serving engine left
    there; here NaN in K and V.  The kernel masks their scores and zeroes
    their values in shared memory, so the output equals the oracle's on the
    clean cache (and has no NaN)."""
    q, k, v, table = baseline_inputs(tq, seq, seed=9)
    ref = oracle_attention(q, k, v, table, query_start, seq, prompt, SCALE)
    k_bad, v_bad = k.clone(), v.clone()
    pages = table[0].tolist()
    for key in range(seq, len(pages) * 128):
        k_bad[pages[key // 128], key % 128] = float("nan")
        v_bad[pages[key // 128], key % 128] = float("nan")
    out = run_cabi(tm, q, k_bad, v_bad, table, query_start, seq, prompt, cuda_device)
    assert not torch.isnan(out.float()).any()
    assert_close(out, ref, f"NaN beyond seq_len {seq}")


def test_page_placement_invariance_bit_exact(tm, cuda_device):
    """Moving pages to other physical slots leaves the output bit-identical."""
    seq = 8192
    q, k, v, table = baseline_inputs(seq, seq, seed=11)
    out1 = run_cabi(tm, q, k, v, table, 0, seq, seq, cuda_device)
    gen = torch.Generator().manual_seed(12)
    perm = torch.randperm(k.shape[0], generator=gen)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    k2, v2 = k[perm].contiguous(), v[perm].contiguous()
    table2 = inv[table.long()].to(torch.int32)
    out2 = run_cabi(tm, q, k2, v2, table2, 0, seq, seq, cuda_device)
    assert torch.equal(out1.view(torch.int16), out2.view(torch.int16))
    out3 = run_cabi(tm, q, k, v, table, 0, seq, seq, cuda_device)
    assert torch.equal(out1.view(torch.int16), out3.view(torch.int16)), "not deterministic"


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_head_sharded_entry_point(tm, cuda_device, kv_heads):
    """tpsa_paged_attention_heads on a kv-head slice equals the full op's slice."""
    seq = 3000
    q, k, v, table = baseline_inputs(seq, seq, seed=21)
    full = run_cabi(tm, q, k, v, table, 0, seq, seq, cuda_device)
    for r in range(8 // kv_heads):
        h0, h1 = r * kv_heads, (r + 1) * kv_heads
        qs = q[:, 4 * h0:4 * h1].contiguous()
        ks, vs = k[:, :, h0:h1].contiguous(), v[:, :, h0:h1].contiguous()
        part = run_cabi(tm, qs, ks, vs, table, 0, seq, seq, cuda_device, kv_heads=kv_heads)
        d = (part.float() - full[:, 4 * h0:4 * h1].float()).abs()
        assert float(d.max()) <= MAX_ABS and float(d.mean()) <= MEAN_ABS / 4


def test_bad_page_is_flagged_not_faulted(tm, cuda_device):
    """An out-of-range physical page id reads zeros and sets the status bit."""
    seq = 512
    q, k, v, table = baseline_inputs(seq, seq, seed=31)
    bad = table.clone()
    bad[0, 2] = k.shape[0] + 5
    qd, kd, vd, td = (t.to(cuda_device) for t in (q, k, v, bad))
    out = torch.empty_like(qd)
    ws = workspace_for(tm, seq, 0, seq, seq, 8, cuda_device)
    tm._native.paged_attention(qd, kd, vd, td, out, 0, seq, seq, SCALE, workspace=ws)
    torch.cuda.synchronize()
    status = tm._native.device_status(0)
    assert status & tm._native.DEVICE_BAD_PAGE
    assert status & tm._native.DEVICE_WAIT_TIMEOUT == 0
    assert torch.isfinite(out.float()).all()
    assert tm._native.device_status(0) == 0  # reading cleared it


@pytest.mark.parametrize("spike_key", [200, 760])
def test_reference_moves_in_upper_half_of_tile(tm, cuda_device, spike_key):
    """A key whose score exceeds every earlier key's by far more than the
    lazy reference threshold (2^8 after scaling), in keys 64-127 of a tile
    that is not the first of its item: the softmax's reference max moves on
    that tile, and O and the row sum accumulated so far are rescaled (to
    zero here).  Every row that sees the key follows its value row; all rows
    are checked against the oracle."""
    seq = 1024
    gen = torch.Generator().manual_seed(31 + spike_key)
    pages = seq // 128
    table = torch.randperm(2 * pages, generator=gen)[:pages].to(torch.int32).view(1, -1)
    u = torch.randn(128, generator=gen)
    q = (u + 0.1 * torch.randn(seq, 32, 128, generator=gen)).to(torch.bfloat16)
    k = (0.1 * torch.randn(2 * pages, 128, 8, 128, generator=gen)).to(torch.bfloat16)
    v = torch.randn(2 * pages, 128, 8, 128, generator=gen).to(torch.bfloat16)
    page, off = divmod(spike_key, 128)
    assert off % 128 >= 64, "the spike must sit in keys 64-127 of a page-aligned tile"
    k[table[0, page], off] = (8.0 * u / u.norm() * 11.3).to(torch.bfloat16)
    out = run_cabi(tm, q, k, v, table, 0, seq, seq, cuda_device)
    ref = oracle_attention(q, k, v, table, 0, seq, seq, SCALE)
    assert_close(out, ref, f"spike at key {spike_key}")
    # The rows that see the spike follow its value row.
    row = spike_key + 10
    assert float((out[row].float() - v[table[0, page], off].float().repeat_interleave(4, 0)).abs().max()) < 0.05
