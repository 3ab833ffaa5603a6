"""Packed ragged batches (varlen) through the C ABI.

Semantics: the reference's packed-batch helper reference_attention_ragged_python
(operator/tests/triangle_v2_reference.py:437-487) computes a packed batch as
the batch-one operator applied to each request's slice of rows.  Every case
here checks each request's rows against the CPU oracle on that request alone
(same key sets, its own pages of the shared pool), within the parity
tolerance.
"""

from __future__ import annotations

import pytest
import torch

from gpu_helpers import assert_close, run_cabi
from inputs import SCALE, varlen_inputs
from oracle.triangle_oracle import oracle_attention

pytestmark = pytest.mark.gpu


def _run_varlen(tm, dev, q, k, v, tables, cu, seq_lens, prompt_lens):
    out = torch.full_like(q, float("nan"), device=dev)
    tm._native.paged_attention_varlen(q.to(dev), k.to(dev), v.to(dev), tables.to(dev), out, cu,
                                      seq_lens, prompt_lens, SCALE)
    torch.cuda.synchronize(dev)
    assert tm._native.device_status(dev.index or 0) == 0
    return out.cpu()


def _check_against_oracle(out, q, k, v, per_request, cu, specs, what):
    for i, (rows, seq, prompt) in enumerate(specs):
        got = out[cu[i]:cu[i + 1]]
        ref = oracle_attention(q[cu[i]:cu[i + 1]], k, v, per_request[i], seq - rows, seq, prompt,
                               SCALE)
        assert_close(got, ref.to(torch.bfloat16), f"{what} request {i} ({rows}/{seq}/{prompt})")


# (query rows, seq_len, prompt_len): ragged last blocks (37, 65, 200),
# chunked requests (rows < seq_len), prompt_len > seq_len (sparse tail
# moved past the chunk), requests that cross 521 and the dense tail, one
# exactly block-aligned request.
MIXED = [
    (37, 37, 37),
    (200, 900, 900),
    (64, 1024, 4096),
    (530, 530, 530),
    (65, 2113, 2113),
    (1000, 1700, 2500),
    (128, 128, 128),
]


def test_varlen_mixed_batch_matches_oracle_per_request(tm, cuda_device):
    q, k, v, tables, per_request, cu = varlen_inputs(MIXED, seed=21)
    out = _run_varlen(tm, cuda_device, q, k, v, tables, cu, [s for _, s, _ in MIXED],
                      [p for _, _, p in MIXED])
    _check_against_oracle(out, q, k, v, per_request, cu, MIXED, "mixed")


def test_varlen_more_than_one_launch(tm, cuda_device):
    """19 requests: launches of 16 and 3 requests reuse one workspace."""
    gen = torch.Generator().manual_seed(5)
    specs = []
    for _ in range(19):
        seq = int(torch.randint(40, 1400, (1,), generator=gen))
        rows = int(torch.randint(1, seq + 1, (1,), generator=gen))
        specs.append((rows, seq, seq + int(torch.randint(0, 300, (1,), generator=gen))))
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=22)
    out = _run_varlen(tm, cuda_device, q, k, v, tables, cu, [s for _, s, _ in specs],
                      [p for _, _, p in specs])
    _check_against_oracle(out, q, k, v, per_request, cu, specs, "19 requests")


def test_varlen_split_kv_requests(tm, cuda_device):
    """Long dense tails split across items inside a varlen launch."""
    specs = [(1024, 12288, 12288), (256, 9000, 9000), (64, 3000, 3000)]
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=23)
    seq_lens, prompt_lens = [s for _, s, _ in specs], [p for _, _, p in specs]
    assert tm._native.varlen_workspace_size(cu, seq_lens, prompt_lens) > 2048, \
        "the batch must use split-KV partial slots"
    out = _run_varlen(tm, cuda_device, q, k, v, tables, cu, seq_lens, prompt_lens)
    _check_against_oracle(out, q, k, v, per_request, cu, specs, "split")


def test_varlen_equals_batch_one_calls(tm, cuda_device):
    """Each request's rows equal a batch-one call on the same inputs."""
    specs = [(300, 300, 300), (96, 777, 777), (513, 1500, 1600)]
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=24)
    out = _run_varlen(tm, cuda_device, q, k, v, tables, cu, [s for _, s, _ in specs],
                      [p for _, _, p in specs])
    for i, (rows, seq, prompt) in enumerate(specs):
        one = run_cabi(tm, q[cu[i]:cu[i + 1]], k, v, per_request[i], seq - rows, seq, prompt,
                       cuda_device)
        assert_close(out[cu[i]:cu[i + 1]], one, f"request {i} vs batch-one")


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_varlen_heads_packs_layer_slices(tm, cuda_device, kv_heads):
    """tpsa_paged_attention_varlen_heads: one rank's kv-head slice of several
    layers, their caches in one page pool and each layer's block table offset
    to its own pages, in one launch; every layer's rows checked against the
    oracle on that layer alone."""
    layers, rows, seq = 8 // kv_heads, 700, 1800
    gen = torch.Generator().manual_seed(40 + kv_heads)
    logical = (seq + 127) // 128
    qs, ks, vs, tables = [], [], [], []
    for _ in range(layers):
        qs.append(torch.randn(rows, 4 * kv_heads, 128, generator=gen).to(torch.bfloat16))
        ks.append(torch.randn(2 * logical, 128, kv_heads, 128, generator=gen).to(torch.bfloat16))
        vs.append(torch.randn(2 * logical, 128, kv_heads, 128, generator=gen).to(torch.bfloat16))
        tables.append(torch.randperm(2 * logical, generator=gen)[:logical].to(torch.int32))
    pool_k, pool_v = torch.cat(ks), torch.cat(vs)
    packed_tables = torch.stack([t + j * 2 * logical for j, t in enumerate(tables)])
    cu = [rows * j for j in range(layers + 1)]
    seq_lens = [seq] * layers
    q = torch.cat(qs).to(cuda_device)
    out = torch.full_like(q, float("nan"))
    tm._native.paged_attention_varlen(q, pool_k.to(cuda_device), pool_v.to(cuda_device),
                                      packed_tables.to(cuda_device), out, cu, seq_lens, seq_lens,
                                      SCALE, kv_heads=kv_heads)
    torch.cuda.synchronize(cuda_device)
    assert tm._native.device_status(cuda_device.index or 0) == 0
    out = out.cpu()
    for j in range(layers):
        ref = oracle_attention(qs[j], ks[j], vs[j], tables[j].view(1, -1), seq - rows, seq, seq,
                               SCALE)
        assert_close(out[cu[j]:cu[j + 1]], ref.to(torch.bfloat16), f"layer {j} of {layers}")


def test_varlen_unwritten_slots_never_reach_the_output(tm, cuda_device):
    """Each request's cache slots at or beyond its seq_len, and the pool's
    unused pages, hold NaN in K and V; every request still matches the
    oracle on the clean pool (one request's last sparse block runs a
    composite tile whose band edge passes its seq_len)."""
    specs = MIXED + [(92, 1180, 4000)]
    q, k, v, tables, per_request, cu = varlen_inputs(specs, seed=23)
    k_bad, v_bad = k.clone(), v.clone()
    used = set()
    for (_, seq, _), row in zip(specs, per_request):
        pages = row[0].tolist()
        used.update(pages)
        for key in range(seq, len(pages) * 128):
            k_bad[pages[key // 128], key % 128] = float("nan")
            v_bad[pages[key // 128], key % 128] = float("nan")
    for page in set(range(k.shape[0])) - used:
        k_bad[page] = float("nan")
        v_bad[page] = float("nan")
    out = _run_varlen(tm, cuda_device, q, k_bad, v_bad, tables, cu, [s for _, s, _ in specs],
                      [p for _, _, p in specs])
    assert not torch.isnan(out.float()).any()
    _check_against_oracle(out, q, k, v, per_request, cu, specs, "NaN beyond seq_len")
