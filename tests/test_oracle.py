"""The CPU oracle, pinned against the reference's own oracle and known answers.

Fixtures in tests/golden were produced by importing the reference module
(operator/tests/triangle_v2_reference.py) in the build container.  Known
answers below restate the expectations of the reference's CPU tests
(operator/tests/test_triangle_v2_reference.py, test_project_contract.py,
test_query_span_contract.py, package/tests/test_planning_stats.py).
"""

from __future__ import annotations

import json
import random
from pathlib import Path

import numpy as np
import pytest
import torch

from inputs import SCALE, baseline_inputs, inputs_digest, reference_case_inputs
from oracle import triangle_oracle as o

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_cases.json").read_text())
OUTS = np.load(GOLDEN / "reference_cases.npz")
G = o.PRODUCTION


def test_intervals_match_reference_grid():
    grid = json.loads((GOLDEN / "intervals.json").read_text())
    assert len(grid) > 300
    for q, seq, prompt, ivs in grid:
        assert [list(x) for x in o.selected_intervals(q, seq, prompt)] == ivs, (q, seq, prompt)


def test_closed_form_mask_equals_intervals():
    for prompt in (600, 649, 700, 1024, 2048):
        for seq in (1, 300, 521, 522, 700, prompt):
            if seq > prompt:
                continue
            rows = np.arange(0, seq)
            keys = np.arange(0, seq + 40)
            m = o.visible_mask(rows, keys, seq, prompt)
            for q in rows:
                want = np.zeros(keys.size, dtype=bool)
                for b, e in o.selected_intervals(int(q), seq, prompt):
                    want[b:e] = True
                assert np.array_equal(m[q], want), (q, seq, prompt)


def test_sparse_begin_merge_and_gap():
    assert G.sparse_begin == 521
    assert o.selected_token_indices(520, 521, 2048) == tuple(range(521))
    sep = o.selected_token_indices(521, 522, 2048)
    assert sep[:8] == tuple(range(8)) and sep[8:] == tuple(range(9, 522))
    assert len(sep) == 521 and 8 not in sep


def test_final_128_rows_dense():
    assert o.sparse_end(1024) == 896
    assert o.selected_intervals(895, 1024, 1024) == ((0, 8), (383, 896))
    for q in range(896, 1024):
        assert o.selected_intervals(q, 1024, 1024) == ((0, q + 1),)


def test_project_contract_golden_values():
    span = o.QuerySpan(544, 576, True)
    assert o.submitted_span_intervals(span, 8320) == ((0, 8), (32, 576))
    assert o.submitted_span_intervals(o.QuerySpan(1024, 1056, True), 8320) == ((0, 8), (512, 1056))
    assert o.submitted_span_intervals(o.QuerySpan(0, 32, False), 8320) == ((0, 32),)
    assert o.submitted_span_intervals(o.QuerySpan(8192, 8224, False), 8320) == ((0, 8224),)
    assert o.bsnd_element_offset(128 + 11, 3, [7, 2, 19]) == 273792
    assert o.selected_intervals(520, 524, 1024) == ((0, 521),)
    assert o.selected_intervals(521, 524, 1024) == ((0, 8), (9, 522))
    assert o.selected_intervals(522, 524, 1024) == ((0, 8), (10, 523))
    assert o.selected_intervals(896, 897, 1024) == ((0, 897),)


@pytest.mark.parametrize("q0,tq,prompt", [(0, 1024, 1024), (500, 65, 2048), (766, 35, 2048),
                                          (894, 4, 1024), (8127, 65, 16384), (3, 200, 600)])
def test_query_span_row_coverage(q0, tq, prompt):
    sb, se = G.sparse_begin, o.sparse_end(prompt)
    spans = o.split_query_spans(q0, tq, sb, se)
    rows = []
    for s in spans:
        assert s.end - s.begin <= G.q_tile
        assert (s.begin - q0) // G.q_tile == (s.end - 1 - q0) // G.q_tile
        rows.extend(range(s.begin, s.end))
        for q in range(s.begin, s.end):
            assert s.sparse == (sb <= q < se)
        # A sparse span never submits a key outside the union of its rows' sets.
        if s.sparse:
            allowed = set()
            for q in range(s.begin, s.end):
                allowed.update(o.selected_token_indices(q, q0 + tq, prompt))
            sub = {k for b, e in o.submitted_span_intervals(s, q0 + tq) for k in range(b, e)}
            assert sub <= allowed
    assert rows == list(range(q0, q0 + tq))


def _empty_cache(pages, g):
    return [[[[0.0] * g.head_dim for _ in range(g.kv_heads)] for _ in range(g.page_size)]
            for _ in range(pages)]


def _set(cache, table, tok, h, vec, g):
    p, off = divmod(tok, g.page_size)
    cache[table[p]][off][h] = list(vec)


def test_gqa_query_heads_share_kv_head():
    g = o.Geometry(query_heads=8, kv_heads=2, head_dim=1, page_size=2, q_tile=2, sink_tokens=1,
                   local_window=1, dense_tail=1)
    table = [1]
    key, value = _empty_cache(2, g), _empty_cache(2, g)
    _set(value, table, 0, 0, [3.0], g)
    _set(value, table, 0, 1, [7.0], g)
    out = o.reference_attention_python([[[0.0]] * 8], key, value, table, 0, 1, 4, 1.0, g)
    assert [h[0] for h in out[0]] == [3.0] * 4 + [7.0] * 4


def test_sink_and_local_share_one_softmax():
    g = o.Geometry(query_heads=4, kv_heads=1, head_dim=1, page_size=4, q_tile=2, sink_tokens=2,
                   local_window=2, dense_tail=0)
    assert g.sparse_begin == 5
    table = [1, 0]
    key, value = _empty_cache(2, g), _empty_cache(2, g)
    for t in (0, 1):
        _set(value, table, t, 0, [10.0], g)
    _set(value, table, 2, 0, [1000.0], g)  # poison: excluded token
    for t in (3, 4, 5):
        _set(value, table, t, 0, [1.0], g)
    out = o.reference_attention_python([[[0.0]] * 4], key, value, table, 5, 6, 20, 1.0, g)
    for h in out[0]:
        assert abs(h[0] - (2 * 10.0 + 3 * 1.0) / 5) < 1e-12


def test_random_noncontiguous_table_invariance():
    g = o.Geometry(query_heads=4, kv_heads=1, head_dim=2, page_size=4, q_tile=2, sink_tokens=1,
                   local_window=2, dense_tail=1)
    rng = random.Random(20260728)
    table = rng.sample(range(7), 3)
    cache, ident = _empty_cache(7, g), _empty_cache(3, g)
    for t in range(12):
        _set(cache, table, t, 0, [float(t), float(-t)], g)
        _set(ident, [0, 1, 2], t, 0, [float(t), float(-t)], g)
    query = [[[0.25, -0.125]] * 4]
    a = o.reference_attention_python(query, cache, cache, table, 8, 9, 16, 2 ** -0.5, g)
    b = o.reference_attention_python(query, ident, ident, [0, 1, 2], 8, 9, 16, 2 ** -0.5, g)
    assert np.allclose(a, b, atol=1e-12)


def test_query_tiling_and_ragged_batch_invariance():
    g = o.Geometry(query_heads=4, kv_heads=1, head_dim=2, page_size=4, q_tile=4, sink_tokens=1,
                   local_window=2, dense_tail=2)
    rng = random.Random(13)
    cache = _empty_cache(5, g)
    for p in range(5):
        for t in range(4):
            cache[p][t][0] = [rng.uniform(-0.5, 0.5) for _ in range(2)]
    query = [[[rng.uniform(-0.4, 0.4) for _ in range(2)] for _ in range(4)] for _ in range(9)]
    table = [2, 0, 3]
    full = o.reference_attention_python(query, cache, cache, table, 3, 12, 16, 2 ** -0.5, g)
    tiled, off = [], 0
    for n in (4, 4, 1):
        tiled += o.reference_attention_python(query[off:off + n], cache, cache, table, 3 + off, 12, 16,
                                              2 ** -0.5, g)
        off += n
    assert np.allclose(full, tiled, atol=1e-12)
    packed = o.reference_attention_ragged_python(query[:4] + query[:5], cache, cache, [[4], [2, 0, 4]],
                                                 [0, 7], [4, 12], [16, 16], [4, 5], 2 ** -0.5, g)
    sep = (o.reference_attention_python(query[:4], cache, cache, [4], 0, 4, 16, 2 ** -0.5, g)
           + o.reference_attention_python(query[:5], cache, cache, [2, 0, 4], 7, 12, 16, 2 ** -0.5, g))
    assert np.allclose(packed, sep, atol=1e-12)


@pytest.mark.parametrize("case", META["cases"], ids=[c["name"] for c in META["cases"]])
def test_oracle_matches_reference_fixture(case):
    q, k, v, table = reference_case_inputs(case["query_start"], case["query_tokens"], case["seq_len"],
                                           case["seed"])
    assert inputs_digest(q, k, v, table) == case["digest"], "input generator drifted"
    assert table[0].tolist() == case["table"]
    out = o.oracle_attention(q, k, v, table, case["query_start"], case["seq_len"], case["prompt_len"], SCALE)
    gold = torch.from_numpy(OUTS[case["name"]])
    assert float((out[case["rows"]] - gold).abs().max()) < 2e-5


def test_rowwise_and_blocked_oracles_agree():
    q, k, v, table = baseline_inputs(1200, 1200, seed=3)
    a = o.oracle_attention(q, k, v, table, 0, 1200, 1200, SCALE)
    rows = list(range(0, 1200, 7))
    b = o.oracle_attention_rowwise(q, k, v, table, 0, 1200, 1200, SCALE, rows=rows)
    assert float((a[rows] - b[rows]).abs().max()) < 2e-5


def test_shared_softmax_sentinel_fixture():
    s = META["sentinels"]["shared_softmax"]
    assert abs(s["value"] - s["joint_expected"]) < 1e-2
    table = torch.tensor([s["table"]], dtype=torch.int32)
    k = torch.zeros(s["pages"], 128, 8, 128, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    for tok in range(522):
        p, off = o.physical_location(tok, s["table"])
        v[p, off] = 10.0 if tok < 8 else (1000.0 if tok == 8 else 1.0)
    out = o.oracle_attention(torch.zeros(1, 32, 128, dtype=torch.bfloat16), k, v, table, 521, 522,
                             2048, SCALE)
    assert abs(float(out[0, 0, 0]) - s["value"]) < 1e-5


def test_visited_bitmap_counts_pairs():
    bm = o.visited_bitmap(300, 1, 600, 900, 1024)
    assert int(np.unpackbits(bm.view(np.uint8)).sum()) == o.count_pairs(600, 300, 900, 1024)


def test_saved_qk_crossover_known_answer():
    # package/tests/test_planning_stats.py:103-120: 2261-token prompt saves 1,300,078 QK pairs.
    rows = range(521, 2261 - 128)
    assert sum(q - 520 for q in rows) == 1_300_078
