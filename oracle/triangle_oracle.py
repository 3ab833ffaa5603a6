"""CPU oracle for TriangleMix paged sparse prefill attention.

TEST INFRASTRUCTURE ONLY.  This module is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(the CUDA kernel behind ``libtpsa.so``) never calls into it.

It restates, in our own code, the algorithm of the reference project's CPU
oracle ``operator/tests/triangle_v2_reference.py`` (file:line citations are
inside that project):

* ``selected_intervals``          <- triangle_v2_reference.py:193-232
* ``sparse_end``                  <- triangle_v2_reference.py:185-190
* ``split_query_spans``           <- triangle_v2_reference.py:95-149
* ``submitted_span_intervals``    <- triangle_v2_reference.py:152-182
* ``physical_location``           <- triangle_v2_reference.py:255-270
* ``reference_attention_python``  <- triangle_v2_reference.py:374-434
* ``reference_attention_ragged_python`` <- triangle_v2_reference.py:437-487
* ``oracle_attention_rowwise``    <- triangle_v2_reference.py:490-587
  (same per-row gather + fp32 softmax; used as the timed CPU baseline)
* ``oracle_attention``            blocked fp32 evaluation of the same key
  sets (64 rows at a time, exact per-row masks); used by the parity tests.

Parity of this restatement is pinned against the reference itself: the
fixtures under ``tests/golden/`` were produced by importing the reference
module in the build container (``tests/golden/make_golden.py``), and
``tests/test_oracle.py`` checks this module against them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import numpy as np


@dataclass(frozen=True)
class Geometry:
    """Schedule and tensor constants (reference triangle_v2_reference.py:31-72)."""

    query_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    page_size: int = 128
    q_tile: int = 32
    sink_tokens: int = 8
    local_window: int = 512
    dense_tail: int = 128

    def __post_init__(self) -> None:
        if min(self.query_heads, self.kv_heads, self.head_dim, self.page_size, self.q_tile) <= 0:
            raise ValueError("head counts, dimensions, page size, and tile must be positive")
        if self.query_heads % self.kv_heads:
            raise ValueError("query_heads must be divisible by kv_heads")
        if min(self.sink_tokens, self.local_window, self.dense_tail) < 0:
            raise ValueError("schedule sizes must be non-negative")

    @property
    def group_size(self) -> int:
        return self.query_heads // self.kv_heads

    @property
    def sparse_begin(self) -> int:
        # First row whose sink and window no longer touch (q == sink + window
        # still yields one contiguous dense prefix).
        return self.sink_tokens + self.local_window + 1


PRODUCTION = Geometry()

Intervals = tuple[tuple[int, int], ...]


def sparse_end(prompt_len: int, g: Geometry = PRODUCTION) -> int:
    """First absolute row of the dense tail."""
    if prompt_len < 0:
        raise ValueError("prompt_len must be non-negative")
    return max(0, prompt_len - g.dense_tail)


def selected_intervals(q: int, seq_len: int, prompt_len: int, g: Geometry = PRODUCTION) -> Intervals:
    """Half-open logical key intervals of query row ``q``."""
    if q < 0 or seq_len < 0 or prompt_len < 0:
        raise ValueError("positions must be non-negative")
    causal_end = min(q + 1, seq_len)
    if causal_end <= 0:
        return ()
    if not (g.sparse_begin <= q < sparse_end(prompt_len, g)):
        return ((0, causal_end),)
    sink = min(g.sink_tokens, causal_end)
    local = min(max(0, q - g.local_window), causal_end)
    if local <= sink:  # touching or overlapping: one dense prefix
        return ((0, causal_end),)
    out = []
    if sink:
        out.append((0, sink))
    if local < causal_end:
        out.append((local, causal_end))
    return tuple(out)


def selected_token_indices(q: int, seq_len: int, prompt_len: int, g: Geometry = PRODUCTION) -> tuple[int, ...]:
    return tuple(k for b, e in selected_intervals(q, seq_len, prompt_len, g) for k in range(b, e))


@dataclass(frozen=True)
class QuerySpan:
    begin: int
    end: int
    sparse: bool


def split_query_spans(query_start: int, query_tokens: int, sparse_begin: int,
                      sparse_end_position: int, g: Geometry = PRODUCTION) -> tuple[QuerySpan, ...]:
    """Cut every q tile at the dense/sparse row boundaries (reference span contract)."""
    if query_start < 0 or query_tokens <= 0 or sparse_begin < 0 or sparse_end_position < 0:
        raise ValueError("invalid span arguments")
    spans: list[QuerySpan] = []
    for tile0 in range(0, query_tokens, g.q_tile):
        lo = query_start + tile0
        hi = query_start + min(query_tokens, tile0 + g.q_tile)
        cuts = sorted({lo, hi} | {c for c in (sparse_begin, sparse_end_position) if lo < c < hi})
        tile_spans: list[QuerySpan] = []
        for b, e in zip(cuts, cuts[1:]):
            span = QuerySpan(b, e, sparse_begin <= b < sparse_end_position)
            if tile_spans and tile_spans[-1].sparse == span.sparse and tile_spans[-1].end == b:
                span = QuerySpan(tile_spans.pop().begin, e, span.sparse)
            tile_spans.append(span)
        spans.extend(tile_spans)
    return tuple(spans)


def submitted_span_intervals(span: QuerySpan, seq_len: int, g: Geometry = PRODUCTION) -> Intervals:
    """KV intervals one homogeneous span may submit to QK/PV."""
    q_end = min(span.end, seq_len)
    if q_end <= 0:
        return ()
    if not span.sparse:
        return ((0, q_end),)
    sink = min(g.sink_tokens, seq_len)
    local = min(max(0, span.begin - g.local_window), q_end)
    if local <= sink:
        return ((0, q_end),)
    out = []
    if sink:
        out.append((0, sink))
    if local < q_end:
        out.append((local, q_end))
    return tuple(out)


def physical_location(token: int, block_table: Sequence[int], g: Geometry = PRODUCTION) -> tuple[int, int]:
    """Logical token -> (physical page, offset in page)."""
    if token < 0:
        raise ValueError("logical_token must be non-negative")
    page, off = divmod(token, g.page_size)
    if page >= len(block_table):
        raise ValueError("block_table does not cover logical_token")
    phys = int(block_table[page])
    if phys < 0:
        raise ValueError("block_table contains a negative physical page")
    return phys, off


def bsnd_element_offset(token: int, kv_head: int, block_table: Sequence[int], g: Geometry = PRODUCTION) -> int:
    """Element offset of (token, kv_head, d=0) in a BSND paged cache."""
    phys, off = physical_location(token, block_table, g)
    return ((phys * g.page_size + off) * g.kv_heads + kv_head) * g.head_dim


def visible_mask(rows: np.ndarray, keys: np.ndarray, seq_len: int, prompt_len: int,
                 g: Geometry = PRODUCTION) -> np.ndarray:
    """Boolean [len(rows), len(keys)]: key k enters row q's softmax.

    Closed form of ``selected_intervals``; tests check the two agree.
    """
    q = np.asarray(rows, dtype=np.int64)[:, None]
    k = np.asarray(keys, dtype=np.int64)[None, :]
    causal = (k <= q) & (k < seq_len)
    sparse = (q >= g.sparse_begin) & (q < sparse_end(prompt_len, g))
    band = (k < g.sink_tokens) | (k >= q - g.local_window)
    return causal & (~sparse | band)


# ---------------------------------------------------------------- attention
def _softmax_weighted(scores: list[float], values: list[Sequence[float]]) -> list[float]:
    mx = max(scores)
    w = [math.exp(s - mx) for s in scores]
    den = math.fsum(w)
    return [math.fsum(wi * float(v[d]) for wi, v in zip(w, values)) / den for d in range(len(values[0]))]


def reference_attention_python(query, key_cache, value_cache, block_table, query_start: int,
                               seq_len: int, prompt_len: int, scale: float,
                               g: Geometry = PRODUCTION) -> list:
    """Pure-Python paged GQA attention with one joint softmax (small cases)."""
    if query_start < 0 or query_start + len(query) > seq_len:
        raise ValueError("query rows extend beyond seq_len")
    if len(block_table) < (seq_len + g.page_size - 1) // g.page_size:
        raise ValueError("block_table does not cover seq_len")
    out = []
    for i, qrow in enumerate(query):
        toks = selected_token_indices(query_start + i, seq_len, prompt_len, g)
        heads = []
        for h, qv in enumerate(qrow):
            kvh = h // g.group_size
            keys, vals = [], []
            for t in toks:
                p, o = physical_location(t, block_table, g)
                keys.append(key_cache[p][o][kvh])
                vals.append(value_cache[p][o][kvh])
            scores = [math.fsum(float(a) * float(b) for a, b in zip(qv, kk)) * float(scale) for kk in keys]
            heads.append(_softmax_weighted(scores, vals))
        out.append(heads)
    return out


def reference_attention_ragged_python(packed_query, key_cache, value_cache, block_tables, query_starts,
                                      seq_lens, prompt_lens, query_lengths, scale,
                                      g: Geometry = PRODUCTION) -> list:
    """Packed ragged batch = concatenation of per-request batch-one results."""
    n = len(query_lengths)
    if any(len(x) != n for x in (block_tables, query_starts, seq_lens, prompt_lens)):
        raise ValueError("ragged metadata lengths disagree")
    if sum(query_lengths) != len(packed_query):
        raise ValueError("query_lengths do not cover packed_query")
    out, off = [], 0
    for i, ql in enumerate(query_lengths):
        if ql <= 0:
            raise ValueError("each ragged query length must be positive")
        out.extend(reference_attention_python(packed_query[off:off + ql], key_cache, value_cache,
                                              block_tables[i], query_starts[i], seq_lens[i],
                                              prompt_lens[i], scale, g))
        off += ql
    return out


def _logical_kv(cache, table, seq_len: int, g: Geometry):
    """Gather the paged cache into logical order, fp32 [seq_len, Hkv, D]."""
    import torch

    pages = (seq_len + g.page_size - 1) // g.page_size
    phys = table.reshape(-1)[:pages].to(device="cpu", dtype=torch.int64)
    if phys.numel() < pages:
        raise ValueError("block_table does not cover seq_len")
    if bool((phys < 0).any()) or bool((phys >= cache.shape[0]).any()):
        raise ValueError("block_table holds a page outside the cache")
    return cache.index_select(0, phys).float().reshape(-1, cache.shape[2], g.head_dim)[:seq_len]


def _check_shapes(query, key_cache, value_cache, query_start, seq_len, g: Geometry):
    if query.dim() != 3 or query.shape[2] != g.head_dim:
        raise ValueError("query must be [Tq, Hq, D]")
    if key_cache.dim() != 4 or tuple(key_cache.shape[1:]) != (g.page_size, key_cache.shape[2], g.head_dim):
        raise ValueError("key cache must be [pages, page, Hkv, D]")
    if tuple(value_cache.shape) != tuple(key_cache.shape):
        raise ValueError("value cache shape must equal key cache shape")
    if query.shape[1] != key_cache.shape[2] * g.group_size:
        raise ValueError("query heads must be group_size x kv heads")
    if query_start + query.shape[0] > seq_len:
        raise ValueError("query rows extend beyond seq_len")


def prepare_logical_kv(key_cache, value_cache, block_table, seq_len: int, g: Geometry = PRODUCTION):
    """Logical-order fp32 K and V (the reference oracle's one gather per call)."""
    return (_logical_kv(key_cache, block_table, seq_len, g),
            _logical_kv(value_cache, block_table, seq_len, g))


def oracle_attention_rowwise(query, key_cache, value_cache, block_table, query_start: int,
                             seq_len: int, prompt_len: int, scale: float,
                             g: Geometry = PRODUCTION, rows: Sequence[int] | None = None,
                             logical_kv=None):
    """Per-row gather + fp32 softmax, the reference oracle's own method.

    ``rows`` restricts evaluation to a subset of query rows (others stay 0)
    and ``logical_kv`` (from ``prepare_logical_kv``) reuses one gather; the
    CPU baseline uses both to time a bounded sample.
    """
    import torch

    _check_shapes(query, key_cache, value_cache, query_start, seq_len, g)
    hkv = key_cache.shape[2]
    if logical_kv is None:
        logical_kv = prepare_logical_kv(key_cache, value_cache, block_table, seq_len, g)
    lk, lv = logical_kv
    qf = query.float()
    out = torch.zeros_like(qf)
    for r in (range(qf.shape[0]) if rows is None else rows):
        ivs = selected_intervals(query_start + r, seq_len, prompt_len, g)
        if len(ivs) == 1:  # a dense row: one contiguous range, read in place
            k, v = lk[ivs[0][0]:ivs[0][1]], lv[ivs[0][0]:ivs[0][1]]
        else:
            idx = torch.cat([torch.arange(b, e, dtype=torch.int64) for b, e in ivs])
            k = lk.index_select(0, idx)
            v = lv.index_select(0, idx)
        gq = qf[r].reshape(hkv, g.group_size, g.head_dim)
        p = torch.softmax(torch.einsum("hgd,thd->hgt", gq, k) * float(scale), dim=-1)
        out[r] = torch.einsum("hgt,thd->hgd", p, v).reshape(-1, g.head_dim)
    return out


def oracle_attention(query, key_cache, value_cache, block_table, query_start: int, seq_len: int,
                     prompt_len: int, scale: float, g: Geometry = PRODUCTION, block_rows: int = 64):
    """Blocked fp32 evaluation of exactly the same key sets (fast CPU oracle).

    For each block of query rows the scores are computed against the union of
    the rows' key sets and every row is masked with ``visible_mask``.
    """
    import torch

    _check_shapes(query, key_cache, value_cache, query_start, seq_len, g)
    hkv = key_cache.shape[2]
    lk = _logical_kv(key_cache, block_table, seq_len, g)
    lv = _logical_kv(value_cache, block_table, seq_len, g)
    qf = query.float()
    tq = qf.shape[0]
    out = torch.empty_like(qf)
    se = sparse_end(prompt_len, g)
    for r0 in range(0, tq, block_rows):
        r1 = min(tq, r0 + block_rows)
        q_lo, q_hi = query_start + r0, query_start + r1  # absolute rows
        all_sparse = q_lo >= g.sparse_begin and q_hi <= se
        if all_sparse:
            keys = np.concatenate([np.arange(0, g.sink_tokens),
                                   np.arange(max(g.sink_tokens, q_lo - g.local_window), q_hi)])
        else:
            keys = np.arange(0, q_hi)
        mask = torch.from_numpy(visible_mask(np.arange(q_lo, q_hi), keys, seq_len, prompt_len, g))
        kidx = torch.from_numpy(keys.astype(np.int64))
        k = lk.index_select(0, kidx)  # [K, Hkv, D]
        v = lv.index_select(0, kidx)
        gq = qf[r0:r1].reshape(r1 - r0, hkv, g.group_size, g.head_dim)
        s = torch.einsum("rhgd,khd->rhgk", gq, k) * float(scale)
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[r0:r1] = torch.einsum("rhgk,khd->rhgd", p, v).reshape(r1 - r0, -1, g.head_dim)
    return out


def visited_bitmap(query_tokens: int, query_heads: int, query_start: int, seq_len: int,
                   prompt_len: int, g: Geometry = PRODUCTION) -> np.ndarray:
    """Expected visited-key bitmap, uint32 [Tq * Hq, ceil(seq_len / 32)].

    Bit k of row (t * Hq + h) is set iff key k is in query row
    (query_start + t)'s selected intervals (all heads of a row share it).
    """
    words = (seq_len + 31) // 32
    out = np.zeros((query_tokens, words), dtype=np.uint32)
    keys = np.arange(words * 32)
    for r0 in range(0, query_tokens, 256):
        r1 = min(query_tokens, r0 + 256)
        m = visible_mask(np.arange(query_start + r0, query_start + r1), keys, seq_len, prompt_len, g)
        bits = m.reshape(r1 - r0, words, 32).astype(np.uint64)
        out[r0:r1] = (bits << np.arange(32, dtype=np.uint64)).sum(axis=2).astype(np.uint32)
    return np.repeat(out, query_heads, axis=0)


def count_pairs(query_start: int, query_tokens: int, seq_len: int, prompt_len: int,
                g: Geometry = PRODUCTION) -> int:
    """Number of (row, key) pairs in the key sets of all rows (per head)."""
    total = 0
    for q in range(query_start, query_start + query_tokens):
        total += sum(e - b for b, e in selected_intervals(q, seq_len, prompt_len, g))
    return total
