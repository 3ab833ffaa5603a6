"""Seeded synthetic inputs shared by the fixture generator and the tests.

``reference_case_inputs`` follows the input recipe of the reference's NPU
correctness matrix (operator/tests/npu_v2_correctness.py:238-274 in the
reference project): N(0, 1) * 0.5 values cast to bf16, logical pages mapped
through a permutation of ``logical + 7`` physical pages, with the first and
last entries swapped if the permutation happens to be consecutive.

``baseline_inputs`` is the BASELINE configuration recipe: N(0, 1) bf16 with
``torch.Generator().manual_seed(seed)`` and a random permutation of
``2 x logical`` physical pages.
"""

from __future__ import annotations

import hashlib
import math

import torch

QUERY_HEADS = 32
KV_HEADS = 8
HEAD_DIM = 128
PAGE = 128
SCALE = HEAD_DIM ** -0.5


def noncontiguous_table(logical: int, physical: int, gen: torch.Generator) -> torch.Tensor:
    perm = torch.randperm(physical, generator=gen, dtype=torch.int64)
    table = perm[:logical].clone()
    if logical > 1 and bool(torch.all(table[1:] == table[:-1] + 1)):
        table[0], table[-1] = table[-1].clone(), table[0].clone()
    return table.to(torch.int32).view(1, -1).contiguous()


def reference_case_inputs(query_start: int, query_tokens: int, seq_len: int, seed: int,
                          kv_heads: int = KV_HEADS):
    if query_start + query_tokens > seq_len:
        raise ValueError("query extends beyond seq_len")
    gen = torch.Generator().manual_seed(seed)
    logical = math.ceil(seq_len / PAGE)
    physical = logical + 7
    table = noncontiguous_table(logical, physical, gen)
    q = torch.randn(query_tokens, kv_heads * 4, HEAD_DIM, generator=gen).mul_(0.5).to(torch.bfloat16)
    shape = (physical, PAGE, kv_heads, HEAD_DIM)
    k = torch.randn(shape, generator=gen).mul_(0.5).to(torch.bfloat16)
    v = torch.randn(shape, generator=gen).mul_(0.5).to(torch.bfloat16)
    return q, k, v, table


def baseline_inputs(query_tokens: int, seq_len: int, seed: int = 0, kv_heads: int = KV_HEADS,
                    spare_pages: int | None = None):
    gen = torch.Generator().manual_seed(seed)
    logical = math.ceil(seq_len / PAGE)
    physical = 2 * logical if spare_pages is None else logical + spare_pages
    table = noncontiguous_table(logical, physical, gen)
    q = torch.randn(query_tokens, kv_heads * 4, HEAD_DIM, generator=gen).to(torch.bfloat16)
    shape = (physical, PAGE, kv_heads, HEAD_DIM)
    k = torch.randn(shape, generator=gen).to(torch.bfloat16)
    v = torch.randn(shape, generator=gen).to(torch.bfloat16)
    return q, k, v, table


def inputs_digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.int32
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def varlen_inputs(specs, seed: int = 0, spare_pages: int = 5):
    """A packed ragged batch over one shared page pool.

    ``specs`` lists (query_rows, seq_len, prompt_len) per request; request i's
    query rows are the last ``query_rows`` of its first ``seq_len`` tokens.
    Pages of all requests are drawn without replacement from one random
    permutation of the pool, so every request has its own scattered pages.
    Returns (packed query, key pool, value pool, block_tables [B, max_pages]
    padded with page 0, per-request [1, pages] tables, cu_seqlens_q).
    """
    gen = torch.Generator().manual_seed(seed)
    logical = [math.ceil(seq / PAGE) for _, seq, _ in specs]
    physical = sum(logical) + spare_pages
    perm = torch.randperm(physical, generator=gen, dtype=torch.int64)
    cols = max(logical)
    tables = torch.zeros(len(specs), cols, dtype=torch.int32)
    per_request, used = [], 0
    for i, n in enumerate(logical):
        row = perm[used:used + n].to(torch.int32)
        used += n
        tables[i, :n] = row
        per_request.append(row.view(1, -1).contiguous())
    cu = [0]
    for rows, _, _ in specs:
        cu.append(cu[-1] + rows)
    q = torch.randn(cu[-1], QUERY_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    shape = (physical, PAGE, KV_HEADS, HEAD_DIM)
    k = torch.randn(shape, generator=gen).to(torch.bfloat16)
    v = torch.randn(shape, generator=gen).to(torch.bfloat16)
    return q, k, v, tables.contiguous(), per_request, cu
