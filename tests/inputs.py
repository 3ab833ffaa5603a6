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
