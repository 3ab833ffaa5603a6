"""KV-head partition across ranks, on CPU with the gloo backend.

Each rank takes its slice of one layer with the library's sharding helpers.
It runs the CPU oracle on that slice, standing in for the GPU kernel (which
needs no collective), and all-gathers the head slices. Rank 0 checks that the
gathered output equals the oracle on the whole layer.
The slices are independent, so the result must be bit-identical.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seq: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    pages = (seq + 127) // 128
    table = torch.randperm(2 * pages, generator=gen)[:pages].to(torch.int32).view(1, -1)
    q = torch.randn(seq, 32, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(2 * pages, 128, 8, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(2 * pages, 128, 8, 128, generator=gen).to(torch.bfloat16)
    return q, k, v, table


def _rank_main(rank: int, world: int, port: int, seq: int, result_q) -> None:
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from __graft_entry__ import load_package
    from oracle.triangle_oracle import oracle_attention

    tm = load_package()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, table = _layer(seq, 3)
        qs, ks, vs, (lo, hi) = tm.sharding.shard_layer(q, k, v, rank, world)
        assert (hi - lo) * world == 8 and qs.shape[1] == 4 * (hi - lo)
        out = oracle_attention(qs, ks, vs, table, 0, seq, seq, 128 ** -0.5).to(torch.bfloat16)
        full = tm.sharding.gather_output(out, world)
        if rank == 0:
            ref = oracle_attention(q, k, v, table, 0, seq, seq, 128 ** -0.5).to(torch.bfloat16)
            result_q.put(("ok", bool(torch.equal(full, ref)), tuple(full.shape)))
    except Exception as e:  # reported to the parent, which fails the test
        result_q.put(("error", repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_partition_gather_matches_full_layer(world):
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 704, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, equal, shape = result_q.get(timeout=10)
    assert status == "ok", equal
    assert shape == (704, 32, 128)
    assert equal


def test_kv_head_range_contract():
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    sh = load_package().sharding
    for world in (1, 2, 4, 8):
        ranges = [sh.kv_head_range(r, world) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    with pytest.raises(ValueError):
        sh.kv_head_range(0, 3)
    with pytest.raises(ValueError):
        sh.kv_head_range(2, 2)
