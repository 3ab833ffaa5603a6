"""KV-head partition of one attention layer across the GPUs of a node.

Query head ``h`` reads only KV head ``h // 4`` (GQA 4:1; reference
operator/tests/triangle_v2_reference.py:410), so a layer splits into
independent KV-head groups with no exchange. Rank ``r`` of ``world`` owns KV heads
``[r * 8 / world, (r + 1) * 8 / world)`` and the query heads that read them,
and runs the operator on its slice through ``tpsa_paged_attention_heads``.
There is no data-path collective. ``gather_output`` all-gathers the slices along the
head axis, and only validation uses it.

The reference has no multi-device path: its plugin sends tensor-parallel
callers to the dense fallback (package/src/vllm_ascend_trianglemix/plugin.py:
1251-1253).
"""

from __future__ import annotations

import torch

KV_HEADS = 8
GROUP_SIZE = 4
SUPPORTED_WORLD_SIZES = (1, 2, 4, 8)


def kv_head_range(rank: int, world: int, kv_heads: int = KV_HEADS) -> tuple[int, int]:
    """KV heads ``[lo, hi)`` owned by ``rank``. ``world`` must divide the heads."""
    if world <= 0 or kv_heads % world != 0:
        raise ValueError(f"world size {world} must divide the {kv_heads} KV heads")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world size {world}")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def shard_query(query: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """Query heads that read KV heads ``[lo, hi)``, as a contiguous ``[Tq, 4*(hi-lo), D]``."""
    return query[:, GROUP_SIZE * lo:GROUP_SIZE * hi].contiguous()


def shard_cache(cache: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """KV heads ``[lo, hi)`` of a BSND paged cache, as a contiguous ``[P, 128, hi-lo, D]``."""
    return cache[:, :, lo:hi].contiguous()


def shard_layer(query, key_cache, value_cache, rank: int, world: int):
    """This rank's slice of one layer: ``(query, key_cache, value_cache, (lo, hi))``."""
    lo, hi = kv_head_range(rank, world, key_cache.shape[2])
    return (shard_query(query, lo, hi), shard_cache(key_cache, lo, hi),
            shard_cache(value_cache, lo, hi), (lo, hi))


def gather_output(out_shard: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather head slices ``[Tq, Hq/world, D]`` into ``[Tq, Hq, D]`` (validation only)."""
    import torch.distributed as dist

    parts = [torch.empty_like(out_shard) for _ in range(world)]
    dist.all_gather(parts, out_shard.contiguous(), group=group)
    return torch.cat(parts, dim=1)
