"""Host-side partitioning of the sparse-KV decode path across GPUs.

Two layouts, both one process per GPU:

* sequence sharding (multi-sequence batches): every (sequence, layer, KV head)
  unit is independent, so each rank owns whole sequences -- their pool blocks,
  block tables, representatives and tails -- and no data-path collective is
  needed;
* KV-head sharding (one long sequence): rank r owns a contiguous range of KV
  heads (and their query heads); after attention each rank holds
  [layers][its query heads][128] and an all-gather over the heads assembles
  [layers][QH][128] on every rank.

These helpers are pure host logic (no CUDA), shared by bench.py and the
multi-rank tests.
"""
from __future__ import annotations


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [first, first + count) share of `total` items for `rank`.

    The first `total % world` ranks get one extra item, so counts differ by at
    most one and the union over ranks is exactly range(total).
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def shard_sequences(seqs: int, world: int, rank: int) -> tuple[int, int]:
    """Sequences owned by `rank` under sequence sharding."""
    return shard_range(seqs, world, rank)


def shard_kv_heads(kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """KV heads owned by `rank` under KV-head sharding (needs world <= kv_heads
    and kv_heads % world == 0 so every rank's output block has the same size
    for the all-gather)."""
    if world > kv_heads or kv_heads % world:
        raise ValueError("KV-head sharding needs world to divide kv_heads")
    return shard_range(kv_heads, world, rank)


def assemble_heads(per_rank, group: int):
    """Concatenate per-rank attention outputs [layers][rank_QH][D] along heads
    in rank order: the layout an all-gather over KV-head shards produces."""
    import numpy as np

    return np.concatenate([np.asarray(x) for x in per_rank], axis=-2)
