"""Row sharding helpers for multi-GPU runs.

Rows of a batch are independent (no cross-row interaction in DeBERTa.swift:274-447), so the
forward shards by contiguous row blocks with a full weight replica per GPU and no collective
on the data path. This is the host-side statement of the split ``gdc_classify_sharded``
(C ABI) makes.
"""
from __future__ import annotations


def shard_bounds(n_rows: int, world: int, rank: int):
    """Contiguous block of rows owned by `rank`: (start, count). The first n_rows % world
    ranks get one extra row (identical to gdc_classify_sharded)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)
