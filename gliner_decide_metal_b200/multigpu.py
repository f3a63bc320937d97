"""Row sharding helpers for multi-GPU runs.

Rows of a batch are independent (no cross-row interaction in DeBERTa.swift:274-447), so the
forward shards by contiguous row blocks with a full weight replica per GPU and no collective
on the data path. The same split is used by ``gdc_classify_sharded`` (C ABI) and by
``bench.py`` ranks; the only collectives are a barrier and a max of the per-rank device time.
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


def max_over_ranks(value: float, dist, device=None) -> float:
    """Max of a scalar over all ranks of the default process group (value if not initialised)."""
    if dist is None or not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
