"""world_size-2 gloo tests (CPU) of the multi-GPU host logic: row sharding covers every
row once and matches gdc_classify_sharded's split, the device-time reduction is a max over
ranks, and a rank that fails before the collective is detected by the survivor through the
process-group timeout (no hang)."""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from bench import max_over_ranks
    from gliner_decide_metal_b200.multigpu import shard_bounds
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    try:
        if mode == "shard":
            start, count = shard_bounds(37, world, rank)
            rows = list(range(start, start + count))
            gathered = [None] * world
            dist.all_gather_object(gathered, rows)
            m = max_over_ranks(10.0 + rank * 2.5, dist)
            (Path(out_dir) / f"r{rank}.txt").write_text(f"{gathered}|{m}")
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("simulated rank failure before the timing collective")
            try:
                max_over_ranks(1.0, dist)
                (Path(out_dir) / "r0.txt").write_text("no-error")
            except Exception as e:  # the survivor learns of the failure instead of hanging
                (Path(out_dir) / "r0.txt").write_text("detected:" + type(e).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("worker hung")
    return procs


def test_shard_bounds_single_process():
    from gliner_decide_metal_b200.multigpu import shard_bounds
    for n in (0, 1, 7, 32, 256, 1001):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                s, c = shard_bounds(n, world, r)
                rows += list(range(s, s + c))
            assert rows == list(range(n))


def test_gloo_sharding_and_max_over_ranks(tmp_path):
    _run("shard", tmp_path)
    for r in range(2):
        gathered, m = (tmp_path / f"r{r}.txt").read_text().split("|")
        assert eval(gathered) == [list(range(0, 19)), list(range(19, 37))]
        assert float(m) == 12.5


def test_gloo_failed_rank_is_detected(tmp_path):
    procs = _run("fail", tmp_path)
    assert procs[1].exitcode != 0
    assert (tmp_path / "r0.txt").read_text().startswith("detected:")
