"""BASELINE config 1 microbenchmarks through the C ABI: the disentangled attention
(q, k, v [32, 16, 256, 64] N(0,1); PQ / PK from a [512, 1024] N(0,1) table projected by
N(0, 0.02) weights; key lengths U[64, 256]) and the residual LayerNorm (x, res
[8192, 1024] N(0,1), eps 1e-7). Device buffers come from torch; each call is timed with CUDA
events over ``--reps`` launches after 3 warm-up launches, cycling 8 input sets so that
consecutive launches do not reuse L2-resident inputs.

    python -m gliner_decide_metal_b200.microbench [--batch 32] [--seq 256] [--reps 50]
"""
from __future__ import annotations

import argparse
import sys

import numpy as np


def _time(torch, fn, reps):
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3  # microseconds


def attention(batch=32, seq=256, reps=50, seed=1):
    import torch
    from ._lib import lib
    rng = np.random.Generator(np.random.PCG64(seed))
    E = 1024
    rel = rng.standard_normal((512, E), dtype=np.float32)
    wq = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    wk = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    pos = torch.from_numpy(np.concatenate([rel @ wq.T, rel @ wk.T], axis=1).astype(np.float16)).cuda()
    sets = []
    for _ in range(8):
        qkv = torch.from_numpy(rng.standard_normal((batch * seq, 3 * E), dtype=np.float32).astype(np.float16)).cuda()
        lens = rng.integers(min(64, seq), seq + 1, batch)
        mask = torch.from_numpy((np.arange(seq)[None, :] < lens[:, None]).astype(np.float16)).cuda()
        sets.append((qkv, mask, torch.empty((batch * seq, E), dtype=torch.float16, device="cuda")))

    def run(i):
        qkv, mask, ctx = sets[i % 8]
        st = lib.gdc_disentangled_attention(qkv.data_ptr(), pos.data_ptr(), mask.data_ptr(), ctx.data_ptr(), batch,
                                            seq, 16, None)
        if st != 0:
            raise RuntimeError(lib.gdc_last_error().decode())

    us = _time(torch, run, reps)
    if lib.gdc_kernels_check_errors() != 0:
        raise RuntimeError(lib.gdc_last_error().decode())
    flops = 16 * 4 * 2 * seq * seq * 64 * batch
    byts = 4 * batch * 16 * seq * 64 * 2 + 2 * 16 * 512 * 64 * 2 + batch * seq * 2
    return us, flops / us / 1e6, byts / us / 1e3


def layer_norm(rows=8192, cols=1024, reps=50, seed=2):
    import torch
    from ._lib import lib
    rng = np.random.Generator(np.random.PCG64(seed))
    sets = [tuple(torch.from_numpy(rng.standard_normal((rows, cols), dtype=np.float32).astype(np.float16)).cuda()
                  for _ in range(2)) + (torch.empty((rows, cols), dtype=torch.float16, device="cuda"),)
            for _ in range(8)]
    g = torch.ones(cols, dtype=torch.float16, device="cuda")
    b = torch.zeros(cols, dtype=torch.float16, device="cuda")

    def run(i):
        x, r, o = sets[i % 8]
        st = lib.gdc_residual_layer_norm(x.data_ptr(), r.data_ptr(), g.data_ptr(), b.data_ptr(), o.data_ptr(), rows,
                                         cols, 1e-7, None)
        if st != 0:
            raise RuntimeError(lib.gdc_last_error().decode())

    us = _time(torch, run, reps)
    byts = 3 * rows * cols * 2 + 2 * cols * 2
    return us, byts / us / 1e3


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m gliner_decide_metal_b200.microbench")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args(argv)
    us, tf, gbs = attention(args.batch, args.seq, args.reps)
    print(f"attention B={args.batch} H=16 L={args.seq} d=64: {us:.1f} us, {tf:.1f} TFLOP/s (gathered-dot count), "
          f"{gbs:.0f} GB/s algorithmic")
    us, gbs = layer_norm(args.batch * args.seq, 1024, args.reps)
    print(f"residual LayerNorm [{args.batch * args.seq}, 1024]: {us:.1f} us, {gbs:.0f} GB/s algorithmic")
    return 0


if __name__ == "__main__":
    sys.exit(main())
