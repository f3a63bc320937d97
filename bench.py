#!/usr/bin/env python3
"""Throughput benchmark of the B200 GLiNER2.5-Decide classification forward.

Workload: DeBERTa-v3-large (24 layers) + GLiNER classification MLP,
batch 32, L=256 bucket, fp16 random-init weights (seed 0), synthetic rows with text
lengths U[40, 230] and 1 single-label task x 5 labels. A step is one forward pass over
one such batch. With ``--gpus N`` (launched one process per GPU by torchrun) every rank
runs its own batches (weak scaling: rows are independent, no collective on the data
path); timing is device-side (CUDA events on the model's stream), max over ranks.

Printed JSON line (rank 0):
  value     sequences/s over all ranks, inputs resident in HBM (gdc_classify_device)
  e2e       the same metric through gdc_classify with host buffers (H2D of the step's
            inputs and D2H of its logits inside the timed region)
  roofline  the dominant kernel (the tcgen05 projection GEMM family): algorithmic FLOPs /
            its device time, against the measured bf16 burst peak in MEASURED_PEAKS.json
            (the timed region is a fraction of a second at full clock); ``kernels`` gives
            every kernel class the same way (GEMMs against the tensor peak, attention
            against both HBM and tensor peaks, LayerNorm / embedding against HBM)
  cpu_baseline  the CPU restatement of the reference forward (oracle/, numpy fp32 BLAS,
            all host threads) on a bounded sample of the same workload (rank 0, N=1)
  dense_grid  the same K steps with row packing off (every one of the B x L positions
            through the encoder, as the reference computes them), with a check that the
            last step's logits are bit-identical to the packed run's
  config4   BASELINE config 4 (256 rows per GPU, L=512, text U[200, 500]) on every rank,
            device-timed, max over ranks: the configuration written for the scaling run

Per-kernel times come from a second pass of the same steps that replays a captured copy
of the forward with an event node after every kernel group (the stage profiler), one
synchronised replay per step; the sum of its intervals is reported beside the plain
step time.

Row packing: each batch row's positions up to its last valid token (or active marker)
are packed back to back and only those rows go through the encoder kernels; roofline
FLOPs and bytes count the packed rows.

``--impl reference`` times that CPU restatement alone (the reference itself is Swift/MLX
for Apple silicon and cannot run here) and prints its line with ``"impl": "reference"``;
it does not map libgdc.so. ``--micro`` prints the BASELINE config 1 kernel
microbenchmarks (attention and residual LayerNorm through the C ABI) instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "sequences/sec, DeBERTa-v3-large b32 L256 fp16, 1/2/4/8 B200; % roofline"
UNIT = "sequences/sec"
BATCH, SEQ = 32, 256
LAYERS = 24
HIDDEN, INTER = 1024, 4096
HEADS = 16
N_RESIDENT_BATCHES = 8
# (N, K) of the four encoder projections
GEMMS = {"qkv_gemm": (3 * HIDDEN, HIDDEN), "out_gemm": (HIDDEN, HIDDEN), "ffn_up_gemm": (INTER, HIDDEN),
         "ffn_down_gemm": (HIDDEN, INTER)}
# Algorithmic FLOPs of the four encoder projections per token, 24 layers.
GEMM_FLOPS_PER_TOKEN = sum(2 * n * k for n, k in GEMMS.values()) * LAYERS
# QK, c2p, p2c, PV as gathered dots, per (query, key) pair of one layer's 16 heads
ATTN_FLOPS_PER_PAIR_LAYER = HEADS * 4 * 2 * 64
POS_QK_BYTES = 512 * 2 * HIDDEN * 2  # one layer's PQ | PK table


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    ap.add_argument("--weights", type=str, default=None, help="reuse an existing weights file")
    ap.add_argument("--no-dense-leg", action="store_true", help="skip the dense-grid comparison run")
    ap.add_argument("--no-config4", action="store_true", help="skip the BASELINE config 4 leg")
    ap.add_argument("--micro", action="store_true", help="BASELINE config 1 kernel microbenchmarks only")
    ap.add_argument("--reps", type=int, default=50, help="launches per microbenchmark (--micro)")
    return ap.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def max_over_ranks(value: float, dist, device=None) -> float:
    """Max of a scalar over all ranks of the default process group (value if not initialised)."""
    if dist is None or not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weights_path(rank, world, dist, explicit):
    if explicit:
        return Path(explicit)
    path = Path(tempfile.gettempdir()) / "gdc_bench_weights_seed0_l24.safetensors"
    if rank == 0 and not path.exists():
        from gliner_decide_metal_b200 import synthetic
        tmp = path.with_suffix(".tmp")
        synthetic.write_weights(tmp, seed=0, num_layers=LAYERS)
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()
    return path


# ----------------------------------------------------------------------------- CPU arm

def cpu_reference_sample(budget_s: float, min_rows: int = 1, max_rows: int = BATCH, seed: int = 3):
    """Time the oracle's fp32 forward on rows of the benchmark batch, one row per call,
    until `budget_s` is used. Returns (seq_per_s, rows, seconds, threads)."""
    from oracle import reference_forward as rf
    from gliner_decide_metal_b200 import synthetic
    try:
        from threadpoolctl import threadpool_limits
        limiter = threadpool_limits(limits=cpu_threads())
    except Exception:
        limiter = None
    w = synthetic.make_weights(seed=0, num_layers=LAYERS)
    W = rf.OracleWeights(w, rf.OracleConfig())
    proj = rf.relative_projections(W, fp16_rounding=False)
    batch = synthetic.config2(seed=seed)
    # warm-up one row (BLAS thread pool start-up)
    rf.forward(W, batch.input_ids[:1], batch.attention_mask[:1], batch.marker_indices[:1], batch.marker_mask[:1],
               fp16_rounding=False, projections=proj)
    rows = 0
    t0 = time.perf_counter()
    while rows < max_rows and (rows < min_rows or time.perf_counter() - t0 < budget_s):
        i = rows % BATCH
        rf.forward(W, batch.input_ids[i:i + 1], batch.attention_mask[i:i + 1], batch.marker_indices[i:i + 1],
                   batch.marker_mask[i:i + 1], fp16_rounding=False, projections=proj)
        rows += 1
    dt = time.perf_counter() - t0
    del limiter
    return rows / dt, rows, dt, cpu_threads()


def run_reference_arm(args, rank):
    """The CPU restatement of the reference forward alone. Imports only host-side modules
    (the synthetic generators and the oracle); libgdc.so is never mapped."""
    if rank != 0:
        return 0
    from oracle import reference_forward as rf
    from gliner_decide_metal_b200 import synthetic
    threads = cpu_threads()
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=threads)
    except Exception:
        pass
    w = synthetic.make_weights(seed=0, num_layers=LAYERS)
    W = rf.OracleWeights(w, rf.OracleConfig())
    proj = rf.relative_projections(W, fp16_rounding=False)
    batch = synthetic.config2(seed=3)
    rows_per_step = 1

    def step(i):
        r = i % BATCH
        rf.forward(W, batch.input_ids[r:r + 1], batch.attention_mask[r:r + 1], batch.marker_indices[r:r + 1],
                   batch.marker_mask[r:r + 1], fp16_rounding=False, projections=proj)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    sample = (f"{rows_per_step} row of the b32 L256 batch per step (one full 24-layer forward at L=256), "
              f"{args.steps} steps")
    from gliner_decide_metal_b200._lib import lib
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "BASELINE config 2: DeBERTa-v3-large + GLiNER MLP, B=32, L=256 bucket",
                       "batch": BATCH, "seq_len": SEQ, "rows_per_step": rows_per_step},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "product_library_mapped": bool(lib.loaded),
            "note": "CPU restatement (oracle/reference_forward.py, numpy fp32 BLAS) of DeBERTa.swift's forward; "
                    "the reference's Swift/MLX code needs macOS + Apple silicon and cannot run on this host"}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed regions."""

    FIELDS = ("timestamp,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        # GPUs of this job by UUID (nvidia-smi numbers GPUs physically, CUDA by visibility)
        self.uuids = {str(u).lower().removeprefix("gpu-") for u in uuids}
        self.proc = None
        self.windows = []
        self.path = Path(tempfile.gettempdir()) / f"gdc_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark(self, t0: float, t1: float):
        """Wall-clock bounds of one timed region; only samples inside the regions are kept."""
        self.windows.append((t0, t1))

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        import datetime
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10 or parts[1].lower().removeprefix("gpu-") not in self.uuids:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        main = []
        if self.windows:
            t0, t1 = self.windows[0]
            main = [r for r in rows if t0 <= r[0] <= t1 + 0.1]
            rows = [r for r in rows if any(a <= r[0] <= b + 0.1 for a, b in self.windows)] or \
                [r for r in rows if r[0] >= t0][:len(self.uuids)]
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in rows for n, v in zip(names, r[3]) if v.lower() == "active"}
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": rows[-1][2],
                "reasons": sorted(reasons), "samples": len(rows),
                "main_region_samples": len(main),
                "main_region_sm_mhz": statistics.median(r[1] for r in main) if main else None,
                "window": "nvidia-smi every 50 ms, samples inside the timed regions of this run "
                          "(device-timed steps, profiled replays, dense grid, e2e, config 4)"}


# ----------------------------------------------------------------------------- roofline

def kernel_classes(prof, steps, rows_timed, sum_ext2, sum_bl, markers_per_step, peaks, scale):
    """Per kernel class: device ms per step, launches, algorithmic FLOPs / bytes per launch,
    achieved rates and fractions of the measured peaks. The profiled replay records an event
    node after every kernel group, which makes every interval a little longer; each class
    keeps its share of the profiled step and `scale` (plain / profiled step time) maps it onto
    the uninstrumented step, so the class times add up to the plain step time
    (`raw_ms_per_step` keeps the measured interval sum). These shares agree with the ncu
    launch list of the same workload within a few percent."""
    out = {}
    tensor_peak, hbm_peak = peaks["bf16_tflops"], peaks["hbm_gbs"]

    def entry(name, flops, byts, bound):
        raw_ns, launches = prof.get(name, (0, 0))
        if not raw_ns or not launches:
            return None
        ns = raw_ns * scale
        sec = ns * 1e-9
        e = {"ms_per_step": ns / 1e6 / steps, "raw_ms_per_step": raw_ns / 1e6 / steps, "launches": launches,
             "us_per_launch": ns / 1e3 / launches, "bound": bound}
        if flops:
            e["tflops"] = flops / sec / 1e12
            e["tensor_frac"] = e["tflops"] / tensor_peak
            e["flops_per_launch"] = flops / launches
        if byts:
            e["gbs"] = byts / sec / 1e9
            e["hbm_frac"] = e["gbs"] / hbm_peak
            e["bytes_per_launch"] = byts / launches
        return e

    for name, (n, k) in GEMMS.items():
        flops = 2.0 * n * k * rows_timed * LAYERS
        byts = 2.0 * LAYERS * (rows_timed * (k + n) + steps * (n * k + n))
        out[name] = entry(name, flops, byts, "tensor")
    attn_flops = float(ATTN_FLOPS_PER_PAIR_LAYER) * sum_ext2 * LAYERS
    attn_bytes = LAYERS * (4.0 * rows_timed * HIDDEN * 2 + steps * POS_QK_BYTES + 2.0 * sum_bl)
    out["attention"] = entry("attention", attn_flops, attn_bytes, "hbm+tensor")
    ln_bytes = 2 * LAYERS * (3.0 * rows_timed * HIDDEN * 2 + steps * 2 * HIDDEN * 2)
    out["layer_norm"] = entry("layer_norm", None, ln_bytes, "hbm")
    emb_bytes = rows_timed * (2.0 * HIDDEN * 2 + 6) + steps * 2 * HIDDEN * 2
    out["embedding"] = entry("embedding", None, emb_bytes, "hbm")
    cls_flops = 2.0 * markers_per_step * steps * (HIDDEN * 2 * HIDDEN + 2 * HIDDEN)
    out["classifier"] = entry("classifier", cls_flops, None, "latency")
    return {k: v for k, v in out.items() if v is not None}


# ----------------------------------------------------------------------------- microbench

def run_micro(args):
    """BASELINE config 1 microbenchmarks through the C ABI (kernel-level entry points):
    disentangled attention (q, k, v [32, 16, 256, 64] N(0,1); PQ / PK from a [512, 1024]
    N(0,1) table projected by N(0, 0.02) weights; key lengths U[64, 256]) and the residual
    LayerNorm (x, res [8192, 1024] N(0,1), eps 1e-7). Each is timed with CUDA events over
    --reps launches after 3 warm-up launches, cycling 8 input sets (larger than L2 in total)."""
    import torch
    from gliner_decide_metal_b200._lib import lib
    peaks = measured_peaks()

    def timed(fn, reps):
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

    rng = np.random.Generator(np.random.PCG64(1))
    B, L, E = 32, 256, HIDDEN
    rel = rng.standard_normal((512, E), dtype=np.float32)
    wq = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    wk = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    pos = torch.from_numpy(np.concatenate([rel @ wq.T, rel @ wk.T], axis=1).astype(np.float16)).cuda()
    sets = []
    for _ in range(8):
        qkv = torch.from_numpy(rng.standard_normal((B * L, 3 * E), dtype=np.float32).astype(np.float16)).cuda()
        lens = rng.integers(64, L + 1, B)
        mask = torch.from_numpy((np.arange(L)[None, :] < lens[:, None]).astype(np.float16)).cuda()
        sets.append((qkv, mask, torch.empty((B * L, E), dtype=torch.float16, device="cuda")))

    def attn(i):
        qkv, mask, ctx = sets[i % 8]
        st = lib.gdc_disentangled_attention(qkv.data_ptr(), pos.data_ptr(), mask.data_ptr(), ctx.data_ptr(), B, L,
                                            HEADS, None)
        if st != 0:
            raise RuntimeError(lib.gdc_last_error().decode())

    us = timed(attn, args.reps)
    if lib.gdc_kernels_check_errors() != 0:
        raise RuntimeError(lib.gdc_last_error().decode())
    flops = HEADS * 4 * 2 * L * L * 64 * B
    byts = 4 * B * HEADS * L * 64 * 2 + POS_QK_BYTES // 2 + B * L * 2
    print(json.dumps({"micro": "attention", "config": "BASELINE config 1: B=32 H=16 L=256 d=64, key lengths "
                      "U[64,256], all positions", "us": us, "tflops": flops / us / 1e6,
                      "tensor_frac": flops / us / 1e6 / peaks["bf16_tflops"], "gbs": byts / us / 1e3,
                      "hbm_frac": byts / us / 1e3 / peaks["hbm_gbs"], "flops": flops, "bytes": byts}), flush=True)

    rows, cols = 8192, 1024
    lsets = [tuple(torch.from_numpy(rng.standard_normal((rows, cols), dtype=np.float32).astype(np.float16)).cuda()
                   for _ in range(2)) + (torch.empty((rows, cols), dtype=torch.float16, device="cuda"),)
             for _ in range(8)]
    g = torch.ones(cols, dtype=torch.float16, device="cuda")
    b = torch.zeros(cols, dtype=torch.float16, device="cuda")

    def ln(i):
        x, r, o = lsets[i % 8]
        st = lib.gdc_residual_layer_norm(x.data_ptr(), r.data_ptr(), g.data_ptr(), b.data_ptr(), o.data_ptr(), rows,
                                         cols, 1e-7, None)
        if st != 0:
            raise RuntimeError(lib.gdc_last_error().decode())

    us = timed(ln, args.reps)
    byts = 3 * rows * cols * 2 + 2 * cols * 2
    print(json.dumps({"micro": "residual_layer_norm", "config": "BASELINE config 1: [8192, 1024] + residual",
                      "us": us, "gbs": byts / us / 1e3, "hbm_frac": byts / us / 1e3 / peaks["hbm_gbs"],
                      "bytes": byts}), flush=True)
    return 0


# ----------------------------------------------------------------------------- native arm

def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank)
    if args.micro:
        return run_micro(args)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic

    wpath = weights_path(rank, world, dist, args.weights)
    model = g.GLiNERDecideClassifier(wpath, device=local)
    stream = torch.cuda.ExternalStream(model.stream, device=torch.device("cuda", local))
    dev_name = f"cuda:{local}"

    def to_dev(b):
        return dict(ids=torch.from_numpy(b.input_ids.astype(np.int32)).cuda(local),
                    mask=torch.from_numpy(b.attention_mask.astype(np.float16)).cuda(local),
                    mi=torch.from_numpy(b.marker_indices.astype(np.int32)).cuda(local),
                    mm=torch.from_numpy(b.marker_mask.astype(np.float32)).cuda(local))

    # HBM-resident inputs: N_RESIDENT_BATCHES distinct batches per rank.
    batches = [synthetic.config2(seed=1000 * rank + 3 + i) for i in range(N_RESIDENT_BATCHES)]
    dev = [to_dev(b) for b in batches]
    hm, o = batches[0].marker_indices.shape[1:]
    # Packed encoder rows per batch (the extent rule of csrc/kernels/pack.cu): the GEMM and
    # attention work the forward actually has to do.
    layouts = [g.packed_row_layout(b.attention_mask, b.marker_indices, b.marker_mask) for b in batches]
    packed_rows = [int(off[-1]) for _, off in layouts]
    ext2 = [int((ext.astype(np.int64) ** 2).sum()) for ext, _ in layouts]
    logits = torch.empty((BATCH, hm, o), dtype=torch.float32, device=dev_name)
    torch.cuda.synchronize(local)

    def step(i, d=None, B=BATCH, L=SEQ, out=None):
        d = d if d is not None else dev[i % N_RESIDENT_BATCHES]
        model.classify_device(B, L, hm, o, d["ids"].data_ptr(), d["mask"].data_ptr(), d["mi"].data_ptr(),
                              d["mm"].data_ptr(), (out if out is not None else logits).data_ptr())

    def barrier():
        if world > 1:
            dist.barrier()

    def mor(x: float) -> float:
        return max_over_ranks(x, dist if world > 1 else None, device=dev_name)

    for i in range(max(args.warmup, 3)):
        step(i)
    model.check_errors()

    def timed_region(n_steps, fn, profiled=False):
        if profiled:
            model.profile_reset()
            model.profile_enable(True)
        barrier()
        torch.cuda.synchronize(local)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        ev0.record(stream)
        for i in range(n_steps):
            fn(i)
        ev1.record(stream)
        torch.cuda.synchronize(local)
        t1 = time.time()
        barrier()
        if profiled:
            model.profile_enable(False)
        clocks.mark(t0, t1)
        return ev0.elapsed_time(ev1)

    # ---- timed region (device), clocks sampled during it and the later legs
    devs = list(range(torch.cuda.device_count())) if world > 1 else [local]
    clocks = ClockSampler([torch.cuda.get_device_properties(d).uuid for d in devs])
    clocks.start()
    time.sleep(0.4)  # let the sampler start before the load
    ms = timed_region(args.steps, step)
    model.check_errors()
    ms_max = mor(ms)
    packed_last = logits.clone()
    # ---- the same steps replayed with an event node after every kernel group
    for i in range(2):  # first call of the profiled shape runs eagerly, the second captures
        model.profile_enable(True)
        step(i)
        model.profile_enable(False)
    ms_prof = timed_region(args.steps, step, profiled=True)
    prof = model.profile_read()
    model.check_errors()
    seqs = BATCH * args.steps * world
    value = seqs / (ms_max / 1e3)

    # ---- the same steps on the dense [B, L] grid (the reference's layout), for comparison
    dense = None
    if not args.no_dense_leg:
        model.row_packing = False
        for i in range(3):
            step(i)
        ms_dense = mor(timed_region(args.steps, step))
        model.check_errors()
        same = bool(torch.equal(logits.view(torch.int32), packed_last.view(torch.int32)))
        model.row_packing = True
        for i in range(3):
            step(i)
        dense = {"value": seqs / (ms_dense / 1e3), "ms_per_step": ms_dense / args.steps,
                 "rows_per_step": BATCH * SEQ,
                 "last_step_logits_bit_identical_to_packed": same}

    # ---- e2e through the public API with host buffers
    host_inputs = [g.DecisionInput(b.input_ids, b.attention_mask, b.marker_indices, b.marker_mask) for b in batches]
    for i in range(2):
        model.classify(host_inputs[i % N_RESIDENT_BATCHES])
    barrier()
    torch.cuda.synchronize(local)
    t0w = time.time()
    t0 = time.perf_counter()
    for i in range(args.steps):
        model.classify(host_inputs[i % N_RESIDENT_BATCHES])
    e2e_local = time.perf_counter() - t0
    clocks.mark(t0w, time.time())
    e2e_s = mor(e2e_local)
    e2e_value = seqs / e2e_s
    R = BATCH * hm * o
    h2d = BATCH * SEQ * (4 + 2) + R * (4 + 4)   # int32 ids, fp16 mask, int32 markers, fp32 marker mask
    d2h = R * (4 + 2)                            # fp32 + fp16 logits

    # ---- 256 rows per GPU, L=512 (the scaling configuration)
    c4 = None
    if not args.no_config4:
        c4b = synthetic.config4(seed=5 + 1000 * rank)
        c4d = to_dev(c4b)
        c4_hm, c4_o = c4b.marker_indices.shape[1:]
        c4_rows = c4b.input_ids.shape[0]
        c4_logits = torch.empty((c4_rows, c4_hm, c4_o), dtype=torch.float32, device=dev_name)

        def step4(i):
            model.classify_device(c4_rows, 512, c4_hm, c4_o, c4d["ids"].data_ptr(), c4d["mask"].data_ptr(),
                                  c4d["mi"].data_ptr(), c4d["mm"].data_ptr(), c4_logits.data_ptr())

        for i in range(3):
            step4(i)
        c4_steps = max(3, args.steps // 4)
        ms4 = mor(timed_region(c4_steps, step4))
        model.check_errors()
        _, off4 = g.packed_row_layout(c4b.attention_mask, c4b.marker_indices, c4b.marker_mask)
        c4 = {"value": c4_rows * c4_steps * world / (ms4 / 1e3), "unit": "rows/sec", "ms_per_step": ms4 / c4_steps,
              "steps": c4_steps, "rows_per_gpu": c4_rows, "seq_len": 512, "n_gpus": world,
              "packed_rows_per_step": int(off4[-1]),
              "workload": "BASELINE config 4: 256 rows per GPU, L=512, text lengths U[200,500], 1 task x 5 labels; "
                          "device-timed, max over ranks"}

    time.sleep(0.3)  # let the sampler flush the samples of the last region
    clk = clocks.stop()

    # ---- roofline: every kernel class, the GEMM family as the dominant kernel
    peaks = measured_peaks()
    rows_timed = sum(packed_rows[i % N_RESIDENT_BATCHES] for i in range(args.steps))
    sum_ext2 = sum(ext2[i % N_RESIDENT_BATCHES] for i in range(args.steps))
    prof_sum_ms = sum(v[0] for v in prof.values()) / 1e6
    intervals = sum(v[1] for v in prof.values())
    event_overhead_ns = max(0.0, (prof_sum_ms - ms) * 1e6 / max(1, intervals))
    scale = min(1.0, ms / prof_sum_ms) if prof_sum_ms > 0 else 1.0
    kernels = kernel_classes(prof, args.steps, rows_timed, sum_ext2, BATCH * SEQ * args.steps, R, peaks, scale)
    gemm_ns = sum(kernels[n]["ms_per_step"] * args.steps * 1e6 for n in GEMMS if n in kernels)
    gemm_raw_ns = sum(prof.get(n, (0, 0))[0] for n in GEMMS)
    gemm_launches = sum(prof.get(n, (0, 0))[1] for n in GEMMS)
    gemm_flops = GEMM_FLOPS_PER_TOKEN * rows_timed
    achieved_tflops = gemm_flops / (gemm_ns * 1e-9) / 1e12 if gemm_ns else None
    traffic = None
    tpath = ROOT / "profiles" / "gemm_traffic.json"
    if tpath.exists():
        try:
            tj = json.loads(tpath.read_text())
            # the capture is one batch's launches; scale to this run's mean packed rows
            traffic = tj["bytes_per_launch"] * (rows_timed / args.steps) / tj.get("packed_rows", BATCH * SEQ)
        except Exception:
            traffic = None
    gemm_bytes = sum(kernels[n]["bytes_per_launch"] * kernels[n]["launches"] for n in GEMMS if n in kernels)
    roofline = {"kernel": "gemm_pair_kernel (cta_group::2 tcgen05; QKV / out / FFN-up / FFN-down projections)",
                "bound": "tensor",
                "measured_in": f"second pass of the same {args.steps} steps replaying a captured forward with an "
                               "event node after every kernel group, one synchronised replay per step; the "
                               f"intervals sum to {prof_sum_ms / args.steps:.3f} ms/step against "
                               f"{ms / args.steps:.3f} ms/step uninstrumented; every class keeps its share of the "
                               f"profiled step, scaled by {scale:.4f} onto the plain step",
                "achieved_raw": gemm_flops / (gemm_raw_ns * 1e-9) / 1e12 if gemm_raw_ns else None,
                "event_overhead_us_per_interval": event_overhead_ns / 1e3,
                "achieved": achieved_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": (achieved_tflops / peaks["bf16_tflops"]) if achieved_tflops else None,
                "peak_source": f"{peaks['source']} bf16_tflops (burst: the timed region is a fraction of a second)",
                "frac_of_sustained": (achieved_tflops / peaks["bf16_tflops_sustained"]) if achieved_tflops else None,
                "traffic": traffic,
                "traffic_source": "profiles/gemm_traffic.json: ncu dram__bytes_read.sum + dram__bytes_write.sum per "
                                  "launch, layer-0 projections of one batch of this workload averaged, scaled by "
                                  "this run's mean packed rows over the captured batch's",
                "algorithmic_bytes_per_launch_avg": gemm_bytes / max(1, gemm_launches),
                "algorithmic_units": f"{rows_timed / args.steps:.1f} packed rows per step (of {BATCH * SEQ} dense)",
                "launches": gemm_launches,
                "flops_per_launch_avg": gemm_flops / max(1, gemm_launches),
                "kernels": kernels,
                "profiled_ms_per_step": prof_sum_ms / args.steps}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, rows, dt, thr = cpu_reference_sample(args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": thr, "kind": "port",
               "sample": f"{rows} rows of the b32 L256 batch, one 24-layer fp32 forward per row, {dt:.1f} s "
                         "(oracle/reference_forward.py, numpy BLAS)"}

    launches_per_step = 2 + LAYERS * 7 + 3  # row pack, embedding, 7 per layer, classifier
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": "BASELINE config 2: DeBERTa-v3-large (24 layers) + GLiNER MLP, B=32, "
                                       "L=256 bucket, text lengths U[40,230], 1 task x 5 labels, random-init "
                                       "N(0,0.02) fp16 weights",
                           "batch_per_gpu": BATCH, "seq_len": SEQ, "parallelism": f"rows x{world} (no collective)",
                           "resident_batches": N_RESIDENT_BATCHES,
                           "rows": "packed: each batch row's positions up to its last valid token run through "
                                   "the encoder (logits bit-identical to the dense grid); "
                                   f"{rows_timed / args.steps:.0f} of {BATCH * SEQ} rows per step",
                           "l2": "no flush: each step streams 0.87 GB of weights (> 126 MB L2) and cycles "
                                 f"{N_RESIDENT_BATCHES} distinct input batches"},
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "api": "gdc_classify (host numpy int64 ids / fp16 mask / int64 markers / fp32 marker mask)"},
                "gpu_launches": launches_per_step * args.steps,
                "dense_grid": dense,
                "config4": c4,
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clk}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
