"""The reference's benchmark CLI (Sources/gliner-decide-metal/main.swift) on this backend.

Two modes, as there:

* latency (default): classify the whole input ``--iterations`` times after ``--warmup``
  runs and print ``p50_ms`` / ``p95_ms`` / ``mean_ms`` of the wall time the classifier
  reports (main.swift:287-312), optionally the per-stage profile of the last run;
* batch (``--batch-size N``): classify the rows in chunks of N, padding the last chunk to N
  by repeating its last row when ``--pad-batch`` is given and keeping only the valid rows'
  logits (``makeBatchChunk``, main.swift:7-51 and 241-284), then print ``batch_total_ms``
  and ``batch_rows_per_sec``.

``--output`` saves the logits (the last run's in latency mode, all rows in batch mode) to a
safetensors file under the key ``logits``, as the reference does. Without the reference's
checkpoint and sample inputs, ``--synthetic config0|config2|config4`` builds the BASELINE
configuration's seeded input and ``--write-weights`` creates seeded random weights at the
``--weights`` path when the file does not exist.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from typing import Tuple

import numpy as np

from . import DecisionInput, DeBERTaV2Configuration, GLiNERDecideClassifier
from .safetensors_io import save_file


def make_batch_chunk(inp: DecisionInput, start: int, end: int, pad_to: int) -> Tuple[DecisionInput, int]:
    """Rows [start, end) of ``inp``; when fewer than ``pad_to``, padded to ``pad_to`` rows by
    repeating the last valid row (main.swift:7-51). Returns (chunk, valid row count)."""
    if not 0 <= start < end <= inp.input_ids.shape[0]:
        raise ValueError(f"chunk [{start}, {end}) outside the {inp.input_ids.shape[0]} input rows")
    valid = end - start
    idx = np.arange(start, end)
    if valid < pad_to:
        idx = np.concatenate([idx, np.full(pad_to - valid, end - 1)])
    chunk = DecisionInput(inp.input_ids[idx], inp.attention_mask[idx], inp.marker_indices[idx], inp.marker_mask[idx])
    return chunk, valid


def run_batch(model, inp: DecisionInput, batch_size: int, pad_batch: bool, warmup: int = 3):
    """Batch mode: (logits of every row [B, Hm, O] fp16, total milliseconds)."""
    count = inp.input_ids.shape[0]
    if count <= 0 or batch_size <= 0:
        raise ValueError("batch mode needs at least one row and a positive batch size")
    if warmup > 0:
        warm_end = min(batch_size, count)
        warm, _ = make_batch_chunk(inp, 0, warm_end, batch_size if pad_batch else warm_end)
        for _ in range(max(1, warmup)):
            model.classify(warm)
    t0 = time.perf_counter()
    pieces = []
    for offset in range(0, count, batch_size):
        end = min(offset + batch_size, count)
        chunk, valid = make_batch_chunk(inp, offset, end, batch_size if pad_batch else end - offset)
        pieces.append(model.classify(chunk).logits[:valid])
    logits = np.concatenate(pieces, axis=0)
    return logits, (time.perf_counter() - t0) * 1e3


def run_latency(model, inp: DecisionInput, warmup: int = 3, iterations: int = 20, profile: bool = False):
    """Latency mode: (sorted wall milliseconds of each run, the last InferenceResult)."""
    for _ in range(max(0, warmup)):
        model.classify(inp)
    timings, last = [], None
    for _ in range(max(1, iterations)):
        last = model.classify(inp, collect_profile=profile)
        timings.append(last.wall_milliseconds)
    return sorted(timings), last


def percentiles(sorted_ms):
    """p50 and p95 with the reference's index rule (main.swift:297-299)."""
    n = len(sorted_ms)
    return sorted_ms[n // 2], sorted_ms[min(n - 1, int((n - 1) * 0.95))]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m gliner_decide_metal_b200.benchcli",
                                 description="latency / batch benchmark of the classifier (main.swift)")
    ap.add_argument("--weights", required=True)
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--inputs", help="safetensors with input_ids, attention_mask, marker_indices, marker_mask")
    src.add_argument("--synthetic", choices=("config0", "config2", "config4"), help="seeded BASELINE input")
    ap.add_argument("--write-weights", action="store_true", help="create seeded weights if --weights is missing")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iterations", type=int, default=20)
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--batch-size", type=int, default=0)
    ap.add_argument("--pad-batch", action="store_true")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--vocab", type=int, default=128011)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--output", default=None)
    args = ap.parse_args(argv)
    cfg = DeBERTaV2Configuration(num_hidden_layers=args.layers, vocab_size=args.vocab)
    if args.write_weights and not os.path.exists(args.weights):
        from . import synthetic
        synthetic.write_weights(args.weights, seed=0, num_layers=args.layers, vocab=args.vocab)
    if args.synthetic:
        from . import synthetic
        b = getattr(synthetic, args.synthetic)()
        inp = DecisionInput(b.input_ids, b.attention_mask, b.marker_indices, b.marker_mask)
    else:
        inp = DecisionInput.from_url(args.inputs)
    with GLiNERDecideClassifier(args.weights, configuration=cfg, device=args.device) as model:
        print(f"weights: {args.weights}")
        print(f"inputs: {args.inputs or args.synthetic} {inp.shape}")
        if args.batch_size > 0:
            logits, ms = run_batch(model, inp, args.batch_size, args.pad_batch, args.warmup)
            count = inp.input_ids.shape[0]
            print(f"batch_count: {count}")
            print(f"batch_total_ms: {ms:.3f}")
            print(f"batch_rows_per_sec: {count / (ms / 1e3):.3f}")
            if args.output:
                save_file({"logits": logits}, args.output)
                print(f"output: {args.output}")
            return 0
        timings, last = run_latency(model, inp, args.warmup, args.iterations, args.profile)
        p50, p95 = percentiles(timings)
        print(f"p50_ms: {p50:.3f}")
        print(f"p95_ms: {p95:.3f}")
        print(f"mean_ms: {sum(timings) / len(timings):.3f}")
        if args.profile:
            print("profile:")
            for e in last.events:
                print(f"  {e.name:<42s} {e.milliseconds:8.3f} ms")
        if args.output:
            save_file({"logits": last.logits}, args.output)
            print(f"output: {args.output}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
