"""Batch serving loop of the reference's raw CLI (RawCLI.swift:104-171) over pre-tokenised
examples.

The reference reads JSONL lines ``{id, text, tasks}``, tokenises each with
``NativeDecisionTokenizer.makeInput`` (NativeTokenizer.swift:76-264), groups the inputs by
``(L, maxHeads, maxOptions)``, classifies each group in chunks of ``batch_size`` rows,
decodes every row's tasks (RawCLI.swift:182-223) and writes a JSON array of results in
input order, each with the inference time of its batch divided by the batch size.

With ``--tokenizer DIR`` (a directory holding the checkpoint's ``tokenizer.json`` and
``tokenizer_config.json``) the lines are the reference's own ``RawExample`` JSON
(RawCLI.swift:11-15)::

    {"id": "...", "text": "...",
     "tasks": [{"name": "...", "labels": [...], "multiLabel": false,
                "prompt": "...", "labelDescriptions": {"label": "..."}}]}

and each one goes through ``NativeDecisionTokenizer.make_input`` (``tokenizer.py``), timed
as its preprocessing. Without a tokenizer the loop starts one step later: each line carries
the token ids the tokenizer would produce (schema + text, before padding) and the positions
of its ``[L]`` label markers per task::

    {"id": "...", "token_ids": [...],
     "tasks": [{"name": "...", "labels": [...], "multi_label": false, "marker_positions": [...]}]}

Bucket choice, padding and marker layout are the reference's (``gdc_layout_row``);
grouping, chunking, decoding and the output format are RawCLI's. ``--devices`` splits each
chunk's rows across GPUs (``gdc_classify_sharded``).

Output (``--output`` or stdout): the reference's JSON array
``[{"id", "predictions": [{"task", "labels", "probabilities"}], "preprocessingMilliseconds",
"inferenceMilliseconds"}]``. ``--synthetic-rows N`` replaces ``--jsonl`` with N seeded rows
of BASELINE config 3 (mixed buckets, 1-3 tasks of 2-12 labels, 30% multi-label); the total
rows per second of the run go to stderr.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import numpy as np

from . import (DEFAULT_BUCKETS, DecisionInput, DecisionTask, DeBERTaV2Configuration, GLiNERDecideClassifier,
               InputDoesNotFitError, NoTaskLabelsError, Prediction, classify_sharded, decode_batch,
               make_input_from_tokens)


@dataclass
class TokenizedExample:
    """One JSONL line after tokenisation: full token ids (schema + text, unpadded) and, per
    task, the positions of its label markers."""
    id: str
    token_ids: List[int]
    tasks: List[DecisionTask]
    marker_positions: List[List[int]]


@dataclass
class RawResult:
    id: str
    predictions: List[Prediction]
    preprocessing_ms: float
    inference_ms: float

    def to_json(self) -> dict:
        return {"id": self.id,
                "predictions": [{"task": p.task, "labels": list(p.labels), "probabilities": list(p.probabilities)}
                                for p in self.predictions],
                "preprocessingMilliseconds": self.preprocessing_ms,
                "inferenceMilliseconds": self.inference_ms}


def parse_example(obj: dict) -> TokenizedExample:
    tasks, markers = [], []
    for t in obj["tasks"]:
        tasks.append(DecisionTask(str(t["name"]), tuple(t["labels"]), bool(t.get("multi_label", False))))
        markers.append([int(p) for p in t["marker_positions"]])
    return TokenizedExample(str(obj["id"]), [int(x) for x in obj["token_ids"]], tasks, markers)


def load_jsonl(path) -> List[TokenizedExample]:
    with open(path, "r", encoding="utf-8") as f:
        return [parse_example(json.loads(line)) for line in f if line.strip()]


@dataclass
class RawExample:
    """``RawExample`` (RawCLI.swift:11-15): an id, the text and its decision tasks."""
    id: str
    text: str
    tasks: List[DecisionTask]


def parse_raw_example(obj: dict) -> RawExample:
    """The reference's JSON keys (``DecisionTask`` Codable: name, labels, multiLabel, prompt,
    labelDescriptions; ``multi_label`` is accepted too)."""
    tasks = []
    for t in obj["tasks"]:
        multi = t.get("multiLabel", t.get("multi_label", False))
        tasks.append(DecisionTask(str(t["name"]), tuple(str(x) for x in t["labels"]), bool(multi),
                                  t.get("prompt"), t.get("labelDescriptions", t.get("label_descriptions"))))
    return RawExample(str(obj["id"]), str(obj.get("text", "")), tasks)


def load_raw_jsonl(path) -> List[RawExample]:
    with open(path, "r", encoding="utf-8") as f:
        return [parse_raw_example(json.loads(line)) for line in f if line.strip()]


@dataclass
class _Pending:
    index: int
    example: object  # TokenizedExample or RawExample (id, tasks)
    input: DecisionInput
    preprocessing_ms: float


def _classify(models, inp: DecisionInput) -> Tuple[np.ndarray, float]:
    """fp32 view of the fp16 logits (as RawCLI's ``asType(.float32)``) and the batch's
    inference milliseconds."""
    if hasattr(models, "classify"):  # one model
        r = models.classify(inp)
        return r.logits_f32, r.wall_milliseconds
    if len(models) == 1:
        return _classify(models[0], inp)
    t0 = time.perf_counter()
    _, logits, _ = classify_sharded(models, inp)
    return logits, (time.perf_counter() - t0) * 1e3


def _decode_chunk(logits: np.ndarray, tasks_per_row: Sequence[Sequence[DecisionTask]]) -> List[List[Prediction]]:
    """``decode`` (RawCLI.swift:182-223) of a whole chunk with one ``gdc_decode`` call."""
    B, hm, _ = logits.shape
    nl = np.zeros((B, hm), np.int32)
    ml = np.zeros((B, hm), np.uint8)
    for r, tasks in enumerate(tasks_per_row):
        for h, t in enumerate(tasks):
            nl[r, h] = len(t.labels)
            ml[r, h] = int(t.multi_label)
    probs, sel = decode_batch(logits, nl, ml)
    out = []
    for r, tasks in enumerate(tasks_per_row):
        preds = []
        for h, t in enumerate(tasks):
            n = len(t.labels)
            preds.append(Prediction(t.name, [t.labels[i] for i in range(n) if sel[r, h, i]], probs[r, h, :n].tolist()))
        out.append(preds)
    return out


def _run_stream_tokens(models, examples: Sequence[TokenizedExample], buckets, batch_size: int) -> List[RawResult]:
    """``group_by="stream"`` over tokenised rows with the layout of ``gdc_layout_row``
    (NativeTokenizer.swift:134-157: smallest bucket, [PAD]=0 padding, mask, markers
    [h * O + o] for o < O) written for a whole chunk at once; each row's preprocessing time is
    its share of its chunk's layout time."""
    order = sorted(set(int(b) for b in buckets))
    if not order:
        raise InputDoesNotFitError(4, f"Encoded schema/text does not fit any requested bucket: {list(buckets)}")
    rows_L = []
    for ex in examples:
        if not ex.marker_positions or any(len(m) == 0 for m in ex.marker_positions):
            raise NoTaskLabelsError(5, "Every decision task must contain at least one label")
        n = len(ex.token_ids)
        L = next((b for b in order if b >= n), None)
        if L is None:
            raise InputDoesNotFitError(4, f"Encoded schema/text does not fit any requested bucket: {order}")
        rows_L.append(L)
    hm = max((len(ex.marker_positions) for ex in examples), default=1)
    o = max((len(m) for ex in examples for m in ex.marker_positions), default=1)

    def prepare(start: int):
        chunk = examples[start:start + batch_size]
        t0 = time.perf_counter()
        B, L = len(chunk), max(rows_L[start:start + batch_size])
        ids = np.zeros((B, L), np.int64)
        mask = np.zeros((B, L), np.float16)
        mi = np.zeros((B, hm, o), np.int64)
        mm = np.zeros((B, hm, o), np.float32)
        for r, ex in enumerate(chunk):
            n = len(ex.token_ids)
            ids[r, :n] = ex.token_ids
            mask[r, :n] = 1
            for h, pos in enumerate(ex.marker_positions):
                mi[r, h, :len(pos)] = pos
                mm[r, h, :len(pos)] = 1
        prep_ms = (time.perf_counter() - t0) * 1e3 / B
        return chunk, DecisionInput(ids, mask, mi, mm), [prep_ms] * B

    return _stream_pipeline(models, list(range(0, len(examples), batch_size)), prepare)


def _stream_pipeline(models, keys: Sequence, prepare) -> List[RawResult]:
    """The stream paths' chunk loop, pipelined: while chunk k is classified (in the C library,
    without the interpreter lock) one worker thread prepares chunk k+1 (``prepare(key)`` ->
    (rows, DecisionInput, per-row preprocessing ms)) and another decodes chunk k-1. Results
    come back in input order."""
    from concurrent.futures import ThreadPoolExecutor
    results: List[RawResult] = []
    if not keys:
        return results

    def finish(chunk, prep, logits, ms):
        return [RawResult(ex.id, preds, p_ms, ms / len(chunk))
                for ex, p_ms, preds in zip(chunk, prep, _decode_chunk(logits, [ex.tasks for ex in chunk]))]

    with ThreadPoolExecutor(max_workers=2) as pool:
        nxt = pool.submit(prepare, keys[0])
        done = None
        for k in range(len(keys)):
            chunk, inp, prep = nxt.result()
            if k + 1 < len(keys):
                nxt = pool.submit(prepare, keys[k + 1])
            logits, ms = _classify(models, inp)
            if done is not None:
                results.extend(done.result())
            done = pool.submit(finish, chunk, prep, logits, ms)
        results.extend(done.result())
    return results


def run_examples(models, examples: Sequence[TokenizedExample], buckets=DEFAULT_BUCKETS,
                 batch_size: int = 32, group_by: str = "shape") -> List[RawResult]:
    """RawCLI.runJSONL (RawCLI.swift:104-171) from the tokenised rows on: layout each row,
    group by (L, maxHeads, maxOptions), classify in chunks of ``batch_size``, decode."""
    if batch_size <= 0:
        raise ValueError("batch_size must be positive")
    if group_by == "stream":
        return _run_stream_tokens(models, examples, buckets, batch_size)
    pending: List[_Pending] = []
    for i, ex in enumerate(examples):
        t0 = time.perf_counter()
        inp = make_input_from_tokens(ex.token_ids, ex.marker_positions, buckets)
        pending.append(_Pending(i, ex, inp, (time.perf_counter() - t0) * 1e3))
    return _classify_pending(models, pending, batch_size, group_by)


def run_raw_examples(models, tokenizer, examples: Sequence[RawExample], buckets=DEFAULT_BUCKETS,
                     batch_size: int = 32, group_by: str = "shape") -> List[RawResult]:
    """RawCLI.runJSONL (RawCLI.swift:104-171) from the raw text: ``makeInput`` per row (its
    time is the row's preprocessing), then grouping, chunking and decoding as above."""
    if batch_size <= 0:
        raise ValueError("batch_size must be positive")
    if group_by == "stream":
        return _run_stream_raw(models, tokenizer, examples, buckets, batch_size)
    pending: List[_Pending] = []
    for i, ex in enumerate(examples):
        t0 = time.perf_counter()
        inp = tokenizer.make_input(ex.text, ex.tasks, buckets)
        pending.append(_Pending(i, ex, inp, (time.perf_counter() - t0) * 1e3))
    return _classify_pending(models, pending, batch_size, group_by)


def _run_stream_raw(models, tokenizer, examples: Sequence[RawExample], buckets, batch_size: int) -> List[RawResult]:
    """``group_by="stream"`` from raw text, pipelined (``_stream_pipeline``): chunk k+1 is
    tokenised and chunk k-1 decoded while chunk k is classified. The marker arrays' width
    comes from the tasks (tasks per row, labels per task), so every chunk has the same marker
    shape without tokenising ahead."""
    hm = max((len(ex.tasks) for ex in examples), default=1)
    o = max((len(t.labels) for ex in examples for t in ex.tasks), default=1)

    def prepare(start: int):
        chunk = examples[start:start + batch_size]
        inputs, prep = [], []
        for ex in chunk:
            t0 = time.perf_counter()
            inputs.append(tokenizer.make_input(ex.text, ex.tasks, buckets))
            prep.append((time.perf_counter() - t0) * 1e3)
        L = max(inp.shape[1] for inp in inputs)
        rows = [_pad_length(_pad_markers(inp, max(hm, inp.shape[2]), max(o, inp.shape[3])), L) for inp in inputs]
        return chunk, DecisionInput.concatenated(rows), prep

    return _stream_pipeline(models, list(range(0, len(examples), batch_size)), prepare)


def _pad_markers(inp: DecisionInput, hm: int, o: int) -> DecisionInput:
    """Marker arrays widened to [1, hm, o]; the new slots have mask 0 (logit -10000, never
    decoded), so the row's own logits do not change."""
    _, _, h0, o0 = inp.shape
    if (h0, o0) == (hm, o):
        return inp
    mi = np.zeros((1, hm, o), inp.marker_indices.dtype)
    mm = np.zeros((1, hm, o), inp.marker_mask.dtype)
    mi[:, :h0, :o0] = inp.marker_indices
    mm[:, :h0, :o0] = inp.marker_mask
    return DecisionInput(inp.input_ids, inp.attention_mask, mi, mm)


def _pad_length(inp: DecisionInput, L: int, pad_id: int = 0) -> DecisionInput:
    """A row padded to a longer bucket: [PAD] ids and mask 0 past its own bucket. A padded
    position is only a masked key, so the row's logits do not change."""
    L0 = inp.shape[1]
    if L0 == L:
        return inp
    ids = np.full((1, L), pad_id, inp.input_ids.dtype)
    mask = np.zeros((1, L), inp.attention_mask.dtype)
    ids[:, :L0] = inp.input_ids
    mask[:, :L0] = inp.attention_mask
    return DecisionInput(ids, mask, inp.marker_indices, inp.marker_mask)


def _classify_pending(models, pending: Sequence["_Pending"], batch_size: int,
                      group_by: str = "shape") -> List[RawResult]:
    """Batches the rows:
    * ``"shape"``: by (L, maxHeads, maxOptions), as RawCLI does;
    * ``"length"``: by bucket length, each chunk's marker arrays widened to its largest
      task / label counts;
    * ``"stream"``: in input order, each chunk padded to the bucket of its longest row and
      every chunk's marker arrays to the largest counts of the whole input (with packed
      encoder rows a row costs the same in any bucket; one batch shape, full batches).
    Every row's logits are the same in all three (added marker slots have mask 0, added
    positions are masked keys)."""
    if group_by not in ("shape", "length", "stream"):
        raise ValueError(f"group_by must be 'shape', 'length' or 'stream', got {group_by!r}")
    groups: Dict[Tuple[int, ...], List[_Pending]] = {}
    for p in pending:
        _, L, hm, o = p.input.shape
        key = (L, hm, o) if group_by == "shape" else ((L,) if group_by == "length" else ())
        groups.setdefault(key, []).append(p)
    results: List[RawResult] = [None] * len(pending)  # type: ignore[list-item]
    hm_all = max((p.input.shape[2] for p in pending), default=1)
    o_all = max((p.input.shape[3] for p in pending), default=1)
    for group in groups.values():
        for start in range(0, len(group), batch_size):
            batch = group[start:start + batch_size]
            if group_by == "stream":
                hm, o = hm_all, o_all
                L = max(p.input.shape[1] for p in batch)
                rows = [_pad_length(_pad_markers(p.input, hm, o), L) for p in batch]
            else:
                hm = max(p.input.shape[2] for p in batch)
                o = max(p.input.shape[3] for p in batch)
                rows = [_pad_markers(p.input, hm, o) for p in batch]
            inp = DecisionInput.concatenated(rows)
            logits, ms = _classify(models, inp)
            for p, preds in zip(batch, _decode_chunk(logits, [p.example.tasks for p in batch])):
                results[p.index] = RawResult(p.example.id, preds, p.preprocessing_ms, ms / len(batch))
    return results


def synthetic_examples(n: int, buckets=DEFAULT_BUCKETS, seed: int = 4) -> List[TokenizedExample]:
    """``n`` seeded BASELINE config 3 rows as tokenised examples."""
    from . import synthetic
    out = []
    for i, (ids, markers, n_labels, ml) in enumerate(synthetic.mixed_rows(n, seed=seed, buckets=buckets)):
        tasks = [DecisionTask(f"task{h}", tuple(f"label{j}" for j in range(k)), m)
                 for h, (k, m) in enumerate(zip(n_labels, ml))]
        out.append(TokenizedExample(f"row{i}", [int(x) for x in ids], tasks, [list(p) for p in markers]))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m gliner_decide_metal_b200.serve", description=__doc__.split("\n")[0])
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--jsonl", help="pre-tokenised examples, one JSON object per line")
    src.add_argument("--synthetic-rows", type=int, help="seeded BASELINE config 3 rows instead of --jsonl")
    ap.add_argument("--weights", required=True, help="fp16 safetensors weights")
    ap.add_argument("--tokenizer", default=None, help="directory with tokenizer.json / tokenizer_config.json: "
                                                       "--jsonl lines are RawExample {id, text, tasks}")
    ap.add_argument("--buckets", default=",".join(str(b) for b in DEFAULT_BUCKETS))
    ap.add_argument("--batch-size", type=int, default=32)
    ap.add_argument("--group-by", choices=("stream", "length", "shape"), default="stream",
                    help="stream: rows in input order, each chunk at its longest row's bucket; "
                         "length: rows of one bucket length; shape: one (L, maxHeads, maxOptions) "
                         "shape per batch as RawCLI")
    ap.add_argument("--devices", default="0", help="comma-separated CUDA devices; rows of a chunk are split")
    ap.add_argument("--layers", type=int, default=24, help="encoder layers in the weights file")
    ap.add_argument("--vocab", type=int, default=128011)
    ap.add_argument("--output", default=None)
    args = ap.parse_args(argv)
    buckets = [int(b) for b in args.buckets.split(",") if b]
    cfg = DeBERTaV2Configuration(num_hidden_layers=args.layers, vocab_size=args.vocab)
    models = [GLiNERDecideClassifier(args.weights, configuration=cfg, device=int(d)) for d in args.devices.split(",")]
    try:
        if args.tokenizer:
            from .tokenizer import NativeDecisionTokenizer
            if not args.jsonl:
                ap.error("--tokenizer reads --jsonl RawExample lines")
            tok = NativeDecisionTokenizer(args.tokenizer)
            examples = load_raw_jsonl(args.jsonl)

            def run(rows):
                return run_raw_examples(models, tok, rows, buckets, args.batch_size, args.group_by)
        else:
            examples = load_jsonl(args.jsonl) if args.jsonl else synthetic_examples(args.synthetic_rows, buckets)

            def run(rows):
                return run_examples(models, rows, buckets, args.batch_size, args.group_by)
        print(f"loaded {len(examples)} examples", file=sys.stderr)
        run(examples[:min(len(examples), args.batch_size)])  # warm-up
        t0 = time.perf_counter()
        results = run(examples)
        dt = time.perf_counter() - t0
        print(f"rows: {len(examples)} total_ms: {dt * 1e3:.1f} rows_per_sec: {len(examples) / dt:.1f}",
              file=sys.stderr)
    finally:
        for m in models:
            m.close()
    data = json.dumps([r.to_json() for r in results])
    if args.output:
        with open(args.output, "w", encoding="utf-8") as f:
            f.write(data)
    else:
        print(data)
    return 0


if __name__ == "__main__":
    sys.exit(main())
