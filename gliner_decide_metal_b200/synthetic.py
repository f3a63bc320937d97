"""Seeded synthetic weights and inputs for the BASELINE configurations.

The real ``fastino/GLiNER2.5-Decide`` checkpoint, its tokenizer and the
``fastino/fast-decisions`` dataset are not available offline, so benchmarks and tests
use random-init weights with the checkpoint's key names and shapes
(``DeBERTa.swift:128-148,199-208,228-229``; ``Tools/prepare_model.py:82-98``) and
token-id rows laid out like the reference's schema formatter
(``NativeTokenizer.swift:90-157``).

Token ids used for the schema's special tokens (the real tokenizer ids are not
available; any id below the vocabulary size is equivalent for the forward):
``[PAD]=0, [CLS]=1, [SEP]=2, [P]=128001, [L]=128002, [SEP_STRUCT]=128003,
[SEP_TEXT]=128004, "("=128005, ")"=128006``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .safetensors_io import save_file

PAD, CLS, SEP = 0, 1, 2
TOK_P, TOK_L, TOK_SEP_STRUCT, TOK_SEP_TEXT, TOK_OPEN, TOK_CLOSE = (
    128001, 128002, 128003, 128004, 128005, 128006)
DEFAULT_BUCKETS = (32, 64, 96, 128, 256, 512)
CLASSIFIER_HIDDEN = 2048  # GLiNER2 classification MLP: hidden -> 2*hidden -> 1


def weight_shapes(num_layers: int = 24, hidden: int = 1024, intermediate: int = 4096,
                  vocab: int = 128011, classifier_hidden: int = CLASSIFIER_HIDDEN):
    """(key, shape, kind) for every tensor of the classification checkpoint, in file
    order. kind is 'w' (N(0, 0.02)), 'g' (LayerNorm gamma = 1) or 'b' (LayerNorm beta = 0)."""
    out = [("encoder.embeddings.word_embeddings.weight", (vocab, hidden), "w"),
           ("encoder.embeddings.LayerNorm.weight", (hidden,), "g"),
           ("encoder.embeddings.LayerNorm.bias", (hidden,), "b"),
           ("encoder.encoder.rel_embeddings.weight", (512, hidden), "w"),
           ("encoder.encoder.LayerNorm.weight", (hidden,), "g"),
           ("encoder.encoder.LayerNorm.bias", (hidden,), "b")]
    for i in range(num_layers):
        p = f"encoder.encoder.layer.{i}"
        for n in ("query", "key", "value"):
            out.append((f"{p}.attention.self.{n}_proj.weight", (hidden, hidden), "w"))
            out.append((f"{p}.attention.self.{n}_proj.bias", (hidden,), "w"))
        out += [(f"{p}.attention.output.dense.weight", (hidden, hidden), "w"),
                (f"{p}.attention.output.dense.bias", (hidden,), "w"),
                (f"{p}.attention.output.LayerNorm.weight", (hidden,), "g"),
                (f"{p}.attention.output.LayerNorm.bias", (hidden,), "b"),
                (f"{p}.intermediate.dense.weight", (intermediate, hidden), "w"),
                (f"{p}.intermediate.dense.bias", (intermediate,), "w"),
                (f"{p}.output.dense.weight", (hidden, intermediate), "w"),
                (f"{p}.output.dense.bias", (hidden,), "w"),
                (f"{p}.output.LayerNorm.weight", (hidden,), "g"),
                (f"{p}.output.LayerNorm.bias", (hidden,), "b")]
    out += [("classifier.0.weight", (classifier_hidden, hidden), "w"),
            ("classifier.0.bias", (classifier_hidden,), "w"),
            ("classifier.2.weight", (1, classifier_hidden), "w"),
            ("classifier.2.bias", (1,), "w")]
    return out


def make_weights(seed: int = 0, num_layers: int = 24, vocab: int = 128011,
                 std: float = 0.02, classifier_hidden: int = CLASSIFIER_HIDDEN) -> dict:
    """Random-init fp16 weights: N(0, std) for matrices, embeddings and biases;
    LayerNorm gamma = 1, beta = 0. Deterministic in ``seed``."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for key, shape, kind in weight_shapes(num_layers, vocab=vocab, classifier_hidden=classifier_hidden):
        if kind == "g":
            out[key] = np.ones(shape, np.float16)
        elif kind == "b":
            out[key] = np.zeros(shape, np.float16)
        else:
            out[key] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float16)
    return out


def write_weights(path, seed: int = 0, num_layers: int = 24, vocab: int = 128011) -> dict:
    w = make_weights(seed, num_layers, vocab)
    save_file(w, path, metadata={"precision": "float16", "scope": "encoder+classification-only",
                                 "source": f"synthetic seed={seed}"})
    return w


@dataclass
class Batch:
    """One ``DecisionInput`` worth of arrays plus the task descriptors per row."""
    input_ids: np.ndarray       # int64 [B, L]
    attention_mask: np.ndarray  # fp16 [B, L]
    marker_indices: np.ndarray  # int64 [B, Hm, O]
    marker_mask: np.ndarray     # fp32 [B, Hm, O]
    n_labels: np.ndarray        # int32 [B, Hm] labels per task (0 = no task)
    multi_label: np.ndarray     # uint8 [B, Hm]


def _schema_row(rng, tasks, text_len, vocab_hi=128000):
    """Token ids of one row laid out like NativeTokenizer.swift:90-133 (schema groups,
    [SEP_STRUCT] between tasks, [SEP_TEXT], text). Each prompt / label text is two ids."""
    ids = []
    markers = []
    for t, n_lab in enumerate(tasks):
        ids += [TOK_OPEN, TOK_P] + list(rng.integers(1000, vocab_hi, 2)) + [TOK_OPEN]
        pos = []
        for _ in range(n_lab):
            pos.append(len(ids))
            ids += [TOK_L] + list(rng.integers(1000, vocab_hi, 2))
        ids += [TOK_CLOSE, TOK_CLOSE]
        markers.append(pos)
        if t < len(tasks) - 1:
            ids.append(TOK_SEP_STRUCT)
    ids.append(TOK_SEP_TEXT)
    ids += list(rng.integers(1000, vocab_hi, text_len))
    return ids, markers


def _stack(rows, L, hm, o):
    B = len(rows)
    ids = np.zeros((B, L), np.int64)
    mask = np.zeros((B, L), np.float16)
    mi = np.zeros((B, hm, o), np.int64)
    mm = np.zeros((B, hm, o), np.float32)
    for b, (tok, markers) in enumerate(rows):
        ids[b, :len(tok)] = tok
        mask[b, :len(tok)] = 1
        for h, pos in enumerate(markers):
            for j, p in enumerate(pos):
                mi[b, h, j] = p
                mm[b, h, j] = 1
    return ids, mask, mi, mm


def config0(seed: int = 1) -> Batch:
    """B=1, L=32: [CLS], 5 x ([L] + 2 ids), [SEP], text to fill 32."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ids = [CLS]
    markers = []
    for _ in range(5):
        markers.append(len(ids))
        ids += [TOK_L] + list(rng.integers(1000, 128000, 2))
    ids.append(SEP)
    ids += list(rng.integers(1000, 128000, 32 - len(ids)))
    a, m, mi, mm = _stack([(ids, [markers])], 32, 1, 5)
    return Batch(a, m, mi, mm, np.array([[5]], np.int32), np.zeros((1, 1), np.uint8))


def fixed_batch(batch: int, seq_len: int, text_lo: int, text_hi: int, seed: int,
                n_labels: int = 5) -> Batch:
    """BASELINE configs 2 and 4: one single-label task of ``n_labels`` labels
    (3 tokens each: marker + 2 ids) after [CLS]; text length U[text_lo, text_hi];
    right-padded to ``seq_len``."""
    rng = np.random.Generator(np.random.PCG64(seed))
    rows = []
    for _ in range(batch):
        ids = [CLS]
        pos = []
        for _ in range(n_labels):
            pos.append(len(ids))
            ids += [TOK_L] + list(rng.integers(1000, 128000, 2))
        ids.append(SEP)
        t = int(rng.integers(text_lo, text_hi + 1))
        ids += list(rng.integers(1000, 128000, t))
        ids = ids[:seq_len]
        rows.append((ids, [pos]))
    a, m, mi, mm = _stack(rows, seq_len, 1, n_labels)
    return Batch(a, m, mi, mm, np.full((batch, 1), n_labels, np.int32), np.zeros((batch, 1), np.uint8))


def config2(seed: int = 3) -> Batch:
    """B=32, L=256, text length U[40, 230], 1 task x 5 labels."""
    return fixed_batch(32, 256, 40, 230, seed)


def config4(rows_per_gpu: int = 256, seed: int = 5) -> Batch:
    """256 rows per GPU, L=512, text length U[200, 500]."""
    return fixed_batch(rows_per_gpu, 512, 200, 500, seed)


def mixed_rows(n_rows: int, seed: int = 4, buckets=DEFAULT_BUCKETS):
    """BASELINE config 3 rows: text length log-uniform [8, 480], 1-3 tasks of 2-12 labels,
    30% multi-label. Rows whose schema + text exceed the largest bucket get their text
    truncated to fit (the reference would reject them with inputDoesNotFit). Returns a
    list of (token_ids, marker_positions, n_labels list, multi_label list)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    top = max(buckets)
    for _ in range(n_rows):
        n_tasks = int(rng.integers(1, 4))
        tasks = [int(rng.integers(2, 13)) for _ in range(n_tasks)]
        ml = [bool(rng.random() < 0.3) for _ in range(n_tasks)]
        text_len = int(round(math.exp(rng.uniform(math.log(8), math.log(480)))))
        ids, markers = _schema_row(rng, tasks, text_len)
        if len(ids) > top:
            ids = ids[:top]
        out.append((ids, markers, tasks, ml))
    return out
