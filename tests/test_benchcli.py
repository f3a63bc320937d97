"""CPU tests of the benchmark CLI helpers (main.swift): batch-chunk padding by repeating
the last row, batch mode keeping only valid rows, the p50 / p95 index rule."""
from __future__ import annotations

import numpy as np
import pytest

import gliner_decide_metal_b200 as g
from gliner_decide_metal_b200 import benchcli


def _input(n=5, L=8, hm=1, o=3):
    rng = np.random.Generator(np.random.PCG64(2))
    return g.DecisionInput(rng.integers(0, 100, (n, L)).astype(np.int64), np.ones((n, L), np.float16),
                           rng.integers(0, L, (n, hm, o)).astype(np.int64), np.ones((n, hm, o), np.float32))


class _Echo:
    """Logits encode the row's first id, so padding and row order are visible."""
    def __init__(self):
        self.shapes = []

    def classify(self, inp, collect_profile=False):
        b = inp.input_ids.shape[0]
        self.shapes.append(inp.shape)
        lg = np.broadcast_to(inp.input_ids[:, :1, None].astype(np.float16), (b,) + inp.marker_indices.shape[1:])
        return g.InferenceResult(np.array(lg), np.array(lg, np.float32), 1000 * (len(self.shapes)))


def test_make_batch_chunk_repeats_last_row():
    inp = _input()
    chunk, valid = benchcli.make_batch_chunk(inp, 3, 5, 4)
    assert valid == 2 and chunk.input_ids.shape[0] == 4
    assert np.array_equal(chunk.input_ids[:2], inp.input_ids[3:5])
    assert np.array_equal(chunk.input_ids[2], inp.input_ids[4]) and np.array_equal(chunk.input_ids[3], inp.input_ids[4])
    assert np.array_equal(chunk.marker_mask[3], inp.marker_mask[4])
    full, valid = benchcli.make_batch_chunk(inp, 0, 4, 4)
    assert valid == 4 and np.array_equal(full.input_ids, inp.input_ids[:4])
    with pytest.raises(ValueError):
        benchcli.make_batch_chunk(inp, 4, 6, 4)


@pytest.mark.parametrize("pad", [True, False])
def test_batch_mode_keeps_valid_rows_in_order(pad):
    inp = _input(n=7)
    m = _Echo()
    logits, _ = benchcli.run_batch(m, inp, 3, pad, warmup=1)
    assert logits.shape == (7, 1, 3)
    assert np.array_equal(logits[:, 0, 0], inp.input_ids[:, 0].astype(np.float16))
    sizes = [s[0] for s in m.shapes]
    assert sizes == ([3, 3, 3, 3] if pad else [3, 3, 3, 1])  # warm-up chunk, then 3 chunks


def test_percentile_rule():
    t = sorted(float(i) for i in range(20))
    assert benchcli.percentiles(t) == (10.0, 18.0)
    assert benchcli.percentiles([5.0]) == (5.0, 5.0)
