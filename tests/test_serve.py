"""CPU tests of the batch serving loop (gliner_decide_metal_b200/serve.py, RawCLI.swift:104-171):
grouping by (L, maxHeads, maxOptions), chunking, input-order results, decode and the JSON
format, with a stand-in model whose logits are a fixed function of the input."""
from __future__ import annotations

import json

import numpy as np

import gliner_decide_metal_b200 as g
from gliner_decide_metal_b200 import serve, synthetic


class _FakeModel:
    def __init__(self):
        self.batches = []

    def classify(self, inp):
        b, L, hm, o = inp.shape
        self.batches.append((b, L, hm, o))
        lg = (np.asarray(inp.marker_indices, np.float32) * 0.05 - 2.0
              + np.asarray(inp.input_ids[:, :1], np.float32)[:, :, None] * 1e-6)
        lg = np.where(np.asarray(inp.marker_mask) > 0, lg, -10000.0).astype(np.float16)
        return g.InferenceResult(lg, lg.astype(np.float32), 1_000_000 * b)


def _examples(n, seed=4):
    out = []
    for i, (ids, markers, n_labels, ml) in enumerate(synthetic.mixed_rows(n, seed=seed)):
        tasks = [g.DecisionTask(f"task{h}", tuple(f"l{h}_{j}" for j in range(n)), m)
                 for h, (n, m) in enumerate(zip(n_labels, ml))]
        out.append(serve.TokenizedExample(f"row{i}", [int(x) for x in ids], tasks, [list(p) for p in markers]))
    return out


def test_groups_chunks_and_keeps_input_order():
    ex = _examples(40)
    model = _FakeModel()
    res = serve.run_examples(model, ex, batch_size=4)
    assert [r.id for r in res] == [e.id for e in ex]
    assert all(b <= 4 for b, *_ in model.batches)
    assert sum(b for b, *_ in model.batches) == len(ex)
    shapes = {}
    for e in ex:
        inp = g.make_input_from_tokens(e.token_ids, e.marker_positions)
        shapes.setdefault(inp.shape[1:], 0)
        shapes[inp.shape[1:]] += 1
    seen = {}
    for b, L, hm, o in model.batches:
        seen[(L, hm, o)] = seen.get((L, hm, o), 0) + b
    assert seen == shapes  # one group per (L, maxHeads, maxOptions), every row once
    for r, e in zip(res, ex):
        inp = g.make_input_from_tokens(e.token_ids, e.marker_positions)
        lg = model.classify(inp).logits_f32
        want = g.decode(lg, e.tasks, 0)
        assert [p.task for p in r.predictions] == [t.name for t in e.tasks]
        for p, w in zip(r.predictions, want):
            assert p.labels == w.labels
            np.testing.assert_allclose(p.probabilities, w.probabilities, rtol=0, atol=0)
        assert r.inference_ms == 1.0  # the batch's time split over its rows


def test_jsonl_round_trip_and_output_format(tmp_path):
    ex = _examples(6, seed=9)
    path = tmp_path / "rows.jsonl"
    with open(path, "w") as f:
        for e in ex:
            f.write(json.dumps({"id": e.id, "token_ids": e.token_ids, "tasks": [
                {"name": t.name, "labels": list(t.labels), "multi_label": t.multi_label, "marker_positions": m}
                for t, m in zip(e.tasks, e.marker_positions)]}) + "\n")
    back = serve.load_jsonl(path)
    assert [(b.id, b.token_ids, b.marker_positions) for b in back] == [(e.id, e.token_ids, e.marker_positions)
                                                                       for e in ex]
    assert [[(t.name, t.labels, t.multi_label) for t in b.tasks] for b in back] == \
        [[(t.name, t.labels, t.multi_label) for t in e.tasks] for e in ex]
    out = [r.to_json() for r in serve.run_examples(_FakeModel(), back)]
    assert set(out[0]) == {"id", "predictions", "preprocessingMilliseconds", "inferenceMilliseconds"}
    assert set(out[0]["predictions"][0]) == {"task", "labels", "probabilities"}
    json.dumps(out)


def test_group_by_length_gives_the_same_predictions():
    """Batching rows of one bucket length with widened marker arrays: fewer batches, the
    same predictions and probabilities for every row."""
    ex = _examples(60, seed=7)
    m1, m2 = _FakeModel(), _FakeModel()
    by_shape = serve.run_examples(m1, ex, batch_size=8)
    by_len = serve.run_examples(m2, ex, batch_size=8, group_by="length")
    assert len(m2.batches) < len(m1.batches)
    assert {L for _, L, _, _ in m2.batches} == {L for _, L, _, _ in m1.batches}
    for a, b in zip(by_shape, by_len):
        assert a.id == b.id
        assert [(p.task, p.labels, p.probabilities) for p in a.predictions] == \
            [(p.task, p.labels, p.probabilities) for p in b.predictions]


def test_group_by_stream_pads_chunks_and_keeps_predictions():
    """Rows in input order, each chunk at its longest row's bucket with the marker arrays of
    the whole input: one batch per chunk, the same predictions for every row."""
    ex = _examples(50, seed=9)
    m1, m2 = _FakeModel(), _FakeModel()
    by_shape = serve.run_examples(m1, ex, batch_size=8)
    by_stream = serve.run_examples(m2, ex, batch_size=8, group_by="stream")
    assert len(m2.batches) == 7 and [b for b, *_ in m2.batches] == [8] * 6 + [2]
    assert len({(hm, o) for _, _, hm, o in m2.batches}) == 1
    for a, b in zip(by_shape, by_stream):
        assert a.id == b.id
        assert [(p.task, p.labels, p.probabilities) for p in a.predictions] == \
            [(p.task, p.labels, p.probabilities) for p in b.predictions]


def test_stream_layout_matches_gdc_layout_row():
    """The stream path's chunk layout equals make_input_from_tokens (gdc_layout_row) row by
    row, padded to the chunk's bucket and the input's marker counts."""
    ex = _examples(70, seed=12)
    model = _FakeModel()
    captured = []
    orig = model.classify

    def spy(inp):
        captured.append(inp)
        return orig(inp)
    model.classify = spy
    serve.run_examples(model, ex, batch_size=16, group_by="stream")
    k = 0
    for inp in captured:
        B, L, hm, o = inp.shape
        for r in range(B):
            one = g.make_input_from_tokens(ex[k].token_ids, ex[k].marker_positions)
            _, L1, h1, o1 = one.shape
            assert L1 <= L and h1 <= hm and o1 <= o
            assert np.array_equal(inp.input_ids[r, :L1], one.input_ids[0])
            assert (inp.input_ids[r, L1:] == 0).all() and (inp.attention_mask[r, L1:] == 0).all()
            assert np.array_equal(inp.attention_mask[r, :L1], one.attention_mask[0])
            assert np.array_equal(inp.marker_indices[r, :h1, :o1], one.marker_indices[0])
            assert np.array_equal(inp.marker_mask[r, :h1, :o1], one.marker_mask[0])
            assert inp.marker_mask[r, h1:].sum() == 0 and inp.marker_mask[r, :, o1:].sum() == 0
            k += 1
    assert k == len(ex)


def test_stream_errors_match_layout_errors():
    import pytest
    ex = _examples(3)
    bad = serve.TokenizedExample("x", ex[0].token_ids, ex[0].tasks, [[]])
    with pytest.raises(g.NoTaskLabelsError):
        serve.run_examples(_FakeModel(), [bad], group_by="stream")
    with pytest.raises(g.InputDoesNotFitError):
        serve.run_examples(_FakeModel(), ex, buckets=[8], group_by="stream")
