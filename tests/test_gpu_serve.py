"""GPU end-to-end tests beyond the bench configuration: BASELINE config 3 (mixed buckets,
1-3 tasks of 2-12 labels, 30% multi-label) through the serving loop against the oracle, and
config 4 (256 rows at L=512, 24 layers) through size-independent properties."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import reference_forward as rf

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2
PROB_ATOL = 1e-3


@pytest.mark.parametrize("group_by", ["shape", "length", "stream"])
def test_config3_serving_loop_matches_oracle(weights_file, group_by):
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import serve, synthetic
    layers, vocab = 2, 128011
    path, w = weights_file(11, layers, vocab)
    model = g.GLiNERDecideClassifier(path, configuration=g.DeBERTaV2Configuration(num_hidden_layers=layers,
                                                                                  vocab_size=vocab))
    ex = []
    for i, (ids, markers, n_labels, ml) in enumerate(synthetic.mixed_rows(24, seed=21)):
        tasks = [g.DecisionTask(f"t{h}", tuple(f"l{j}" for j in range(n)), m) for h, (n, m) in
                 enumerate(zip(n_labels, ml))]
        ex.append(serve.TokenizedExample(f"r{i}", [int(x) for x in ids], tasks, [list(p) for p in markers]))
    res = serve.run_examples(model, ex, batch_size=8, group_by=group_by)
    W = rf.OracleWeights(w, rf.OracleConfig(num_hidden_layers=layers, vocab_size=vocab))
    buckets = set()
    for r, e in zip(res, ex):
        inp = g.make_input_from_tokens(e.token_ids, e.marker_positions)
        buckets.add(inp.shape[1])
        ref = rf.forward(W, inp.input_ids, inp.attention_mask, inp.marker_indices, inp.marker_mask)[0]
        dec = rf.decode(ref, [len(t.labels) for t in e.tasks], [t.multi_label for t in e.tasks])
        for p, t, (pr, sel) in zip(r.predictions, e.tasks, dec):
            n = len(t.labels)
            np.testing.assert_allclose(p.probabilities, pr[:n], atol=PROB_ATOL, rtol=0)
            want = [t.labels[j] for j in sel]
            if t.multi_label:
                tie = np.abs(np.asarray(pr[:n]) - 0.5).min() < 2e-3
            else:
                srt = np.sort(pr[:n])[::-1]
                tie = n > 1 and srt[0] - srt[1] < 2e-3
            if not tie:
                assert p.labels == want, (e.id, t.name)
    assert len(buckets) >= 3  # the rows spread over several buckets
    model.close()


def test_config4_full_size_properties(weights_file):
    """BASELINE config 4 (256 rows, L=512, text U[200,500], 24 layers): permuting rows
    permutes the logits bit-exactly, a row alone equals its row in the batch, and one row
    matches the fp16 oracle."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic
    c4 = synthetic.config4()
    path, w = weights_file(0, 24, 128011)
    model = g.GLiNERDecideClassifier(path)
    inp = g.DecisionInput(c4.input_ids, c4.attention_mask, c4.marker_indices, c4.marker_mask)
    full = model.classify(inp).logits_f32
    assert np.isfinite(full).all()
    perm = np.random.Generator(np.random.PCG64(1)).permutation(len(c4.input_ids))
    pinp = g.DecisionInput(c4.input_ids[perm], c4.attention_mask[perm], c4.marker_indices[perm],
                           c4.marker_mask[perm])
    assert np.array_equal(model.classify(pinp).logits_f32, full[perm])
    one = model.classify(g.DecisionInput(c4.input_ids[200:201], c4.attention_mask[200:201],
                                         c4.marker_indices[200:201], c4.marker_mask[200:201])).logits_f32
    assert np.array_equal(one[0], full[200])
    W = rf.OracleWeights(w, rf.OracleConfig())
    ref = rf.forward(W, c4.input_ids[200:201], c4.attention_mask[200:201], c4.marker_indices[200:201],
                     c4.marker_mask[200:201])
    np.testing.assert_allclose(full[200:201], ref, atol=LOGIT_ATOL, rtol=0)
    model.close()


def test_benchcli_batch_and_latency_modes(weights_file, tmp_path, capsys):
    """The main.swift mirror: batch mode with a padded last chunk returns every row's logits
    bit-identical to one classify of all rows; latency mode reports p50 / p95 / profile."""
    import gliner_decide_metal_b200 as g
    from conftest import load_golden
    from gliner_decide_metal_b200 import benchcli
    from gliner_decide_metal_b200.safetensors_io import load_file
    path, _ = weights_file(7, 2, 1000)
    gld = load_golden("ragged_B3_L40_2L")
    inp = g.DecisionInput(gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    inp.save(tmp_path / "in.safetensors")
    common = ["--weights", str(path), "--inputs", str(tmp_path / "in.safetensors"), "--layers", "2", "--vocab", "1000"]
    assert benchcli.main(common + ["--batch-size", "2", "--pad-batch", "--output", str(tmp_path / "b.safetensors")]) == 0
    out = capsys.readouterr().out
    assert "batch_count: 3" in out and "batch_rows_per_sec" in out
    with g.GLiNERDecideClassifier(path, configuration=g.DeBERTaV2Configuration(num_hidden_layers=2,
                                                                               vocab_size=1000)) as m:
        want = m.classify(inp).logits
    assert np.array_equal(load_file(tmp_path / "b.safetensors")["logits"], want)
    assert benchcli.main(common + ["--iterations", "5", "--warmup", "1", "--profile"]) == 0
    out = capsys.readouterr().out
    assert "p50_ms" in out and "p95_ms" in out and "layer_1_feed_forward" in out


def test_raw_text_serving_matches_oracle(weights_file, tmp_path):
    """RawExample lines through the native tokenizer (synthetic Unigram tokenizer.json built
    with the tokenizers library) and the serving loop, against the oracle on the same rows."""
    import json
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import serve
    from gliner_decide_metal_b200.tokenizer import NativeDecisionTokenizer
    from test_tokenizer import _synthetic
    tok = _synthetic(seed=4)
    tok.save(str(tmp_path / "tokenizer.json"))
    (tmp_path / "tokenizer_config.json").write_text(json.dumps({"tokenizer_class": "DebertaV2Tokenizer"}))
    nt = NativeDecisionTokenizer(tmp_path)
    layers, vocab = 2, 4096
    path, w = weights_file(13, layers, vocab)
    model = g.GLiNERDecideClassifier(path, configuration=g.DeBERTaV2Configuration(num_hidden_layers=layers,
                                                                                  vocab_size=vocab))
    rng = np.random.default_rng(3)
    words = ["good", "bad", "match", "team", "vote", "price", "rain", "sun", "great", "awful"]
    ex = []
    for i in range(12):
        text = " ".join(rng.choice(words, int(rng.integers(3, 40)))).capitalize()
        tasks = [g.DecisionTask("sentiment", ("positive", "negative", "neutral"), False),
                 g.DecisionTask("topic", ("sports", "politics", "weather", "money"), bool(i % 2), prompt="topic")]
        ex.append(serve.RawExample(f"r{i}", text, tasks[: 1 + i % 2]))
    res = serve.run_raw_examples(model, nt, ex, batch_size=4)
    W = rf.OracleWeights(w, rf.OracleConfig(num_hidden_layers=layers, vocab_size=vocab))
    for r, e in zip(res, ex):
        inp = nt.make_input(e.text, e.tasks)
        ref = rf.forward(W, inp.input_ids, inp.attention_mask, inp.marker_indices, inp.marker_mask)[0]
        dec = rf.decode(ref, [len(t.labels) for t in e.tasks], [t.multi_label for t in e.tasks])
        assert [p.task for p in r.predictions] == [t.name for t in e.tasks]
        for p, t, (pr, _) in zip(r.predictions, e.tasks, dec):
            np.testing.assert_allclose(p.probabilities, pr[:len(t.labels)], atol=PROB_ATOL, rtol=0)
    model.close()


def test_stream_serving_sharded_over_two_handles_matches_one(weights_file):
    """The serving loop's stream path with each chunk's rows split over two model handles
    (gdc_classify_sharded; both on device 0 here) gives the same predictions as one handle."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import serve, synthetic
    layers, vocab = 2, 128011
    path, _ = weights_file(11, layers, vocab)
    cfg = g.DeBERTaV2Configuration(num_hidden_layers=layers, vocab_size=vocab)
    models = [g.GLiNERDecideClassifier(path, configuration=cfg, device=0) for _ in range(2)]
    ex = []
    for i, (ids, markers, n_labels, ml) in enumerate(synthetic.mixed_rows(40, seed=31)):
        tasks = [g.DecisionTask(f"t{h}", tuple(f"l{j}" for j in range(n)), m) for h, (n, m) in
                 enumerate(zip(n_labels, ml))]
        ex.append(serve.TokenizedExample(f"r{i}", [int(x) for x in ids], tasks, [list(p) for p in markers]))
    one = serve.run_examples(models[0], ex, batch_size=16, group_by="stream")
    two = serve.run_examples(models, ex, batch_size=16, group_by="stream")
    for a, b in zip(one, two):
        assert a.id == b.id
        for pa, pb in zip(a.predictions, b.predictions):
            assert pa.labels == pb.labels
            np.testing.assert_allclose(pa.probabilities, pb.probabilities, rtol=0, atol=1e-6)
    for m in models:
        m.close()
