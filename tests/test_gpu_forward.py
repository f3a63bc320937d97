"""End-to-end parity of GLiNERDecideClassifier.classify on the GPU (C ABI) against the
golden fixtures (transformers DebertaV2 + GLiNER classifier on seeded weights) and the
fp16-emulating oracle, plus error paths and size-independent properties at the
benchmark's full size."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN_CASES, load_golden
from oracle import reference_forward as rf

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2   # logits within 2e-2 absolute
PROB_ATOL = 1e-3    # probabilities within 1e-3


def _model(weights_file, seed, layers, vocab):
    import gliner_decide_metal_b200 as g
    path, w = weights_file(seed, layers, vocab)
    cfg = g.DeBERTaV2Configuration(num_hidden_layers=layers, vocab_size=vocab)
    return g.GLiNERDecideClassifier(path, configuration=cfg), w


def _selections_agree(a, b, n_labels, multi, margin):
    """Label sets equal wherever the decision is not within `margin` of a tie."""
    import gliner_decide_metal_b200 as g
    pa, sa = g.decode_batch(a, n_labels, multi)
    pb, sb = g.decode_batch(b, n_labels, multi)
    B, Hm, O = a.shape
    for bi in range(B):
        for h in range(Hm):
            n = int(n_labels[bi, h])
            if n == 0:
                continue
            if multi[bi, h]:
                close = np.abs(pa[bi, h, :n] - 0.5).min() < margin
            else:
                srt = np.sort(a[bi, h, :n])[::-1]
                close = n > 1 and (srt[0] - srt[1]) < 2 * margin
            if not close:
                assert np.array_equal(sa[bi, h, :n], sb[bi, h, :n]), (bi, h, a[bi, h, :n], b[bi, h, :n])
    return pa, pb


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_golden_parity(name, weights_file):
    import gliner_decide_metal_b200 as g
    gld = load_golden(name)
    layers, vocab, seed = int(gld["num_layers"]), int(gld["vocab"]), int(gld["weight_seed"])
    model, w = _model(weights_file, seed, layers, vocab)
    inp = g.DecisionInput(gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    res = model.classify(inp)
    got = res.logits_f32
    assert got.shape == gld["logits"].shape
    assert np.isfinite(got).all()
    # marker slots with mask 0 are exactly -10000 (DeBERTa.swift:439-443)
    masked = gld["marker_mask"] <= 0
    assert (got[masked] == -10000.0).all()
    # vs transformers DebertaV2 (fp32/64) and vs the fp16-emulating oracle
    np.testing.assert_allclose(got, gld["logits"], atol=LOGIT_ATOL, rtol=0)
    W = rf.OracleWeights(w, rf.OracleConfig(num_hidden_layers=layers, vocab_size=vocab))
    ref16 = rf.forward(W, gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    np.testing.assert_allclose(got, ref16, atol=LOGIT_ATOL, rtol=0)
    # probabilities and label sets (single-label softmax over each head's valid options).
    # The parity target is the reference's own forward, which computes in fp16 between ops;
    # the fp16-emulating oracle stands for it, and the probabilities must agree with it
    # within 1e-3. The transformers fixture is an fp32 forward with no fp16 rounding, so
    # against it the bound is the fp16 rounding of 24 layers (at most 5e-3 on these cases).
    n_labels = (gld["marker_mask"] > 0).sum(-1).astype(np.int32)
    multi = np.zeros_like(n_labels, dtype=np.uint8)
    pa, pr = _selections_agree(got, ref16.astype(np.float32), n_labels, multi, 1e-3)
    assert np.abs(pa - pr).max() < PROB_ATOL
    pa, pb = _selections_agree(got, gld["logits"].astype(np.float32), n_labels, multi, 1e-3)
    assert np.abs(pa - pb).max() < 5 * PROB_ATOL
    model.close()


def test_config0_probabilities(weights_file):
    """BASELINE config 0 (B=1, L=32, 24 layers, 5 labels): probabilities within 1e-3 of
    the fp16-emulating oracle, same argmax."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic
    c0 = synthetic.config0()
    model, w = _model(weights_file, 0, 24, 128011)
    res = model.classify(g.DecisionInput(c0.input_ids, c0.attention_mask, c0.marker_indices, c0.marker_mask))
    W = rf.OracleWeights(w, rf.OracleConfig())
    ref = rf.forward(W, c0.input_ids, c0.attention_mask, c0.marker_indices, c0.marker_mask)
    np.testing.assert_allclose(res.logits_f32, ref, atol=LOGIT_ATOL, rtol=0)
    (p_ref, s_ref), = rf.decode(ref[0], [5], [False])
    preds = g.decode(res.logits_f32, [g.DecisionTask("t", tuple("abcde"))])
    assert np.abs(np.asarray(preds[0].probabilities) - p_ref).max() < PROB_ATOL
    model.close()


def test_error_paths(weights_file):
    import gliner_decide_metal_b200 as g
    model, _ = _model(weights_file, 7, 2, 1000)
    ids = np.full((1, 16), 5, np.int64)
    mask = np.ones((1, 16), np.float16)
    mi = np.zeros((1, 1, 2), np.int64)
    mm = np.ones((1, 1, 2), np.float32)
    bad = ids.copy()
    bad[0, 3] = 1000  # == vocab
    with pytest.raises(g.InvalidInputError):
        model.classify(g.DecisionInput(bad, mask, mi, mm))
    bad_m = mi.copy()
    bad_m[0, 0, 1] = 16
    with pytest.raises(g.InvalidInputError):
        model.classify(g.DecisionInput(ids, mask, bad_m, mm))
    with pytest.raises(g.GDCError) as e:
        model.classify(g.DecisionInput(np.zeros((1, 513), np.int64), np.ones((1, 513), np.float16), mi, mm))
    assert e.value.status_name == "GDC_ERR_UNSUPPORTED"
    # the model is still usable after errors
    r = model.classify(g.DecisionInput(ids, mask, mi, mm))
    assert np.isfinite(r.logits_f32).all()
    model.close()


def test_input_dtypes_stage_identically(weights_file):
    """Every supported host dtype of the four input arrays (typed staging for int32 / int64
    ids and markers, fp16 / u8 masks, fp32 marker masks; element-wise staging for the rest)
    gives the same logits bit for bit."""
    import gliner_decide_metal_b200 as g
    model, _ = _model(weights_file, 7, 2, 1000)
    gld = load_golden("ragged_B3_L40_2L")
    ids, mask, mi, mm = (gld[k] for k in ("input_ids", "attention_mask", "marker_indices", "marker_mask"))
    base = model.classify(g.DecisionInput(ids.astype(np.int32), mask.astype(np.float16), mi.astype(np.int32),
                                          mm.astype(np.float32))).logits_f32
    for ids_t in (np.int32, np.int64):
        for mask_t in (np.float16, np.float32, np.uint8, np.int32, np.int64):
            for mi_t in (np.int32, np.int64):
                for mm_t in (np.float32, np.float16, np.uint8):
                    got = model.classify(g.DecisionInput(ids.astype(ids_t), mask.astype(mask_t), mi.astype(mi_t),
                                                         mm.astype(mm_t))).logits_f32
                    assert np.array_equal(got, base), (ids_t, mask_t, mi_t, mm_t)
    # a bad id is still reported through the element-wise pass, with its position
    bad = ids.astype(np.int32)
    bad[1, 2] = 1000
    with pytest.raises(g.InvalidInputError, match=r"input_ids\[\d+\] = 1000"):
        model.classify(g.DecisionInput(bad, mask, mi, mm))
    model.close()


def test_profile_events_and_determinism(weights_file):
    import gliner_decide_metal_b200 as g
    model, _ = _model(weights_file, 7, 2, 1000)
    gld = load_golden("ragged_B3_L40_2L")
    inp = g.DecisionInput(gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    a = model.classify(inp, collect_profile=True)
    names = [e.name for e in a.events]
    assert names == ["embedding"] + [f"layer_{i}_{s}" for i in range(2) for s in
                                     ("attention_projection", "attention", "attention_output", "feed_forward")] + [
                         "classifier"]
    assert all(e.nanoseconds > 0 for e in a.events)
    b = model.classify(inp)
    assert np.array_equal(a.logits_f32, b.logits_f32)
    model.close()


def test_graph_replay_matches_eager(weights_file):
    """The first classify of a shape runs the kernels eagerly, the second captures a CUDA
    graph, later ones replay it: all bit-identical, also across an interleaved second
    shape and through gdc_classify_device with caller buffers at other addresses."""
    import torch
    import gliner_decide_metal_b200 as g
    model, _ = _model(weights_file, 7, 2, 1000)
    gld = load_golden("ragged_B3_L40_2L")
    inp = g.DecisionInput(gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    other = g.DecisionInput(gld["input_ids"][:2], gld["attention_mask"][:2], gld["marker_indices"][:2],
                            gld["marker_mask"][:2])
    runs = []
    for i in range(4):
        runs.append(model.classify(inp).logits_f32)
        if i == 1:
            assert np.array_equal(model.classify(other).logits_f32, model.classify(other).logits_f32)
    for r in runs[1:]:
        assert np.array_equal(runs[0], r)
    B, L = inp.input_ids.shape
    _, Hm, O = inp.marker_indices.shape
    dev = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (
        inp.input_ids.astype(np.int32), inp.attention_mask.astype(np.float16),
        inp.marker_indices.astype(np.int32), inp.marker_mask.astype(np.float32))]
    for _ in range(3):
        logits = torch.full((B, Hm, O), float("nan"), dtype=torch.float32, device="cuda")
        model.classify_device(B, L, Hm, O, *(t.data_ptr() for t in dev), logits.data_ptr(),
                              stream=model.stream)
        torch.cuda.synchronize()
        assert np.array_equal(logits.cpu().numpy(), runs[0])
    model.close()


def test_sharded_equals_single(weights_file):
    """classify_sharded over two handles (same device here) equals a single classify."""
    import gliner_decide_metal_b200 as g
    gld = load_golden("ragged_B3_L40_2L")
    m1, _ = _model(weights_file, 7, 2, 1000)
    path, _ = weights_file(7, 2, 1000)
    m2 = g.GLiNERDecideClassifier(path, configuration=g.DeBERTaV2Configuration(num_hidden_layers=2, vocab_size=1000))
    inp = g.DecisionInput(gld["input_ids"], gld["attention_mask"], gld["marker_indices"], gld["marker_mask"])
    single = m1.classify(inp).logits_f32
    _, sharded, st = g.classify_sharded([m1, m2], inp)
    assert st == [0, 0]
    assert np.array_equal(single, sharded)
    m1.close()
    m2.close()


def test_full_size_properties(weights_file):
    """BASELINE config 2 (B=32, L=256, 24 layers): rows are independent, so (a) permuting
    rows permutes the logits bit-exactly, (b) a row classified alone equals its row in the
    batch bit-exactly, (c) eight rows spread over the batch match the fp16 oracle within the
    logit tolerance, with probabilities within 1e-3 and the same argmax."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic
    c2 = synthetic.config2()
    model, w = _model(weights_file, 0, 24, 128011)
    inp = g.DecisionInput(c2.input_ids, c2.attention_mask, c2.marker_indices, c2.marker_mask)
    full = model.classify(inp).logits_f32
    perm = np.random.Generator(np.random.PCG64(0)).permutation(32)
    pinp = g.DecisionInput(c2.input_ids[perm], c2.attention_mask[perm], c2.marker_indices[perm],
                           c2.marker_mask[perm])
    assert np.array_equal(model.classify(pinp).logits_f32, full[perm])
    one = model.classify(g.DecisionInput(c2.input_ids[5:6], c2.attention_mask[5:6], c2.marker_indices[5:6],
                                         c2.marker_mask[5:6])).logits_f32
    assert np.array_equal(one[0], full[5])
    W = rf.OracleWeights(w, rf.OracleConfig())
    rows = [0, 4, 9, 13, 17, 22, 27, 31]
    ref = rf.forward(W, c2.input_ids[rows], c2.attention_mask[rows], c2.marker_indices[rows], c2.marker_mask[rows])
    np.testing.assert_allclose(full[rows], ref, atol=LOGIT_ATOL, rtol=0)
    n_labels = (c2.marker_mask[rows] > 0).sum(-1).astype(np.int32)
    multi = np.zeros_like(n_labels, dtype=np.uint8)
    pa, pr = _selections_agree(full[rows], ref.astype(np.float32), n_labels, multi, 1e-3)
    assert np.abs(pa - pr).max() < PROB_ATOL
    model.close()
