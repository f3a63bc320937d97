"""CPU tests of the parity oracle: pinned against the golden fixtures produced by
transformers' DebertaV2Model (tests/golden/make_golden.py), plus the bit-exact integer
pieces (relative buckets, gather tables, marker flattening, bucket selection, layout)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import load_golden
from oracle import reference_forward as rf


def _weights(g):
    from gliner_decide_metal_b200 import synthetic
    layers, vocab, seed = int(g["num_layers"]), int(g["vocab"]), int(g["weight_seed"])
    w = synthetic.make_weights(seed=seed, num_layers=layers, vocab=vocab)
    return rf.OracleWeights(w, rf.OracleConfig(num_hidden_layers=layers, vocab_size=vocab))


@pytest.mark.parametrize("name", ["ragged_B3_L40_2L", "logbucket_B2_L300_2L", "full_L512_1L"])
def test_oracle_matches_transformers_fixture(name):
    g = load_golden(name)
    W = _weights(g)
    logits, hidden = rf.forward(W, g["input_ids"], g["attention_mask"], g["marker_indices"], g["marker_mask"],
                                fp16_rounding=False, dtype=np.float64, return_hidden=True)
    B, L, E = hidden.shape
    flat = rf.flatten_marker_indices(g["marker_indices"], L)
    mh = hidden.reshape(B * L, E)[flat.reshape(-1)].reshape(g["marker_hidden"].shape)
    assert np.abs(mh - g["marker_hidden"]).max() < 1e-4
    assert np.abs(logits - g["logits"]).max() < 1e-4


@pytest.mark.slow
def test_oracle_matches_transformers_24_layers():
    """BASELINE config 0 on the full 24-layer model (vocabulary 128011)."""
    g = load_golden("config0_24L")
    W = _weights(g)
    logits = rf.forward(W, g["input_ids"], g["attention_mask"], g["marker_indices"], g["marker_mask"],
                        fp16_rounding=False, dtype=np.float64)
    assert np.abs(logits - g["logits"]).max() < 1e-4
    # fp16-rounding emulation stays inside the north-star logit tolerance
    l16 = rf.forward(W, g["input_ids"], g["attention_mask"], g["marker_indices"], g["marker_mask"])
    assert np.abs(l16 - g["logits"]).max() < 2e-2


def test_swapped_p2c_reading_disagrees_with_transformers():
    """Reading DeBERTa.swift:511 `transposed(0, 1)` as a swap (instead of mlx's identity
    permutation on a 2-D array) produces a different model: the fixture rejects it."""
    g = load_golden("ragged_B3_L40_2L")
    W = _weights(g)
    sw = rf.forward(W, g["input_ids"], g["attention_mask"], g["marker_indices"], g["marker_mask"],
                    fp16_rounding=False, dtype=np.float64, p2c_convention="swapped")
    assert np.abs(sw - g["logits"]).max() > 1e-3


def test_relative_bucket_identity_band_and_range():
    r = np.arange(-511, 512)
    b = rf.relative_bucket(r)
    assert np.array_equal(b[np.abs(r) <= 128], r[np.abs(r) <= 128])
    assert b.max() == 255 and b.min() == -255
    assert np.array_equal(b, -b[::-1])                      # odd function
    assert np.all(np.diff(b) >= 0)                           # monotone
    assert np.array_equal(rf.relative_bucket(r[r > 128]), rf.relative_bucket(r[r > 128]))


def test_relative_bucket_is_robust_to_log_rounding():
    """The ceil() argument never lies within 1e-9 of an integer, so libm differences in
    log() (Swift Double vs numpy float64 vs C double) cannot change a bucket. The one
    exception, |r| = 511, is exactly 127: numerator and denominator are the same log()."""
    assert rf.relative_bucket(np.array([511, -511])).tolist() == [255, -255]
    for a in list(range(129, 511)) + list(range(512, 1024)):
        x = math.log(a / 128) / math.log(511 / 128) * 127
        assert abs(x - round(x)) > 1e-9, a


def test_relative_bucket_matches_float32_variant():
    """transformers computes the same bucket in float32; identical for |r| < 512."""
    r = np.arange(-511, 512)
    mid = 128
    absr = np.where((r < mid) & (r > -mid), mid - 1, np.abs(r)).astype(np.float32)
    lp = np.ceil(np.log(absr / np.float32(mid)) / np.log(np.float32(511 / mid)) * np.float32(mid - 1)) + mid
    b32 = np.where(absr <= mid, r, lp * np.sign(r)).astype(np.int32)
    assert np.array_equal(b32, rf.relative_bucket(r))


def test_relative_indices_tables():
    for L in (1, 7, 128, 300, 512):
        c2p, p2c = rf.relative_indices(L)
        q = np.arange(L)[:, None]
        k = np.arange(L)[None, :]
        bucket = rf.relative_bucket(q - k)
        assert np.array_equal(c2p, np.clip(bucket + 256, 0, 511))
        # p2c[k, q] (gather index used at row k, column q) == 256 - bucket(k - q) == 256 + bucket(q - k)
        assert np.array_equal(p2c.T, c2p)
        assert c2p.min() >= 0 and c2p.max() <= 511


def test_flatten_marker_indices():
    mi = np.array([[[1, 4, 7]], [[2, 5, 0]], [[0, 0, 0]]])
    flat = rf.flatten_marker_indices(mi, 40)
    assert flat.tolist() == [[[1, 4, 7]], [[42, 45, 40]], [[80, 80, 80]]]


def test_layout_input_and_bucket_selection():
    ids, mask, mi, mm = rf.layout_input([5, 6, 7, 8, 9], [[1, 3], [2]], buckets=(8, 4, 8, 16))
    assert ids.tolist() == [[5, 6, 7, 8, 9, 0, 0, 0]]
    assert mask.dtype == np.float16 and mask.tolist() == [[1, 1, 1, 1, 1, 0, 0, 0]]
    assert mi.tolist() == [[[1, 3], [2, 0]]] and mm.tolist() == [[[1, 1], [1, 0]]]
    assert rf.select_bucket(32, (64, 32)) == 32
    assert rf.select_bucket(33, (32, 64, 64)) == 64
    with pytest.raises(ValueError):
        rf.select_bucket(513, (32, 512))
    with pytest.raises(ValueError):
        rf.layout_input([1, 2], [[]])


def test_decode_rules():
    lg = np.array([[2.0, 1.0, 0.5, -1.0], [-3.0, -2.0, -2.0, 0.0]])
    (p0, s0), (p1, s1) = rf.decode(lg, [3, 3], [False, True])
    assert s0 == [0] and abs(p0.sum() - 1) < 1e-12
    assert s1 == [1]  # all sigmoids < 0.5: first argmax among the 3 labels (tie -> first)
    (p2, s2), = rf.decode(np.array([[0.1, -0.2, 3.0]]), [3], [True])
    assert s2 == [0, 2]


def test_padding_past_the_extent_does_not_change_logits():
    """The premise of packed encoder rows, checked on the oracle: a row's logits are the same
    whether it is padded to its bucket or cut at its extent (last valid position or active
    marker + 1), because padded positions only ever act as masked keys (weight exactly 0).
    fp64, no fp16 rounding: a padded position that leaked would move the logits by far more
    than the 1e-6 allowed, which only covers BLAS summing a shorter row in another order."""
    from gliner_decide_metal_b200 import synthetic
    layers, vocab = 2, 500
    w = synthetic.make_weights(seed=3, num_layers=layers, vocab=vocab)
    W = rf.OracleWeights(w, rf.OracleConfig(num_hidden_layers=layers, vocab_size=vocab))
    rng = np.random.default_rng(8)
    L = 96
    for case in range(4):
        n = int(rng.integers(5, 60))
        ids = rng.integers(3, vocab, (1, L))
        ids[0, n:] = 0
        mask = np.zeros((1, L), np.float16)
        mask[0, :n] = 1
        if case == 3:
            mask[0, 2:4] = 0  # a hole inside the valid span
        mk = rng.integers(0, n, (1, 2, 3))
        mm = np.ones((1, 2, 3), np.float32)
        mm[0, 1, 2] = 0
        if case == 2:
            mk[0, 1, 1] = n + 7  # an active marker in the padding extends the extent
        ext = max(n, int(mk[mm > 0].max()) + 1)
        full = rf.forward(W, ids, mask, mk, mm, fp16_rounding=False, dtype=np.float64)
        cut = rf.forward(W, ids[:, :ext], mask[:, :ext], mk, mm, fp16_rounding=False, dtype=np.float64)
        np.testing.assert_allclose(cut, full, rtol=0, atol=1e-6)
        if case == 0:
            # control: dropping the last valid position does change the logits
            short = rf.forward(W, ids[:, :n - 1], mask[:, :n - 1], np.minimum(mk, n - 2), mm,
                               fp16_rounding=False, dtype=np.float64)
            assert np.abs(short - full)[mm > 0].max() > 1e-4
