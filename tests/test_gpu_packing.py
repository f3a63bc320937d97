"""Packed encoder rows (padding removal) against the dense [B, L] grid on the GPU.

Each packed row is computed with the same K order, key tiles and relative windows as the
dense position it holds, so the two layouts must give bit-identical logits; the cases
cover ragged rows, rows without any valid token, masks with holes, active markers past
the last valid token, inactive markers past the extent, multi-tile lengths and the
captured-graph replay path."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _model(weights_file, layers=2, vocab=4096, seed=7):
    import gliner_decide_metal_b200 as g
    path, _ = weights_file(seed, layers, vocab)
    cfg = g.DeBERTaV2Configuration(num_hidden_layers=layers, vocab_size=vocab)
    return g.GLiNERDecideClassifier(path, configuration=cfg)


def _ragged(rng, B, L, Hm, O, vocab, lengths=None):
    import gliner_decide_metal_b200 as g
    ids = rng.integers(3, vocab, (B, L)).astype(np.int32)
    mask = np.zeros((B, L), np.float16)
    lens = rng.integers(1, L + 1, B) if lengths is None else np.asarray(lengths)
    markers = np.zeros((B, Hm, O), np.int32)
    mmask = np.zeros((B, Hm, O), np.float32)
    for b in range(B):
        n = int(lens[b])
        mask[b, :n] = 1
        ids[b, n:] = 0
        k = int(rng.integers(1, Hm * O + 1))
        pos = rng.choice(max(n, 1), size=min(k, max(n, 1)), replace=False)
        for j, p in enumerate(pos):
            markers[b, j // O, j % O] = p
            mmask[b, j // O, j % O] = 1
    return g.DecisionInput(ids, mask, markers, mmask)


def _both(model, inp):
    model.row_packing = False
    dense = model.classify(inp).logits.copy()
    model.row_packing = True
    packed = model.classify(inp).logits.copy()
    return dense, packed


@pytest.mark.parametrize("B,L", [(32, 256), (5, 512), (1, 32), (9, 96), (3, 384)])
def test_packed_equals_dense_ragged(weights_file, B, L):
    model = _model(weights_file)
    rng = np.random.default_rng(B * 1000 + L)
    inp = _ragged(rng, B, L, 2, 6, 4096)
    dense, packed = _both(model, inp)
    assert np.isfinite(dense.astype(np.float32)).all()
    assert np.array_equal(dense.view(np.uint16), packed.view(np.uint16))
    model.close()


def test_packed_equals_dense_edge_rows(weights_file):
    """Rows with no valid token (active markers included), a mask with holes, an active
    marker in the padding past the last valid token, an inactive marker past the extent,
    a full-length row, and a one-token row."""
    import gliner_decide_metal_b200 as g
    model = _model(weights_file)
    rng = np.random.default_rng(11)
    B, L, Hm, O = 7, 256, 2, 4
    inp = _ragged(rng, B, L, Hm, O, 4096, lengths=[0, 100, 60, 140, 256, 1, 129])
    ids, mask, mk, mm = inp.input_ids, inp.attention_mask, inp.marker_indices, inp.marker_mask
    mk[0, 0, :2] = [3, 200]
    mm[0, 0, :2] = 1                      # row 0: no valid token, active markers
    mask[1, 10:20] = 0                    # row 1: holes inside the valid span
    mask[1, 150] = 1                      # ... and one valid token far past the span
    mk[2, 1, 0], mm[2, 1, 0] = 230, 1.0   # row 2: active marker in the padding
    mk[3, 1, 3], mm[3, 1, 3] = 250, 0.0   # row 3: inactive marker past the extent
    ext, off = g.packed_row_layout(mask, mk, mm)
    assert list(ext) == [256, 151, 231, 140, 256, 1, 129]
    dense, packed = _both(model, inp)
    assert np.array_equal(dense.view(np.uint16), packed.view(np.uint16))
    assert (packed[mm <= 0].astype(np.float32) == -10000.0).all()
    model.close()


def test_packed_graph_replay_matches_dense(weights_file):
    """The second call of a shape captures a graph and later calls replay it: the packed
    layout is recomputed on the device from each call's mask, so new data of the same
    shape still matches the dense forward."""
    model = _model(weights_file)
    rng = np.random.default_rng(5)
    inputs = [_ragged(rng, 16, 256, 1, 5, 4096) for _ in range(4)]
    model.row_packing = False
    dense = [model.classify(x).logits.copy() for x in inputs]
    model.row_packing = True
    for rep in range(2):
        for x, d in zip(inputs, dense):
            got = model.classify(x).logits
            assert np.array_equal(d.view(np.uint16), got.view(np.uint16)), rep
    model.close()


def test_packed_full_model_config2(weights_file):
    """BASELINE config 2 on the 24-layer model: packed and dense logits identical."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic
    c2 = synthetic.config2()
    model = _model(weights_file, layers=24, vocab=128011, seed=0)
    inp = g.DecisionInput(c2.input_ids, c2.attention_mask, c2.marker_indices, c2.marker_mask)
    dense, packed = _both(model, inp)
    assert np.array_equal(dense.view(np.uint16), packed.view(np.uint16))
    ext, off = g.packed_row_layout(c2.attention_mask, c2.marker_indices, c2.marker_mask)
    assert off[-1] < 32 * 256
    model.close()


def _tail_split(rows: int, n: int, pairs: int, bn: int = 256, max_split: int = 4) -> int:
    """The pair GEMM's tail split for a device row count (kernels/gemm_pair.cu, PairTiles):
    the number of parts each tile of a sparse last wave is cut into (1 = no split)."""
    num_big = -(-rows // 256) * (n // bn)
    rem = num_big % pairs
    f = max_split
    while rem and f >= 2:
        if f * rem <= pairs:
            return f
        f //= 2
    return 1


def test_packed_equals_dense_through_gemm_tail_splits(weights_file):
    """Row lengths chosen so the packed batch spans 20 tiles of 256 rows: the out and
    FFN-down projections (N = 1024) and the QKV projection (N = 3072) then cut their last
    wave into quarter-width tiles and FFN-up (N = 4096) into half-width tiles, while the
    dense grid runs full-width tiles only. The logits must still be bit-identical."""
    import torch
    import gliner_decide_metal_b200 as g
    model = _model(weights_file)
    rng = np.random.default_rng(2024)
    B, L = 32, 256
    lengths = np.full(B, 156) + np.concatenate([d := rng.integers(-60, 61, B // 2), -d])
    inp = _ragged(rng, B, L, 1, 5, 4096, lengths=lengths)
    ext, off = g.packed_row_layout(inp.attention_mask, inp.marker_indices, inp.marker_mask)
    rows = int(off[-1])
    assert 19 * 256 < rows <= 20 * 256
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    assert _tail_split(rows, 1024, pairs) == 4
    assert _tail_split(rows, 3072, pairs) == 4
    assert _tail_split(rows, 4096, pairs) == 2
    assert _tail_split(B * L, 1024, pairs) == 1 and _tail_split(B * L, 4096, pairs) == 1
    dense, packed = _both(model, inp)
    assert np.isfinite(dense.astype(np.float32)).all()
    assert np.array_equal(dense.view(np.uint16), packed.view(np.uint16))
    model.close()
