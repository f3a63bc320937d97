"""CPU tests of the C-ABI library's host side: it loads, exports every symbol declared in
include/gdc.h, and its host logic (bucket selection, row layout, decode, relative index
table, weight-file parsing and error codes) matches the oracle. No GPU calls."""
from __future__ import annotations

import re
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import reference_forward as rf

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol():
    import ctypes

    from gliner_decide_metal_b200 import _lib
    header = (ROOT / "include" / "gdc.h").read_text()
    declared = set(re.findall(r"\b(gdc_[a-z0-9_]+)\s*\(", header))
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, missing
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert declared == bound, (declared ^ bound)
    assert _lib.lib.gdc_abi_version() == 1


def test_select_bucket_matches_oracle():
    import gliner_decide_metal_b200 as g
    rng = np.random.Generator(np.random.PCG64(0))
    for _ in range(300):
        buckets = [int(x) for x in rng.integers(1, 600, rng.integers(1, 7))]
        n = int(rng.integers(0, 700))
        try:
            want = rf.select_bucket(n, buckets)
        except ValueError:
            with pytest.raises(g.InputDoesNotFitError):
                g.select_bucket(n, buckets)
            continue
        assert g.select_bucket(n, buckets) == want
    with pytest.raises(g.InputDoesNotFitError):
        g.select_bucket(1, [])


def test_layout_row_matches_oracle():
    import gliner_decide_metal_b200 as g
    rng = np.random.Generator(np.random.PCG64(1))
    for _ in range(100):
        n = int(rng.integers(1, 520))
        toks = rng.integers(0, 128000, n).tolist()
        n_tasks = int(rng.integers(1, 4))
        markers = [sorted(rng.integers(0, n, int(rng.integers(1, 13))).tolist()) for _ in range(n_tasks)]
        try:
            want = rf.layout_input(toks, markers, pad_id=0)
        except ValueError:
            with pytest.raises(g.InputDoesNotFitError):
                g.make_input_from_tokens(toks, markers)
            continue
        got = g.make_input_from_tokens(toks, markers)
        for a, b in zip((got.input_ids, got.attention_mask, got.marker_indices, got.marker_mask), want):
            assert a.dtype == b.dtype and np.array_equal(a, b)
    with pytest.raises(g.NoTaskLabelsError):
        g.make_input_from_tokens([1, 2, 3], [])
    with pytest.raises(g.NoTaskLabelsError):
        g.make_input_from_tokens([1, 2, 3], [[1], []])


def test_decode_matches_oracle():
    import gliner_decide_metal_b200 as g
    rng = np.random.Generator(np.random.PCG64(2))
    B, Hm, O = 16, 3, 12
    logits = (rng.standard_normal((B, Hm, O)) * 3).astype(np.float32)
    n_labels = rng.integers(0, O + 1, (B, Hm)).astype(np.int32)
    multi = (rng.random((B, Hm)) < 0.3).astype(np.uint8)
    probs, sel = g.decode_batch(logits, n_labels, multi)
    for b in range(B):
        tasks = [(h, int(n_labels[b, h])) for h in range(Hm) if n_labels[b, h] > 0]
        if not tasks:
            continue
        ref = rf.decode(logits[b][[h for h, _ in tasks]], [n for _, n in tasks],
                        [bool(multi[b, h]) for h, _ in tasks])
        for (h, n), (p, s) in zip(tasks, ref):
            np.testing.assert_allclose(probs[b, h, :n], p, rtol=0, atol=1e-12)
            assert np.flatnonzero(sel[b, h, :n]).tolist() == s
            assert (probs[b, h, n:] == 0).all() and (sel[b, h, n:] == 0).all()
    preds = g.decode(logits[0], [g.DecisionTask("t", tuple("abcdefghijkl"[:5]), multi_label=False)])
    assert len(preds) == 1 and len(preds[0].probabilities) == 5


def test_relative_index_table_bit_exact():
    import gliner_decide_metal_b200 as g
    r = np.arange(-511, 512)
    assert np.array_equal(g.relative_index_table(), np.clip(rf.relative_bucket(r) + 256, 0, 511))


def _write_safetensors(path, tensors, header_override=None, truncate=0):
    import json
    header = {}
    off = 0
    blobs = []
    for k, a in tensors.items():
        header[k] = {"dtype": "F16", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(a.tobytes())
    if header_override:
        header.update(header_override)
    raw = json.dumps(header).encode()
    data = b"".join(blobs)
    Path(path).write_bytes(struct.pack("<Q", len(raw)) + raw + data[:len(data) - truncate])


def _load_status(path, layers=1, vocab=64):
    import ctypes

    from gliner_decide_metal_b200._lib import GdcConfig, lib
    cfg = GdcConfig()
    lib.gdc_config_default(ctypes.byref(cfg))
    cfg.num_hidden_layers = layers
    cfg.vocab_size = vocab
    h = ctypes.c_void_p()
    st = lib.gdc_model_load(str(path).encode(), ctypes.byref(cfg), 0, ctypes.byref(h))
    if st == 0:
        lib.gdc_model_free(h)
    return st, lib.gdc_last_error().decode()


def _tiny_weights(layers=1, vocab=64):
    from gliner_decide_metal_b200 import synthetic
    return synthetic.make_weights(seed=1, num_layers=layers, vocab=vocab)


def test_model_load_error_codes(tmp_path):
    """WeightStoreError mirrors: missing key -> 1, wrong shape -> 2; broken files -> 6.
    (A valid file fails only at the device step when no GPU is present.)"""
    w = _tiny_weights()
    p = tmp_path / "missing.safetensors"
    w2 = dict(w)
    del w2["encoder.encoder.layer.0.output.dense.bias"]
    _write_safetensors(p, w2)
    st, msg = _load_status(p)
    assert st == 1 and "encoder.encoder.layer.0.output.dense.bias" in msg

    p = tmp_path / "shape.safetensors"
    w3 = dict(w)
    w3["encoder.encoder.rel_embeddings.weight"] = np.zeros((511, 1024), np.float16)
    _write_safetensors(p, w3)
    st, msg = _load_status(p)
    assert st == 2 and "rel_embeddings" in msg

    p = tmp_path / "vocab.safetensors"
    _write_safetensors(p, w)
    st, msg = _load_status(p, vocab=65)  # the reference hard-checks the embedding row count
    assert st == 2 and "word_embeddings" in msg

    p = tmp_path / "trunc.safetensors"
    _write_safetensors(p, w, truncate=10)
    st, msg = _load_status(p)
    assert st == 6 and "truncated" in msg

    # a weight of the right shape stored as an integer type -> invalid shape (not a float type)
    import json as _json
    p = tmp_path / "dtype.safetensors"
    ent = "encoder.encoder.layer.0.output.dense.bias"
    w4 = dict(w)
    w4[ent] = np.zeros(1024, np.int64)  # 8-byte elements; the header below says I64
    _write_safetensors(p, w4)
    raw = p.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = _json.loads(raw[8:8 + n])
    hdr[ent]["dtype"] = "I64"
    new_raw = _json.dumps(hdr).encode()
    p.write_bytes(struct.pack("<Q", len(new_raw)) + new_raw + raw[8 + n:])
    st, msg = _load_status(p)
    assert st == 2 and "I64" in msg, (st, msg)
    # an unknown dtype name -> I/O (format) error
    hdr[ent]["dtype"] = "Q7"
    new_raw = _json.dumps(hdr).encode()
    p.write_bytes(struct.pack("<Q", len(new_raw)) + new_raw + raw[8 + n:])
    assert _load_status(p)[0] == 6

    p = tmp_path / "garbage.safetensors"
    p.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json at all")
    assert _load_status(p)[0] == 6
    assert _load_status(tmp_path / "nope.safetensors")[0] == 6


def test_model_load_without_gpu_reports_cuda_error(tmp_path):
    from conftest import gpu_available
    if gpu_available():
        pytest.skip("GPU present")
    p = tmp_path / "ok.safetensors"
    _write_safetensors(p, _tiny_weights())
    st, msg = _load_status(p)
    assert st == 7, msg


def test_safetensors_roundtrip_and_decision_input(tmp_path):
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import safetensors_io
    a = {"x": np.arange(6, dtype=np.float16).reshape(2, 3), "y": np.arange(4, dtype=np.int64)}
    safetensors_io.save_file(a, tmp_path / "a.safetensors", metadata={"k": "v"})
    b = safetensors_io.load_file(tmp_path / "a.safetensors")
    assert all(np.array_equal(a[k], b[k]) and a[k].dtype == b[k].dtype for k in a)
    inp = g.make_input_from_tokens([1, 2, 3, 4], [[1, 2]])
    inp.save(tmp_path / "in.safetensors")
    back = g.DecisionInput.from_url(tmp_path / "in.safetensors")
    assert np.array_equal(back.input_ids, inp.input_ids) and back.attention_mask.dtype == np.float16
    safetensors_io.save_file({"input_ids": inp.input_ids}, tmp_path / "bad.safetensors")
    with pytest.raises(g.InvalidInputError):
        g.DecisionInput.from_url(tmp_path / "bad.safetensors")


def test_classify_argument_checks_need_no_gpu():
    """Null handles are rejected before any device work."""
    import ctypes

    from gliner_decide_metal_b200._lib import GdcOutput, lib
    out = GdcOutput()
    assert lib.gdc_classify(None, None, 0, ctypes.byref(out)) == 11
    assert lib.gdc_check_errors(None) == 11
    assert lib.gdc_decode(None, 1, 1, 1, None, None, None, None) == 11


def test_packed_row_layout_rule():
    """Extent rule of the packed encoder rows: last valid position or active marker + 1,
    the full length for a row with no valid position; offsets are the prefix sums."""
    import gliner_decide_metal_b200 as g
    mask = np.zeros((4, 8), np.float16)
    mask[0, :3] = 1
    mask[1, [0, 5]] = 1          # hole
    mask[3, :8] = 1
    mk = np.zeros((4, 1, 2), np.int64)
    mm = np.zeros((4, 1, 2), np.float32)
    mk[0, 0] = [1, 6]
    mm[0, 0] = [1, 1]            # active marker past the last valid token
    mk[1, 0] = [7, 2]
    mm[1, 0] = [0, 1]            # inactive marker past the extent does not count
    mk[2, 0] = [4, 9]
    mm[2, 0] = [1, 1]            # no valid position: full length
    ext, off = g.packed_row_layout(mask, mk, mm)
    assert list(ext) == [7, 6, 8, 8]
    assert list(off) == [0, 7, 13, 21, 29]


def test_decode_edge_cases_match_oracle():
    """Decode edges (RawCLI.swift:182-223): exact ties pick the first label, a logit of 0
    (sigmoid 0.5) is selected, a multi-label task with every sigmoid below 0.5 falls back to
    its argmax, and -10000 fills and huge magnitudes stay finite."""
    import gliner_decide_metal_b200 as g
    cases = [
        ([1.0, 1.0, 0.5], False), ([2.0, 3.0, 3.0, 1.0], False), ([0.0, -1.0], True),
        ([-3.0, -2.0, -2.0], True), ([-10000.0, -10000.0, -10000.0], False), ([-10000.0, -10000.0], True),
        ([80.0, -80.0, 0.0], False), ([1e4, -1e4], True), ([0.0, 0.0, 0.0, 0.0], False), ([0.0, 0.0], True),
    ]
    O = max(len(c) for c, _ in cases)
    for vals, multi in cases:
        logits = np.full((1, 1, O), -10000.0, np.float32)
        logits[0, 0, :len(vals)] = vals
        probs, sel = g.decode_batch(logits, np.array([[len(vals)]], np.int32), np.array([[int(multi)]], np.uint8))
        (p, s), = rf.decode(logits[0][[0]], [len(vals)], [multi])
        np.testing.assert_allclose(probs[0, 0, :len(vals)], p, rtol=0, atol=1e-12)
        assert np.flatnonzero(sel[0, 0, :len(vals)]).tolist() == s, (vals, multi)
        assert np.isfinite(probs).all()
