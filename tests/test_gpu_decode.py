"""gdc_decode_device (the on-device per-task softmax / sigmoid) against the oracle's
restatement of RawCLI.swift:182-223 and the host gdc_decode, through the C ABI.

Rules checked: multi-label tasks take the unshifted sigmoid and select every label with
p >= 0.5, else the first argmax; single-label tasks take the max-subtracted softmax and
select the first argmax; only the first n_labels options of a task are decoded, and the
rest of its slots (and tasks with n_labels = 0) stay at probability 0, not selected."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import reference_forward as rf

pytestmark = pytest.mark.gpu


def _cases():
    """(logits [B, Hm, O] float32, n_labels [B, Hm], multi_label [B, Hm])."""
    rng = np.random.Generator(np.random.PCG64(41))
    B, Hm, O = 64, 3, 12
    # logits on the fp16 grid, as the classifier emits them
    logits = (rng.standard_normal((B, Hm, O)) * 3).astype(np.float16).astype(np.float32)
    n_labels = rng.integers(0, O + 1, (B, Hm)).astype(np.int32)
    multi = (rng.random((B, Hm)) < 0.4).astype(np.uint8)
    # masked slots past each task's labels carry the classifier's -10000 fill
    for b in range(B):
        for h in range(Hm):
            logits[b, h, n_labels[b, h]:] = -10000.0
    # hand-made rows
    logits[0, 0, :4] = [0.0, 0.0, 0.0, 0.0]            # sigmoid exactly 0.5: every label selected
    n_labels[0, 0], multi[0, 0] = 4, 1
    logits[0, 1, :5] = [-1.0, -0.5, -0.5, -2.0, -3.0]  # all below 0.5: first argmax (index 1) of a tie
    n_labels[0, 1], multi[0, 1] = 5, 1
    logits[0, 2, :3] = [2.0, 2.0, 1.0]                 # softmax tie: first argmax
    n_labels[0, 2], multi[0, 2] = 3, 0
    logits[1, 0, :3] = [-10000.0, -10000.0, -10000.0]  # every label masked, single-label: uniform
    n_labels[1, 0], multi[1, 0] = 3, 0
    logits[1, 1, :3] = [-10000.0, -800.0, -10000.0]    # sigmoid underflows to 0 for all: first index
    n_labels[1, 1], multi[1, 1] = 3, 1
    logits[1, 2, :2] = [9.0, 40.0]                     # sigmoid rounds to 1 in float64 for 40
    n_labels[1, 2], multi[1, 2] = 2, 1
    logits[2, 0, :6] = [1e-3, -1e-3, 0.2, 0.2, -0.2, 0.0]
    n_labels[2, 0], multi[2, 0] = 6, 1
    n_labels[2, 1] = 0                                 # no task in this slot
    n_labels[2, 2], multi[2, 2] = 1, 0                 # one label: probability 1
    return logits, n_labels, multi


def test_decode_device_matches_reference_rules_and_host_decode():
    import torch
    from gliner_decide_metal_b200._lib import lib
    logits, n_labels, multi = _cases()
    B, Hm, O = logits.shape
    # a model handle is required by the entry point (device and default stream)
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import safetensors_io, synthetic
    import tempfile
    from pathlib import Path
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "w.safetensors"
        safetensors_io.save_file(synthetic.make_weights(seed=5, num_layers=1, vocab=64), path)
        with g.GLiNERDecideClassifier(path, configuration=g.DeBERTaV2Configuration(num_hidden_layers=1,
                                                                                    vocab_size=64)) as model:
            dl = torch.from_numpy(logits).cuda()
            dn = torch.from_numpy(n_labels).cuda()
            dm = torch.from_numpy(multi).cuda()
            dp = torch.full((B, Hm, O), float("nan"), dtype=torch.float32, device="cuda")
            ds = torch.full((B, Hm, O), 7, dtype=torch.uint8, device="cuda")
            st = lib.gdc_decode_device(model._h, dl.data_ptr(), B, Hm, O, dn.data_ptr(), dm.data_ptr(),
                                       dp.data_ptr(), ds.data_ptr(), None)
            assert st == 0, lib.gdc_last_error().decode()
            model.check_errors()
            probs = dp.cpu().numpy()
            sel = ds.cpu().numpy()
    # host decode (float64) through the C ABI
    hp = np.zeros((B, Hm, O), np.float64)
    hs = np.zeros((B, Hm, O), np.uint8)
    st = lib.gdc_decode(logits.ctypes.data, B, Hm, O, n_labels.ctypes.data, multi.ctypes.data, hp.ctypes.data,
                        hs.ctypes.data)
    assert st == 0
    assert np.array_equal(sel, hs)
    # probabilities: float64 results stored as float32
    assert np.abs(probs.astype(np.float64) - hp).max() <= 1e-6
    # the oracle's restatement, task by task (the reference decodes only tasks that have labels;
    # a slot with n_labels = 0 stays empty)
    for b in range(B):
        for h in range(Hm):
            n = int(n_labels[b, h])
            assert not sel[b, h, n:].any() and not probs[b, h, n:].any()
            if n == 0:
                continue
            (p_ref, sel_ref), = rf.decode(logits[b, h:h + 1], [n], [int(multi[b, h])])
            np.testing.assert_allclose(probs[b, h, :n], p_ref, rtol=0, atol=1e-6)
            assert sorted(np.flatnonzero(sel[b, h, :n]).tolist()) == sorted(sel_ref), (b, h)
    # the hand-made rows
    assert sel[0, 0, :4].tolist() == [1, 1, 1, 1]
    assert sel[0, 1, :5].tolist() == [0, 1, 0, 0, 0]
    assert sel[0, 2, :3].tolist() == [1, 0, 0]
    assert sel[1, 0, :3].tolist() == [1, 0, 0]
    np.testing.assert_allclose(probs[1, 0, :3], [1 / 3] * 3, rtol=0, atol=1e-7)
    assert sel[1, 1, :3].tolist() == [1, 0, 0]
    assert sel[1, 2, :2].tolist() == [1, 1]
    assert not sel[2, 1].any() and not probs[2, 1].any()
    assert sel[2, 2, 0] == 1 and probs[2, 2, 0] == 1.0
