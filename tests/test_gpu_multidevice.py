"""Row sharding across physical GPUs: gdc_classify_sharded with one model handle per device
(one host thread per device, host gather of the logits) against a single-device classify.

Rows are independent (DeBERTa.swift:274-447 has no cross-row term) and every kernel computes
a row the same way whatever else is in its batch, so the sharded logits must equal the
single-device ones bit for bit. Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _devices():
    import torch
    return torch.cuda.device_count()


@pytest.fixture(scope="module")
def models(weights_file):
    n = _devices()
    if n < 2:
        pytest.skip(f"needs two GPUs, {n} visible")
    import gliner_decide_metal_b200 as g
    path, _ = weights_file(0, 24, 128011)
    ms = [g.GLiNERDecideClassifier(path, device=d) for d in range(n)]
    yield ms
    for m in ms:
        m.close()


def test_handles_sit_on_distinct_devices(models):
    from gliner_decide_metal_b200._lib import lib
    assert [lib.gdc_model_device(m.handle) for m in models] == list(range(len(models)))


@pytest.mark.parametrize("config", ["config2", "config4"])
def test_sharded_over_devices_equals_one_device(models, config):
    """BASELINE config 2 (B=32, L=256) and config 4 (256 rows, L=512) split over every visible
    GPU (and over the first two) give the single-device logits bit for bit."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import synthetic
    b = getattr(synthetic, config)()
    inp = g.DecisionInput(b.input_ids, b.attention_mask, b.marker_indices, b.marker_mask)
    single = models[0].classify(inp).logits_f32
    for group in (models[:2], models):
        l16, l32, st = g.classify_sharded(group, inp)
        assert st == [0] * len(group)
        assert np.isfinite(l32).all()
        assert np.array_equal(l32, single)
        assert np.array_equal(l16.astype(np.float32), single)
