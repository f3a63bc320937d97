"""Shared fixtures. GPU tests are marked ``gpu``; CPU tests run with ``-m "not gpu"``."""
from __future__ import annotations

import functools
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


@functools.lru_cache(maxsize=1)
def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def weights_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("weights")


_WEIGHTS_CACHE: dict = {}


@pytest.fixture(scope="session")
def weights_file(weights_dir):
    """weights_file(seed, layers, vocab) -> (path, numpy weights dict); cached per session."""
    from gliner_decide_metal_b200 import safetensors_io, synthetic

    def make(seed: int, layers: int, vocab: int):
        key = (seed, layers, vocab)
        if key not in _WEIGHTS_CACHE:
            w = synthetic.make_weights(seed=seed, num_layers=layers, vocab=vocab)
            path = weights_dir / f"w_s{seed}_l{layers}_v{vocab}.safetensors"
            safetensors_io.save_file(w, path)
            _WEIGHTS_CACHE[key] = (path, w)
        return _WEIGHTS_CACHE[key]

    return make


def load_golden(name: str):
    g = np.load(GOLDEN / f"{name}.npz")
    return {k: g[k] for k in g.files}


GOLDEN_CASES = ["ragged_B3_L40_2L", "logbucket_B2_L300_2L", "full_L512_1L", "config0_24L"]
