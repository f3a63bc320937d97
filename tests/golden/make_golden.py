"""Generate the golden fixtures that pin the CPU oracle.

The reference's own golden logits (``Tools/prepare_model.py:183-229``) come from the
upstream PyTorch model: ``gliner2``'s encoder is ``transformers``' ``DebertaV2Model``
and its classifier is ``Linear -> ReLU -> Linear`` (weights ``classifier.0`` /
``classifier.2``). The real checkpoint is not available offline, so this script runs
``transformers`` 5.5.0 ``DebertaV2Model`` (the DeBERTa-v3-large configuration the
reference hard-codes, ``Configuration.swift:38-48``) on seeded random-init weights from
``gliner_decide_metal_b200.synthetic`` and applies the classifier exactly as
``prepare_model.py:527-544`` does (gather marker rows, classifier, ``-10000`` where the
marker mask is 0).

Fixtures store the inputs, the weight seed / shape parameters (weights are regenerated
deterministically by the tests), the final hidden state at every marker row and the
logits. Run from the repository root::

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from gliner_decide_metal_b200 import synthetic  # noqa: E402

OUT = Path(__file__).resolve().parent


def hf_model(weights: dict, num_layers: int, vocab: int, dtype):
    import torch
    from transformers import DebertaV2Config, DebertaV2Model

    cfg = DebertaV2Config(
        vocab_size=vocab, hidden_size=1024, num_hidden_layers=num_layers,
        num_attention_heads=16, intermediate_size=4096, hidden_act="gelu",
        max_position_embeddings=512, type_vocab_size=0, relative_attention=True,
        max_relative_positions=-1, position_buckets=256, pos_att_type=["p2c", "c2p"],
        norm_rel_ebd="layer_norm", share_att_key=True, position_biased_input=False,
        layer_norm_eps=1e-7, pad_token_id=0, attn_implementation="eager")
    model = DebertaV2Model(cfg)
    state = {k[len("encoder."):]: torch.from_numpy(v.astype(np.float32))
             for k, v in weights.items() if k.startswith("encoder.")}
    missing, unexpected = model.load_state_dict(state, strict=True), None
    model = model.to(dtype).eval()
    return model


def run_case(name, num_layers, vocab, wseed, ids, mask, mi, mm, dtype_name="float64"):
    import torch

    dtype = getattr(torch, dtype_name)
    w = synthetic.make_weights(seed=wseed, num_layers=num_layers, vocab=vocab)
    model = hf_model(w, num_layers, vocab, dtype)
    with torch.inference_mode():
        hidden = model(input_ids=torch.from_numpy(ids.astype(np.int64)),
                       attention_mask=torch.from_numpy(mask.astype(np.int64))).last_hidden_state
    hidden = hidden.to(torch.float64).numpy()
    B, L, E = hidden.shape
    flat = mi.astype(np.int64) + (np.arange(B) * L)[:, None, None]
    rows = hidden.reshape(B * L, E)[flat.reshape(-1)]
    w0 = w["classifier.0.weight"].astype(np.float64)
    b0 = w["classifier.0.bias"].astype(np.float64)
    w2 = w["classifier.2.weight"].astype(np.float64)
    b2 = w["classifier.2.bias"].astype(np.float64)
    v = (np.maximum(rows @ w0.T + b0, 0) @ w2.T + b2).reshape(mi.shape)
    logits = np.where(mm > 0, v, -10000.0)
    np.savez_compressed(
        OUT / f"{name}.npz", num_layers=num_layers, vocab=vocab, weight_seed=wseed,
        input_ids=ids.astype(np.int64), attention_mask=mask.astype(np.float16),
        marker_indices=mi.astype(np.int64), marker_mask=mm.astype(np.float32),
        marker_hidden=rows.reshape(*mi.shape, E).astype(np.float32),
        logits=logits.astype(np.float32), hf_dtype=dtype_name)
    print(name, "logits", logits.reshape(-1)[:6])


def ragged_inputs(rng, lengths, L, vocab, hm, o):
    B = len(lengths)
    ids = np.zeros((B, L), np.int64)
    mask = np.zeros((B, L), np.float16)
    mi = np.zeros((B, hm, o), np.int64)
    mm = np.zeros((B, hm, o), np.float32)
    for b, n in enumerate(lengths):
        ids[b, :n] = rng.integers(3, vocab, n)
        mask[b, :n] = 1
        for h in range(hm):
            k = int(rng.integers(1, o + 1))
            mi[b, h, :k] = rng.integers(0, n, k)
            mm[b, h, :k] = 1
    return ids, mask, mi, mm


def main():
    # 1) BASELINE config 0 on the full 24-layer model with the real vocabulary size.
    c0 = synthetic.config0(seed=1)
    run_case("config0_24L", 24, 128011, 0, c0.input_ids, c0.attention_mask,
             c0.marker_indices, c0.marker_mask, dtype_name="float32")
    rng = np.random.Generator(np.random.PCG64(11))
    # 2) ragged batch, padding, odd L, 2 layers
    ids, mask, mi, mm = ragged_inputs(rng, [40, 23, 7], 40, 1000, 2, 3)
    run_case("ragged_B3_L40_2L", 2, 1000, 7, ids, mask, mi, mm)
    # 3) L=300: relative distances beyond the 128 identity band (log buckets), padding
    ids, mask, mi, mm = ragged_inputs(rng, [300, 181], 300, 1000, 1, 4)
    run_case("logbucket_B2_L300_2L", 2, 1000, 8, ids, mask, mi, mm)
    # 4) L=512, full bucket range, one layer
    ids, mask, mi, mm = ragged_inputs(rng, [512], 512, 1000, 3, 2)
    run_case("full_L512_1L", 1, 1000, 9, ids, mask, mi, mm)


if __name__ == "__main__":
    main()
