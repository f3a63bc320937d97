"""CPU restatement of the GLiNER2.5-Decide classification forward (TEST INFRASTRUCTURE).

This module is the parity oracle. It is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline / reference arm,
and only as the checker or as the timed CPU baseline. The product path
(``gliner_decide_metal_b200``) never calls it.

It restates, in numpy, the reference's MLX forward of
``Sources/GLiNERDecideCore/DeBERTa.swift`` (shantanugoel/gliner-decide-metal):

* relative-position buckets ........ DeBERTa.swift:521-551 (``makeRelativePositions``)
* c2p / p2c index tables ........... DeBERTa.swift:498-519 (``cachedRelativeData``)
* init-time relative LN + PQ/PK .... DeBERTa.swift:204-227
* embedding stage .................. DeBERTa.swift:285-292
* QKV split ........................ DeBERTa.swift:298-320
* disentangled attention ........... DeBERTa.swift:322-395 (default fast path: fp16
  relative bias, additive -65504 key mask, SDPA with scale 1/sqrt(192))
* attention output + residual LN ... DeBERTa.swift:412-418, 449-464
* feed-forward ..................... DeBERTa.swift:420-427 (exact-erf GELU)
* classifier ....................... DeBERTa.swift:430-444 (marker gather, MLP, -10000 fill)

Arithmetic lives in mlx-swift (revision 901941965d82e4a216d4d117231d847d194c563d,
Package.swift:16-19), which is not vendored; its ops are restated from their
published semantics: ``addMM(c, a, b) = c + a @ b``; ``MLXFast.layerNorm`` normalises
the last axis with fp32 statistics; ``MLXNN.gelu`` is ``0.5 x (1 + erf(x / sqrt 2))``;
``takeAlong`` gathers along an axis; ``transposed(axes...)`` is an axis PERMUTATION
(so ``transposed(0, 1)`` of a 2-D array, DeBERTa.swift:511, is the identity).

Two precisions:

* ``fp16_rounding=True``: every MLX op output is rounded to fp16 at the point the
  reference materialises an fp16 array (all weights/activations are fp16 in the
  reference, ``prepare_model.py:88-90``). Softmax inside SDPA runs in fp32.
* ``fp16_rounding=False``: float32 end to end (used to pin this restatement against
  ``transformers``' ``DebertaV2Model``, the model the reference's own golden logits
  come from, ``Tools/prepare_model.py:183-229``).

Parity pin: ``tests/golden/make_golden.py`` runs ``transformers`` 5.5.0
``DebertaV2Model`` on the same seeded weights and inputs; ``tests/test_oracle.py``
checks this module against those fixtures.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# ---------------------------------------------------------------------------
# Configuration (Configuration.swift:38-48)
# ---------------------------------------------------------------------------


@dataclass
class OracleConfig:
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    layer_norm_eps: float = 1e-7
    position_buckets: int = 256
    # DeBERTa.swift:505 hard-codes 512 for the bucket function and :352/:371 use a
    # 512-row position table; the configuration's -1 is never read on this path.
    max_relative_positions: int = 512
    vocab_size: int = 128011

    @property
    def head_size(self) -> int:
        return self.hidden_size // self.num_attention_heads


# ---------------------------------------------------------------------------
# Relative positions (DeBERTa.swift:498-551)
# ---------------------------------------------------------------------------


def relative_bucket(relative: np.ndarray, position_buckets: int = 256,
                    max_relative_positions: int = 512) -> np.ndarray:
    """Log-bucketed relative position, DeBERTa.swift:526-547, in float64 like Swift's
    ``Double`` ``log``/``ceil``. ``relative`` is an integer array of ``q - k``."""
    r = np.asarray(relative, dtype=np.int64)
    mid = position_buckets // 2
    abs_pos = np.where((r > -mid) & (r < mid), mid - 1, np.abs(r)).astype(np.int64)
    log_pos = np.ceil(
        np.log(abs_pos.astype(np.float64) / float(mid))
        / np.log(np.float64(max_relative_positions - 1) / float(mid))  # same log() as the numerator:
        # at |r| = 511 the ratio is then exactly 1 and ceil(127.0) = 127, as in Swift
        * float(mid - 1)
    ).astype(np.int64) + mid
    sign = np.where(r < 0, -1, 1)
    return np.where(abs_pos <= mid, r, log_pos * sign).astype(np.int32)


def relative_positions(seq_len: int, position_buckets: int = 256,
                       max_relative_positions: int = 512) -> np.ndarray:
    """[L, L] int32 table ``pos[q, k] = bucket(q - k)`` (DeBERTa.swift:529-550)."""
    q = np.arange(seq_len)[:, None]
    k = np.arange(seq_len)[None, :]
    return relative_bucket(q - k, position_buckets, max_relative_positions)


def relative_indices(seq_len: int, position_buckets: int = 256,
                     max_relative_positions: int = 512, p2c_convention: str = "mlx"):
    """c2p and p2c gather tables (DeBERTa.swift:507-515), each [L, L] int32 in [0, 511].

    ``c2p = clip(pos + 256, 0, 511)``. The p2c table is
    ``clip(-p2cBase + 256, 0, 511)`` with ``p2cBase = positions[0].squeezed(axis: 0)
    .transposed(0, 1)``; mlx-swift's ``transposed(0, 1)`` on a 2-D array is the identity
    permutation, so ``p2c = clip(-pos + 256)`` (``p2c_convention="mlx"``).
    ``p2c_convention="swapped"`` builds ``clip(-pos.T + 256)`` instead; it exists only so
    tests can show that this reading disagrees with ``transformers``.
    """
    pos = relative_positions(seq_len, position_buckets, max_relative_positions)
    span = position_buckets
    c2p = np.clip(pos + span, 0, 2 * span - 1).astype(np.int32)
    if p2c_convention == "mlx":
        base = pos
    elif p2c_convention == "swapped":
        base = pos.T
    else:
        raise ValueError(p2c_convention)
    p2c = np.clip(-base + span, 0, 2 * span - 1).astype(np.int32)
    return c2p, p2c


# ---------------------------------------------------------------------------
# Weights
# ---------------------------------------------------------------------------


@dataclass
class OracleWeights:
    """fp16 weights keyed exactly like the reference's safetensors file
    (DeBERTa.swift:128-148, 199-208, 228-229; prepare_model.py:82-98)."""

    tensors: dict
    config: OracleConfig = field(default_factory=OracleConfig)

    def get(self, key: str) -> np.ndarray:
        return self.tensors[key]

    def layer(self, i: int, name: str) -> np.ndarray:
        return self.tensors[f"encoder.encoder.layer.{i}.{name}"]


# ---------------------------------------------------------------------------
# Forward
# ---------------------------------------------------------------------------


class _Rounder:
    def __init__(self, fp16: bool, compute_dtype=np.float32):
        self.fp16 = fp16
        self.dt = compute_dtype

    def __call__(self, x: np.ndarray) -> np.ndarray:
        if self.fp16:
            return x.astype(np.float16).astype(self.dt)
        return x.astype(self.dt, copy=False)


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float) -> np.ndarray:
    """``MLXFast.layerNorm`` (DeBERTa.swift:103-105): statistics over the last axis in
    at least fp32 (two-pass mean / biased variance), then affine."""
    xf = x.astype(np.float64 if x.dtype == np.float64 else np.float32)
    mean = xf.mean(axis=-1, keepdims=True)
    var = ((xf - mean) ** 2).mean(axis=-1, keepdims=True)
    return (xf - mean) / np.sqrt(var + eps) * gamma.astype(xf.dtype) + beta.astype(xf.dtype)


def gelu(x: np.ndarray) -> np.ndarray:
    """Exact erf GELU, ``MLXNN.gelu`` (DeBERTa.swift:421)."""
    from scipy.special import erf  # scipy is part of the image; oracle-only dependency

    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def relative_projections(w: OracleWeights, fp16_rounding: bool = True, dtype=np.float32):
    """Init-time ``LN(rel_embeddings)`` then per layer ``[PQ;PK] = R [Wq;Wk]^T + [bq;bk]``,
    reshaped [1,512,2,H,d] -> PQ, PK [H, 512, d] (DeBERTa.swift:204-227)."""
    cfg = w.config
    rnd = _Rounder(fp16_rounding, dtype)
    rel = w.get("encoder.encoder.rel_embeddings.weight").astype(dtype)
    R = rnd(layer_norm(rel, w.get("encoder.encoder.LayerNorm.weight"),
                       w.get("encoder.encoder.LayerNorm.bias"), cfg.layer_norm_eps))
    H, d = cfg.num_attention_heads, cfg.head_size
    out = []
    for i in range(cfg.num_hidden_layers):
        wq = w.layer(i, "attention.self.query_proj.weight").astype(dtype)
        bq = w.layer(i, "attention.self.query_proj.bias").astype(dtype)
        wk = w.layer(i, "attention.self.key_proj.weight").astype(dtype)
        bk = w.layer(i, "attention.self.key_proj.bias").astype(dtype)
        pq = rnd(R @ wq.T + bq)  # [512, H*d]
        pk = rnd(R @ wk.T + bk)
        pq = pq.reshape(-1, H, d).transpose(1, 0, 2)  # [H, 512, d]
        pk = pk.reshape(-1, H, d).transpose(1, 0, 2)
        out.append((pq, pk))
    return out


def disentangled_attention(q, k, v, pq, pk, key_valid, c2p_idx, p2c_idx,
                           fp16_rounding: bool = True, dtype=np.float32):
    """Default fast-attention path, DeBERTa.swift:322-395.

    q, k, v: [B, H, L, d]; pq, pk: [H, P, d]; key_valid: [B, L] bool;
    c2p_idx, p2c_idx: [L, L] int. Returns context [B, L, H*d].
    """
    rnd = _Rounder(fp16_rounding, dtype)
    B, H, L, d = q.shape
    scale_f = math.sqrt(3 * d)
    # fp16(sqrt(192)) as the reference builds it (DeBERTa.swift:323-326)
    scale16 = float(np.float16(np.float32(scale_f))) if fp16_rounding else scale_f
    c2p_raw = rnd(q @ pk.transpose(0, 2, 1)[None])  # [B,H,L,P]  (:374)
    c2p = np.take_along_axis(c2p_raw, np.broadcast_to(c2p_idx, (B, H, L, L)), axis=-1)  # (:375)
    p2c_raw = rnd(k @ pq.transpose(0, 2, 1)[None])  # (:376)
    p2c = np.take_along_axis(p2c_raw, np.broadcast_to(p2c_idx, (B, H, L, L)), axis=-1)
    p2c = p2c.transpose(0, 1, 3, 2)  # (:377-378)
    rel_bias = rnd(rnd(c2p + p2c) / scale16)  # (:379)
    # additive key mask (:329-335, :385): valid keys keep the fp16 relative bias; masked
    # keys get -65504. (The reference adds the two in fp16, where -65504 + bias can round
    # to -inf; both give exactly zero weight whenever a row has any valid key. Rows whose
    # keys are all masked are never produced by the reference's input builder; here they
    # keep finite scores, so the mask acts as a constant shift.)
    mask = np.where(key_valid[:, None, None, :], rel_bias, np.asarray(-65504.0, dtype))
    # SDPA (:386-393): fp32 scores, scale = 1/sqrt(192) as Float, softmax, @ v
    sc = (q.astype(np.float32) @ k.astype(np.float32).transpose(0, 1, 3, 2)) * np.float32(1.0 / scale_f)
    sc = sc.astype(dtype) + mask
    probs = softmax(sc, axis=-1)
    ctx = rnd(probs @ v)
    return ctx.transpose(0, 2, 1, 3).reshape(B, L, H * d)


def forward(w: OracleWeights, input_ids, attention_mask, marker_indices, marker_mask,
            fp16_rounding: bool = True, dtype=np.float32, p2c_convention: str = "mlx",
            projections=None, return_hidden: bool = False):
    """Full classify forward (DeBERTa.swift:274-447). Returns logits [B, Hm, O] in
    ``dtype`` (fp16-valued when ``fp16_rounding``)."""
    cfg = w.config
    rnd = _Rounder(fp16_rounding, dtype)
    ids = np.asarray(input_ids).astype(np.int64)
    B, L = ids.shape
    H, d, E = cfg.num_attention_heads, cfg.head_size, cfg.hidden_size
    mask16 = np.asarray(attention_mask).astype(np.float32)
    if fp16_rounding:
        mask16 = mask16.astype(np.float16).astype(np.float32)
    valid = mask16 > 0  # (:329)
    if projections is None:
        projections = relative_projections(w, fp16_rounding, dtype)
    c2p_idx, p2c_idx = relative_indices(L, cfg.position_buckets, cfg.max_relative_positions,
                                        p2c_convention)

    # embedding (:285-292)
    emb = w.get("encoder.embeddings.word_embeddings.weight")[ids].astype(dtype)
    x = rnd(layer_norm(emb, w.get("encoder.embeddings.LayerNorm.weight"),
                       w.get("encoder.embeddings.LayerNorm.bias"), cfg.layer_norm_eps))
    x = rnd(x * mask16.astype(dtype)[:, :, None])

    for i in range(cfg.num_hidden_layers):
        wqkv = np.concatenate([w.layer(i, f"attention.self.{n}_proj.weight") for n in ("query", "key", "value")]).astype(dtype)
        bqkv = np.concatenate([w.layer(i, f"attention.self.{n}_proj.bias") for n in ("query", "key", "value")]).astype(dtype)
        qkv = rnd(x @ wqkv.T + bqkv).reshape(B, L, 3, H, d)  # (:303-311)
        q = qkv[:, :, 0].transpose(0, 2, 1, 3)
        k = qkv[:, :, 1].transpose(0, 2, 1, 3)
        v = qkv[:, :, 2].transpose(0, 2, 1, 3)
        pq, pk = projections[i]
        ctx = disentangled_attention(q, k, v, pq, pk, valid, c2p_idx, p2c_idx, fp16_rounding, dtype)
        # attention output + residual LN (:412-418, :463)
        ao = rnd(ctx @ w.layer(i, "attention.output.dense.weight").astype(dtype).T
                 + w.layer(i, "attention.output.dense.bias").astype(dtype))
        x = rnd(layer_norm(rnd(ao + x), w.layer(i, "attention.output.LayerNorm.weight"),
                           w.layer(i, "attention.output.LayerNorm.bias"), cfg.layer_norm_eps))
        # feed-forward (:420-427)
        h = rnd(x @ w.layer(i, "intermediate.dense.weight").astype(dtype).T
                + w.layer(i, "intermediate.dense.bias").astype(dtype))
        h = rnd(gelu(h))
        y = rnd(h @ w.layer(i, "output.dense.weight").astype(dtype).T
                + w.layer(i, "output.dense.bias").astype(dtype))
        x = rnd(layer_norm(rnd(y + x), w.layer(i, "output.LayerNorm.weight"),
                           w.layer(i, "output.LayerNorm.bias"), cfg.layer_norm_eps))

    logits = classifier(w, x, marker_indices, marker_mask, fp16_rounding, dtype)
    if return_hidden:
        return logits, x
    return logits


def classifier(w: OracleWeights, hidden, marker_indices, marker_mask,
               fp16_rounding: bool = True, dtype=np.float32):
    """Classifier stage, DeBERTa.swift:430-444: ``flat = markerIdx + b*L``; gather rows;
    ``classifier.2(relu(classifier.0(x)))``; ``where(markerMask > 0, v, -10000)``."""
    rnd = _Rounder(fp16_rounding, dtype)
    B, L, E = hidden.shape
    mi = np.asarray(marker_indices).astype(np.int64)
    _, Hm, O = mi.shape
    flat = flatten_marker_indices(mi, L)
    rows = hidden.reshape(B * L, E)[flat.reshape(-1)]
    h = rnd(rows @ w.get("classifier.0.weight").astype(dtype).T + w.get("classifier.0.bias").astype(dtype))
    h = rnd(np.maximum(h, 0))
    v = rnd(h @ w.get("classifier.2.weight").astype(dtype).T + w.get("classifier.2.bias").astype(dtype))
    v = v.reshape(B, Hm, O)
    mm = np.asarray(marker_mask).astype(np.float32)
    return np.where(mm > 0, v, np.asarray(-10000.0, dtype=dtype)).astype(dtype)


def flatten_marker_indices(marker_indices, seq_len: int) -> np.ndarray:
    """``markerIdx + b * L`` (DeBERTa.swift:431-433), int64 [B, Hm, O]. Bit-exact."""
    mi = np.asarray(marker_indices).astype(np.int64)
    return mi + (np.arange(mi.shape[0], dtype=np.int64) * seq_len)[:, None, None]


# ---------------------------------------------------------------------------
# Host-side layout and decode (bit-exact / fp64)
# ---------------------------------------------------------------------------


def select_bucket(unpadded_length: int, buckets) -> int:
    """Smallest bucket >= length over the sorted unique bucket set
    (NativeTokenizer.swift:85-88, 134-137). Raises ValueError (inputDoesNotFit)."""
    ordered = sorted(set(int(b) for b in buckets))
    if not ordered:
        raise ValueError("inputDoesNotFit")
    for b in ordered:
        if b >= unpadded_length:
            return b
    raise ValueError("inputDoesNotFit")


def layout_input(token_ids, marker_positions, buckets=(32, 64, 96, 128, 256, 512), pad_id: int = 0):
    """Padded ids / mask / marker arrays from an already-tokenised row
    (NativeTokenizer.swift:134-157). ``marker_positions[t]`` lists the start index of
    each ``[L]`` token of task t. Returns (ids[1,Lb] int64, mask[1,Lb] fp16,
    marker_indices[1,Hm,O] int64, marker_mask[1,Hm,O] fp32)."""
    if len(marker_positions) == 0 or any(len(p) == 0 for p in marker_positions):
        raise ValueError("noTaskLabels")
    n = len(token_ids)
    lb = select_bucket(n, buckets)
    ids = list(token_ids) + [pad_id] * (lb - n)
    mask = [1.0 if i < n else 0.0 for i in range(lb)]
    hm = max(len(marker_positions), 1)
    o = max(max(len(p) for p in marker_positions), 1)
    flat = [0] * (hm * o)
    fmask = [0.0] * (hm * o)
    for h, positions in enumerate(marker_positions):
        for j, p in enumerate(positions):
            if j < o:
                flat[h * o + j] = p
                fmask[h * o + j] = 1.0
    return (np.asarray(ids, dtype=np.int64)[None],
            np.asarray(mask, dtype=np.float16)[None],
            np.asarray(flat, dtype=np.int64).reshape(1, hm, o),
            np.asarray(fmask, dtype=np.float32).reshape(1, hm, o))


def decode(logits_row: np.ndarray, n_labels, multi_label):
    """Per-task probabilities and selections, RawCLI.swift:182-223 (float64).

    ``logits_row`` is [Hm, O]; task t uses the first ``n_labels[t]`` options.
    Multi-label: unshifted sigmoid, select p >= 0.5, else the first argmax.
    Single-label: max-subtracted softmax, first argmax."""
    out = []
    for t, (n, ml) in enumerate(zip(n_labels, multi_label)):
        x = np.asarray(logits_row[t, :n], dtype=np.float64)
        if ml:
            with np.errstate(over="ignore"):  # exp(10000) = inf gives p = 0, as Double does
                p = 1.0 / (1.0 + np.exp(-x))
            sel = [i for i in range(n) if p[i] >= 0.5]
            if not sel:
                sel = [int(np.argmax(p))]
        else:
            e = np.exp(x - x.max())
            p = e / e.sum()
            sel = [int(np.argmax(p))]
        out.append((p, sel))
    return out
