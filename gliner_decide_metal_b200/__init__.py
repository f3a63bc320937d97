"""B200 backend for the GLiNER2.5-Decide classification forward.

Python mirror of the reference's ``GLiNERDecideCore`` library API (Swift,
shantanugoel/gliner-decide-metal) over the C ABI in ``include/gdc.h``:

* ``DeBERTaV2Configuration``            Configuration.swift:3-49
* ``DecisionInput``                     DeBERTa.swift:22-58 (incl. ``init(url:)``)
* ``ProfileEvent`` / ``InferenceResult`` DeBERTa.swift:7-20
* ``GLiNERDecideClassifier``            DeBERTa.swift:156-272 (``init(weightsURL:...)``, ``classify``)
* ``DecisionTask``                      NativeTokenizer.swift:25-45
* ``make_input_from_tokens``            the bucket / marker layout of
                                        ``NativeDecisionTokenizer.makeInput`` (NativeTokenizer.swift:76-158)
                                        for already-tokenised rows
* ``decode``                            RawCLI.swift:182-223
* errors                                WeightStoreError (Weights.swift:4-19), NativeTokenizerError
                                        (NativeTokenizer.swift:5-23)

All compute runs in ``libgdc.so`` on the GPU. The library is mapped by the first call
that needs it (model load, classify, layout, decode); that call raises ImportError if
the library is missing. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

from ._lib import (GDC_FLOAT16, GDC_FLOAT32, GDC_INT32, GDC_INT64, GDC_UINT8, STATUS_NAMES, GdcConfig, GdcInput,
                   GdcOutput, GdcProfileEvent, lib)

__all__ = [
    "DeBERTaV2Configuration", "DecisionInput", "DecisionTask", "ProfileEvent", "InferenceResult", "Prediction",
    "GLiNERDecideClassifier", "make_input_from_tokens", "select_bucket", "decode", "decode_batch",
    "classify_sharded", "relative_index_table", "packed_row_layout", "GDCError", "MissingWeightError", "InvalidShapeError",
    "InvalidInputError", "InputDoesNotFitError", "NoTaskLabelsError", "DEFAULT_BUCKETS",
]

DEFAULT_BUCKETS = (32, 64, 96, 128, 256, 512)


# --------------------------------------------------------------------------- errors

class GDCError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


class MissingWeightError(GDCError):
    """WeightStoreError.missingWeight"""


class InvalidShapeError(GDCError):
    """WeightStoreError.invalidShape"""


class InvalidInputError(GDCError):
    """WeightStoreError.invalidInput (also the reference's precondition failures)"""


class InputDoesNotFitError(GDCError):
    """NativeTokenizerError.inputDoesNotFit"""


class NoTaskLabelsError(GDCError):
    """NativeTokenizerError.noTaskLabels"""


_ERRORS = {1: MissingWeightError, 2: InvalidShapeError, 3: InvalidInputError, 4: InputDoesNotFitError,
           5: NoTaskLabelsError}


def _check(status: int):
    if status != 0:
        msg = (lib.gdc_last_error() or b"").decode(errors="replace")
        raise _ERRORS.get(status, GDCError)(status, msg)


# --------------------------------------------------------------------------- types

@dataclass(frozen=True)
class DeBERTaV2Configuration:
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    layer_norm_eps: float = 1e-7
    position_buckets: int = 256
    max_relative_positions: int = -1
    hidden_act: str = "gelu"
    pad_token_id: int = 0
    # Word-embedding rows the loader requires (the reference hard-checks 128011).
    vocab_size: int = 128011

    @property
    def head_size(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @staticmethod
    def default() -> "DeBERTaV2Configuration":
        return DeBERTaV2Configuration()


@dataclass
class DecisionInput:
    """input_ids [B, L] int; attention_mask [B, L] (fp16 in the reference);
    marker_indices [B, Hm, O] int; marker_mask [B, Hm, O] fp32."""
    input_ids: np.ndarray
    attention_mask: np.ndarray
    marker_indices: np.ndarray
    marker_mask: np.ndarray

    @staticmethod
    def from_url(path) -> "DecisionInput":
        """``DecisionInput(url:)`` (DeBERTa.swift:40-57)."""
        from .safetensors_io import load_file
        arrays = load_file(path)
        missing = [k for k in ("input_ids", "attention_mask", "marker_indices", "marker_mask") if k not in arrays]
        if missing:
            raise InvalidInputError(3, "Input safetensors must contain input_ids, attention_mask, marker_indices, "
                                       "and marker_mask")
        return DecisionInput(arrays["input_ids"], arrays["attention_mask"], arrays["marker_indices"],
                             arrays["marker_mask"])

    def save(self, path) -> None:
        from .safetensors_io import save_file
        save_file({"input_ids": self.input_ids, "attention_mask": self.attention_mask,
                   "marker_indices": self.marker_indices, "marker_mask": self.marker_mask}, path)

    @property
    def shape(self):
        b, l = self.input_ids.shape
        _, hm, o = self.marker_indices.shape
        return b, l, hm, o

    @staticmethod
    def concatenated(items: Sequence["DecisionInput"]) -> "DecisionInput":
        """Row concatenation (RawCLI.swift:145-150)."""
        return DecisionInput(*(np.concatenate([getattr(x, k) for x in items], axis=0) for k in
                               ("input_ids", "attention_mask", "marker_indices", "marker_mask")))


@dataclass(frozen=True)
class DecisionTask:
    name: str
    labels: tuple
    multi_label: bool = False
    prompt: Optional[str] = None
    label_descriptions: Optional[dict] = None


@dataclass
class ProfileEvent:
    name: str
    nanoseconds: int

    @property
    def milliseconds(self) -> float:
        return self.nanoseconds / 1e6


@dataclass
class InferenceResult:
    """``logits`` are the reference's fp16 values [B, Hm, O]; ``logits_f32`` the same
    values as float32."""
    logits: np.ndarray
    logits_f32: np.ndarray
    wall_nanoseconds: int
    events: list = field(default_factory=list)

    @property
    def wall_milliseconds(self) -> float:
        return self.wall_nanoseconds / 1e6


@dataclass
class Prediction:
    task: str
    labels: list
    probabilities: list


# --------------------------------------------------------------------------- helpers

_DT = {np.dtype(np.int32): GDC_INT32, np.dtype(np.int64): GDC_INT64, np.dtype(np.float16): GDC_FLOAT16,
       np.dtype(np.float32): GDC_FLOAT32, np.dtype(np.uint8): GDC_UINT8}


def _as_supported(a: np.ndarray, allowed) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype not in allowed:
        a = a.astype(allowed[0])
    return a


def _addr(a: np.ndarray) -> int:
    """Address of a C-contiguous array's first element. A writable array goes through the
    ctypes buffer route, about half the per-call cost of ``ndarray.ctypes.data``."""
    if a.flags.writeable and a.size:
        return C.addressof(C.c_char.from_buffer(a))
    return a.ctypes.data


def _make_input(inp: DecisionInput, keep: list) -> GdcInput:
    ids = _as_supported(inp.input_ids, [np.dtype(np.int64), np.dtype(np.int32)])
    mask = _as_supported(inp.attention_mask, [np.dtype(np.float16), np.dtype(np.float32), np.dtype(np.uint8),
                                              np.dtype(np.int32), np.dtype(np.int64)])
    mi = _as_supported(inp.marker_indices, [np.dtype(np.int64), np.dtype(np.int32)])
    mm = _as_supported(inp.marker_mask, [np.dtype(np.float32), np.dtype(np.float16), np.dtype(np.uint8)])
    if ids.ndim != 2 or mask.shape != ids.shape or mi.ndim != 3 or mm.shape != mi.shape or mi.shape[0] != ids.shape[0]:
        raise InvalidInputError(3, f"inconsistent DecisionInput shapes {ids.shape} {mask.shape} {mi.shape} {mm.shape}")
    keep += [ids, mask, mi, mm]
    return GdcInput(ids.shape[0], ids.shape[1], mi.shape[1], mi.shape[2], _addr(ids), _DT[ids.dtype],
                    _addr(mask), _DT[mask.dtype], _addr(mi), _DT[mi.dtype], _addr(mm), _DT[mm.dtype])


def _config(cfg: DeBERTaV2Configuration, flags) -> GdcConfig:
    c = GdcConfig()
    lib.gdc_config_default(C.byref(c))
    c.hidden_size = cfg.hidden_size
    c.intermediate_size = cfg.intermediate_size
    c.num_hidden_layers = cfg.num_hidden_layers
    c.num_attention_heads = cfg.num_attention_heads
    c.layer_norm_eps = cfg.layer_norm_eps
    c.position_buckets = cfg.position_buckets
    c.max_relative_positions = cfg.max_relative_positions
    c.pad_token_id = cfg.pad_token_id
    c.vocab_size = cfg.vocab_size
    (c.use_fused_kernels, c.use_compiled_graph, c.use_fast_attention, c.use_custom_relative_kernel,
     c.use_fused_attention_kernel) = [int(bool(f)) for f in flags]
    return c


# --------------------------------------------------------------------------- model

class GLiNERDecideClassifier:
    """``GLiNERDecideClassifier`` (DeBERTa.swift:156-272) on one CUDA device."""

    def __init__(self, weights_url, configuration: DeBERTaV2Configuration = DeBERTaV2Configuration(),
                 use_fused_kernels: bool = False, use_compiled_graph: bool = False, use_fast_attention: bool = True,
                 use_custom_relative_kernel: bool = False, use_fused_attention_kernel: bool = False,
                 device: int = 0):
        self.configuration = configuration
        cfg = _config(configuration, (use_fused_kernels, use_compiled_graph, use_fast_attention,
                                      use_custom_relative_kernel, use_fused_attention_kernel))
        h = C.c_void_p()
        _check(lib.gdc_model_load(str(Path(weights_url)).encode(), C.byref(cfg), int(device), C.byref(h)))
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    @property
    def classifier_hidden(self) -> int:
        return lib.gdc_model_classifier_hidden(self._h)

    @property
    def stream(self) -> int:
        return lib.gdc_model_stream(self._h) or 0

    @property
    def row_packing(self) -> bool:
        """Packed encoder rows (only each batch row's positions up to its last valid token or
        active marker run through the encoder) or the reference's dense [B, L] grid; the
        logits are bit-identical. On by default."""
        return bool(lib.gdc_model_row_packing(self._h))

    @row_packing.setter
    def row_packing(self, on: bool):
        _check(lib.gdc_model_set_row_packing(self._h, int(bool(on))))

    def close(self):
        if getattr(self, "_h", None):
            lib.gdc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def classify(self, input: DecisionInput, collect_profile: bool = False) -> InferenceResult:
        keep: list = []
        gin = _make_input(input, keep)
        b, hm, o = gin.batch, gin.max_heads, gin.max_options
        logits = np.empty((b, hm, o), np.float32)
        l16 = np.empty((b, hm, o), np.uint16)
        cap = 8 * self.configuration.num_hidden_layers + 8
        events = (GdcProfileEvent * cap)()
        out = GdcOutput(_addr(logits), _addr(l16), 0, events, cap, 0)
        _check(lib.gdc_classify(self._h, C.byref(gin), int(bool(collect_profile)), C.byref(out)))
        evs = [ProfileEvent(events[i].name.decode(), int(events[i].nanoseconds)) for i in range(out.events_count)]
        return InferenceResult(l16.view(np.float16), logits, int(out.wall_ns), evs)

    # -- device-resident path (used by benchmarks) --------------------------
    def classify_device(self, batch, seq_len, max_heads, max_options, ids_ptr, mask_ptr, markers_ptr,
                        marker_mask_ptr, logits_ptr, logits16_ptr=0, stream=0):
        _check(lib.gdc_classify_device(self._h, batch, seq_len, max_heads, max_options, ids_ptr, mask_ptr,
                                       markers_ptr, marker_mask_ptr, logits_ptr, logits16_ptr or None,
                                       stream or None))

    def check_errors(self):
        _check(lib.gdc_check_errors(self._h))

    def profile_enable(self, on: bool = True):
        _check(lib.gdc_profile_enable(self._h, int(on)))

    def profile_reset(self):
        _check(lib.gdc_profile_reset(self._h))

    def profile_read(self) -> dict:
        ev = (GdcProfileEvent * 32)()
        launches = (C.c_int32 * 32)()
        n = lib.gdc_profile_read(self._h, ev, 32, launches)
        return {ev[i].name.decode(): (int(ev[i].nanoseconds), int(launches[i])) for i in range(n)}


def classify_sharded(models: Sequence[GLiNERDecideClassifier], input: DecisionInput):
    """Row-sharded classify over one model per device (host threads, host gather).
    Returns (logits fp16, logits fp32, per-device status list)."""
    keep: list = []
    gin = _make_input(input, keep)
    b, hm, o = gin.batch, gin.max_heads, gin.max_options
    logits = np.empty((b, hm, o), np.float32)
    l16 = np.empty((b, hm, o), np.uint16)
    out = GdcOutput(_addr(logits), _addr(l16), 0, None, 0, 0)
    arr = (C.c_void_p * len(models))(*[m.handle for m in models])
    per = (C.c_int * len(models))()
    st = lib.gdc_classify_sharded(arr, len(models), C.byref(gin), C.byref(out), per)
    statuses = [int(x) for x in per]
    _check(st)
    return l16.view(np.float16), logits, statuses


# --------------------------------------------------------------------------- host logic

def select_bucket(unpadded_length: int, buckets=DEFAULT_BUCKETS) -> int:
    """Smallest bucket >= length (NativeTokenizer.swift:85-88,134-137)."""
    arr = (C.c_int32 * len(buckets))(*[int(b) for b in buckets])
    out = C.c_int32()
    _check(lib.gdc_select_bucket(int(unpadded_length), arr, len(buckets), C.byref(out)))
    return int(out.value)


def make_input_from_tokens(token_ids: Sequence[int], marker_positions: Sequence[Sequence[int]],
                           buckets=DEFAULT_BUCKETS, pad_id: int = 0) -> DecisionInput:
    """Row layout of ``NativeDecisionTokenizer.makeInput`` after tokenisation
    (NativeTokenizer.swift:81-82,134-157): smallest bucket, [PAD]-padded ids, fp16 mask,
    marker indices / mask [1, Hm, O]. Raises NoTaskLabelsError / InputDoesNotFitError."""
    toks = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32))
    flat = np.ascontiguousarray(np.asarray([p for task in marker_positions for p in task], dtype=np.int32))
    offs = np.zeros(len(marker_positions) + 1, np.int32)
    offs[1:] = np.cumsum([len(t) for t in marker_positions]) if len(marker_positions) else []
    bk = np.ascontiguousarray(np.asarray(buckets, dtype=np.int32))
    L, hm, o = C.c_int32(), C.c_int32(), C.c_int32()
    P = lambda a: a.ctypes.data_as(C.POINTER(C.c_int32))  # noqa: E731
    st = lib.gdc_layout_row(P(toks), len(toks), P(flat) if len(flat) else None, P(offs), len(marker_positions),
                            P(bk), len(bk), int(pad_id), C.byref(L), C.byref(hm), C.byref(o), None, 0, None, None,
                            None, 0)
    if st != 3:  # sizes are reported before the buffer check
        _check(st)
    ids = np.empty(L.value, np.int32)
    mask = np.empty(L.value, np.float32)
    mk = np.empty(hm.value * o.value, np.int32)
    mm = np.empty(hm.value * o.value, np.float32)
    _check(lib.gdc_layout_row(P(toks), len(toks), P(flat) if len(flat) else None, P(offs), len(marker_positions),
                              P(bk), len(bk), int(pad_id), C.byref(L), C.byref(hm), C.byref(o), P(ids), len(ids),
                              mask.ctypes.data_as(C.POINTER(C.c_float)), P(mk),
                              mm.ctypes.data_as(C.POINTER(C.c_float)), len(mk)))
    return DecisionInput(ids.astype(np.int64)[None], mask.astype(np.float16)[None],
                         mk.astype(np.int64).reshape(1, hm.value, o.value), mm.reshape(1, hm.value, o.value))


def decode_batch(logits: np.ndarray, n_labels: np.ndarray, multi_label: np.ndarray):
    """Vectorised ``decode`` over [B, Hm, O] logits via the C ABI (float64).
    Returns (probabilities [B,Hm,O] f64, selected [B,Hm,O] u8)."""
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
    b, hm, o = lg.shape
    nl = np.ascontiguousarray(np.asarray(n_labels, dtype=np.int32).reshape(b, hm))
    ml = np.ascontiguousarray(np.asarray(multi_label, dtype=np.uint8).reshape(b, hm))
    probs = np.empty((b, hm, o), np.float64)
    sel = np.empty((b, hm, o), np.uint8)
    _check(lib.gdc_decode(lg.ctypes.data, b, hm, o, nl.ctypes.data, ml.ctypes.data, probs.ctypes.data,
                          sel.ctypes.data))
    return probs, sel


def decode(logits: np.ndarray, tasks: Sequence[DecisionTask], row: int = 0):
    """``RawCLI.decode`` (RawCLI.swift:182-223): per task, sigmoid + threshold 0.5 with
    argmax fallback (multi-label) or softmax + argmax over the task's labels."""
    lg = np.asarray(logits, dtype=np.float32)
    if lg.ndim == 3:
        lg = lg[row]
    hm, o = lg.shape
    nl = np.zeros((1, hm), np.int32)
    ml = np.zeros((1, hm), np.uint8)
    for h, t in enumerate(tasks):
        nl[0, h] = len(t.labels)
        ml[0, h] = int(t.multi_label)
    probs, sel = decode_batch(lg[None], nl, ml)
    out = []
    for h, t in enumerate(tasks):
        n = len(t.labels)
        out.append(Prediction(t.name, [t.labels[i] for i in range(n) if sel[0, h, i]], probs[0, h, :n].tolist()))
    return out


def packed_row_layout(attention_mask: np.ndarray, marker_indices: np.ndarray, marker_mask: np.ndarray):
    """Host statement of the packed-row layout the device computes (``csrc/kernels/pack.cu``):
    per batch row the extent ``ext`` = 1 + max(last position with mask > 0, last marker index
    with marker_mask > 0 inside [0, L)), or L for a row with no position of mask > 0, and the
    offsets ``seq_off`` = [0, cumsum(ext)]; ``seq_off[-1]`` is the encoder's packed row count.
    Returns (ext int32 [B], seq_off int64 [B + 1])."""
    mask = np.asarray(attention_mask)
    B, L = mask.shape
    idx = np.asarray(marker_indices).reshape(B, -1)
    act = np.asarray(marker_mask).reshape(B, -1) > 0
    ext = np.empty(B, np.int32)
    for b in range(B):
        valid = np.nonzero(mask[b].astype(np.float32) > 0)[0]
        if valid.size == 0:
            ext[b] = L
            continue
        e = int(valid[-1]) + 1
        mk = idx[b][act[b] & (idx[b] >= 0) & (idx[b] < L)]
        if mk.size:
            e = max(e, int(mk.max()) + 1)
        ext[b] = e
    return ext, np.concatenate([[0], np.cumsum(ext, dtype=np.int64)])


def relative_index_table() -> np.ndarray:
    """The 1023-entry c2p/p2c gather index table used by the attention kernels."""
    t = np.empty(1023, np.int32)
    _check(lib.gdc_relative_index_table(256, 512, t.ctypes.data_as(C.POINTER(C.c_int32))))
    return t
