"""ctypes binding of ``libgdc.so`` (declarations in ``include/gdc.h``).

The library is built in-tree by ``gliner_decide_metal_b200.build``. There is no
fallback: if the shared library is missing or fails to load, the first call through
``lib`` raises ImportError. The library is mapped on that first call, not at import, so
that host-only users of the package (the synthetic-data generators, the safetensors
reader) do not load it.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("GDC_LIBRARY", Path(__file__).resolve().parent / "libgdc.so"))

GDC_OK = 0
STATUS_NAMES = {
    0: "GDC_OK", 1: "GDC_ERR_MISSING_WEIGHT", 2: "GDC_ERR_INVALID_SHAPE", 3: "GDC_ERR_INVALID_INPUT",
    4: "GDC_ERR_INPUT_DOES_NOT_FIT", 5: "GDC_ERR_NO_TASK_LABELS", 6: "GDC_ERR_IO", 7: "GDC_ERR_CUDA",
    8: "GDC_ERR_OUT_OF_MEMORY", 9: "GDC_ERR_TIMEOUT", 10: "GDC_ERR_UNSUPPORTED", 11: "GDC_ERR_NULL_POINTER",
    12: "GDC_ERR_PARTIAL",
}
GDC_INT32, GDC_INT64, GDC_FLOAT16, GDC_FLOAT32, GDC_UINT8 = range(5)


class GdcConfig(C.Structure):
    _fields_ = [("hidden_size", C.c_int32), ("intermediate_size", C.c_int32), ("num_hidden_layers", C.c_int32),
                ("num_attention_heads", C.c_int32), ("layer_norm_eps", C.c_float), ("position_buckets", C.c_int32),
                ("max_relative_positions", C.c_int32), ("pad_token_id", C.c_int32), ("vocab_size", C.c_int32),
                ("use_fused_kernels", C.c_int32), ("use_compiled_graph", C.c_int32),
                ("use_fast_attention", C.c_int32), ("use_custom_relative_kernel", C.c_int32),
                ("use_fused_attention_kernel", C.c_int32)]


class GdcInput(C.Structure):
    _fields_ = [("batch", C.c_int32), ("seq_len", C.c_int32), ("max_heads", C.c_int32), ("max_options", C.c_int32),
                ("input_ids", C.c_void_p), ("ids_dtype", C.c_int), ("attention_mask", C.c_void_p),
                ("mask_dtype", C.c_int), ("marker_indices", C.c_void_p), ("marker_dtype", C.c_int),
                ("marker_mask", C.c_void_p), ("marker_mask_dtype", C.c_int)]


class GdcProfileEvent(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("nanoseconds", C.c_uint64)]


class GdcOutput(C.Structure):
    _fields_ = [("logits", C.c_void_p), ("logits_f16", C.c_void_p), ("wall_ns", C.c_uint64),
                ("events", C.POINTER(GdcProfileEvent)), ("events_capacity", C.c_int32),
                ("events_count", C.c_int32)]


# (name, restype, argtypes) for every function declared in include/gdc.h
_vp, _i32, _i64, _f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float
_pi32 = C.POINTER(C.c_int32)
SIGNATURES = [
    ("gdc_config_default", None, [C.POINTER(GdcConfig)]),
    ("gdc_model_load", C.c_int, [C.c_char_p, C.POINTER(GdcConfig), C.c_int, C.POINTER(_vp)]),
    ("gdc_model_free", None, [_vp]),
    ("gdc_model_device", C.c_int, [_vp]),
    ("gdc_model_classifier_hidden", C.c_int, [_vp]),
    ("gdc_classify", C.c_int, [_vp, C.POINTER(GdcInput), C.c_int, C.POINTER(GdcOutput)]),
    ("gdc_classify_device", C.c_int, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gdc_check_errors", C.c_int, [_vp]),
    ("gdc_model_stream", _vp, [_vp]),
    ("gdc_model_set_row_packing", C.c_int, [_vp, C.c_int]),
    ("gdc_model_row_packing", C.c_int, [_vp]),
    ("gdc_profile_enable", C.c_int, [_vp, C.c_int]),
    ("gdc_profile_reset", C.c_int, [_vp]),
    ("gdc_profile_read", C.c_int, [_vp, C.POINTER(GdcProfileEvent), C.c_int, _pi32]),
    ("gdc_classify_sharded", C.c_int, [C.POINTER(_vp), C.c_int, C.POINTER(GdcInput), C.POINTER(GdcOutput),
                                       C.POINTER(C.c_int)]),
    ("gdc_decode", C.c_int, [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    ("gdc_decode_device", C.c_int, [_vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    ("gdc_select_bucket", C.c_int, [_i32, _pi32, _i32, _pi32]),
    ("gdc_layout_row", C.c_int, [_pi32, _i32, _pi32, _pi32, _i32, _pi32, _i32, _i32, _pi32, _pi32, _pi32, _pi32,
                                 _i32, C.POINTER(C.c_float), _pi32, C.POINTER(C.c_float), _i32]),
    ("gdc_relative_index_table", C.c_int, [_i32, _i32, _pi32]),
    ("gdc_residual_layer_norm", C.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    ("gdc_disentangled_attention", C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    ("gdc_disentangled_attention_scalar", C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    ("gdc_disentangled_attention_noalloc", C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    ("gdc_linear", C.c_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i64, _i32, _vp]),
    ("gdc_kernels_check_errors", C.c_int, []),
    ("gdc_selftest_wait_timeout", C.c_int, [_i32, _vp]),
    ("gdc_last_error", C.c_char_p, []),
    ("gdc_abi_version", C.c_int, []),
    ("gdc_build_info", C.c_char_p, []),
]


def load():
    """Maps libgdc.so and sets the ctypes signature of every function in include/gdc.h."""
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python gliner_decide_metal_b200/build.py` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class _LazyLibrary:
    """Attribute access loads libgdc.so once (thread-safe) and forwards to it."""

    def __init__(self):
        import threading
        self._lock = threading.Lock()
        self._cdll = None

    def _get(self):
        if self._cdll is None:
            with self._lock:
                if self._cdll is None:
                    self._cdll = load()
        return self._cdll

    @property
    def loaded(self) -> bool:
        return self._cdll is not None

    def __getattr__(self, name):
        return getattr(self._get(), name)


lib = _LazyLibrary()
