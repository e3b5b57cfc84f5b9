"""ctypes binding of libbasalt_cuda.so (include/basalt_cuda.h).

There is no CPU fallback: if the library is missing, loading raises. A missing GPU surfaces as a
``BasaltUnsupportedOperationException`` from the first engine call, never as a silent switch to
another implementation.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "libbasalt_cuda.so"
HEADER = PACKAGE.parent / "include" / "basalt_cuda.h"

BST_OK = 0
BST_INVALID = -1
BST_SHAPE = -2
BST_UNKNOWN_HANDLE = -3
BST_CONTEXT = -4
BST_GRAPH = -5
BST_PANIC = -6
BST_OOM = -7
BST_UNSUPPORTED = -8

FAMILY_PADDED_DECODER = 1
FAMILY_DECODER = 2
FAMILY_CHAR_LM = 3
FAMILY_LAST_TOKEN = 4

DTYPE_F32 = 0
DTYPE_BF16 = 1

KERNEL_CLASSES = 15


class ModelSpecStruct(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int32), ("vocabulary", ctypes.c_int32),
                ("window", ctypes.c_int32), ("dimension", ctypes.c_int32),
                ("layers", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("weight_dtype", ctypes.c_int32),
                ("kv_dtype", ctypes.c_int32), ("max_rows", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 6)]


TOKEN_SINK = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                              ctypes.c_int32)

_P = ctypes.POINTER
_i32p = _P(ctypes.c_int32)
_i64p = _P(ctypes.c_int64)
_f32p = _P(ctypes.c_float)
_f64p = _P(ctypes.c_double)
_u64 = ctypes.c_uint64

SIGNATURES = {
    "bst_abi_version": (ctypes.c_int32, []),
    "bst_device_count": (ctypes.c_int32, [_i32p]),
    "bst_engine_create": (ctypes.c_int32, [_P(ModelSpecStruct), ctypes.c_int32, _P(_u64)]),
    "bst_engine_destroy": (ctypes.c_int32, [_u64]),
    "bst_parameter_count": (ctypes.c_int32, [_u64, _i32p]),
    "bst_parameter_info": (ctypes.c_int32, [_u64, ctypes.c_int32, ctypes.c_char_p,
                                            ctypes.c_int32, _i64p]),
    "bst_set_parameter": (ctypes.c_int32, [_u64, ctypes.c_char_p, _f32p, ctypes.c_int64]),
    "bst_get_parameter": (ctypes.c_int32, [_u64, ctypes.c_char_p, _f32p, ctypes.c_int64]),
    "bst_save": (ctypes.c_int32, [_u64, ctypes.c_char_p]),
    "bst_load": (ctypes.c_int32, [_u64, ctypes.c_char_p]),
    "bst_scores": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32, _f64p]),
    "bst_generate": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_int32, _i32p, TOKEN_SINK, ctypes.c_void_p]),
    "bst_sample": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                    ctypes.c_int32, ctypes.c_float, ctypes.c_int32, _i32p,
                                    TOKEN_SINK, ctypes.c_void_p]),
    "bst_generate_logits": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32, _i32p, _f32p]),
    "bst_sample_logits": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_float, ctypes.c_int32, _i32p,
                                           _f32p]),
    "bst_generate_logits_rows": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int32, _i32p, ctypes.c_int32, _i32p,
                                                  _f32p]),
    "bst_sample_logits_rows": (ctypes.c_int32, [_u64, _i32p, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_float, ctypes.c_int32,
                                                _i32p, ctypes.c_int32, _i32p, _f32p]),
    "bst_generate_device": (ctypes.c_int32, [_u64, ctypes.c_void_p, ctypes.c_int32,
                                             ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    "bst_sample_device": (ctypes.c_int32, [_u64, ctypes.c_void_p, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                           ctypes.c_int32, ctypes.c_void_p]),
    "bst_seed": (ctypes.c_int32, [_u64, ctypes.c_int64]),
    "bst_get_rng_state": (ctypes.c_int32, [_u64, _i64p]),
    "bst_set_rng_state": (ctypes.c_int32, [_u64, ctypes.c_int64]),
    "bst_begin_scope": (ctypes.c_int32, [_u64]),
    "bst_end_scope": (ctypes.c_int32, [_u64, _i32p]),
    "bst_scope_depth": (ctypes.c_int32, [_u64, _i32p]),
    "bst_engine_stats": (ctypes.c_int32, [_u64, _i64p]),
    "bst_engine_stream": (ctypes.c_int32, [_u64, _P(ctypes.c_void_p)]),
    "bst_profile_enable": (ctypes.c_int32, [_u64, ctypes.c_int32]),
    "bst_profile_reset": (ctypes.c_int32, [_u64]),
    "bst_profile_read": (ctypes.c_int32, [_u64, ctypes.c_int32, ctypes.c_char_p, ctypes.c_int32,
                                          _i64p, _f64p, _f64p, _f64p]),
    "bst_matmul": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_int64]),
    "bst_matmul_static": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int64]),
    "bst_recognize_model": (ctypes.c_int32, [_P(ctypes.c_char_p), _i32p, _i64p, ctypes.c_int32,
                                             ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                             _P(ModelSpecStruct)]),
    "bst_engine_create_from_parameters": (ctypes.c_int32, [
        _P(ctypes.c_char_p), _i32p, _i64p, _P(_f32p), ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        _P(_u64)]),
    "bst_context_create": (ctypes.c_int32, [ctypes.c_int32, _P(_u64)]),
    "bst_context_destroy": (ctypes.c_int32, [_u64]),
    "bst_tensor_create": (ctypes.c_int32, [_u64, ctypes.c_int32, _i64p, ctypes.c_int32, _f32p,
                                           _P(_u64)]),
    "bst_tensor_transfer": (ctypes.c_int32, [_u64, _u64, ctypes.c_int32, _P(_u64)]),
    "bst_tensor_read": (ctypes.c_int32, [_u64, _u64, _f32p, ctypes.c_int64]),
    "bst_tensor_write": (ctypes.c_int32, [_u64, _u64, _f32p, ctypes.c_int64]),
    "bst_tensor_info": (ctypes.c_int32, [_u64, _u64, _i32p, _i32p, _i64p, ctypes.c_int32]),
    "bst_tensor_release": (ctypes.c_int32, [_u64, _u64, _i32p]),
    "bst_execute_queue": (ctypes.c_int32, [_u64, ctypes.c_void_p, ctypes.c_int32]),
    "bst_context_stats": (ctypes.c_int32, [_u64, _i64p]),
    "bst_context_clear_graph": (ctypes.c_int32, [_u64]),
    "bst_last_error": (ctypes.c_int32, [_u64, ctypes.c_char_p, ctypes.c_int32]),
    "bst_write_synthetic_weights": (ctypes.c_int32, [_P(ModelSpecStruct), ctypes.c_char_p,
                                                     ctypes.c_int64, ctypes.c_double]),
    "bst_synthetic_prompts": (ctypes.c_int32, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.c_int32, _i32p]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads libbasalt_cuda.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise ImportError(
                f"{LIBRARY} is missing: build it with `python -m basalt_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error(handle: int = 0) -> str:
    buf = ctypes.create_string_buffer(1024)
    load().bst_last_error(handle, buf, len(buf))
    return buf.value.decode(errors="replace")
