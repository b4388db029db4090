"""ctypes bindings of librokoko_b200.so (the C ABI declared in include/rk_b200.h).

The library is built in-tree by `python -m rokoko_b200.build`; importing this
module never falls back to anything else: if the shared library is missing or
does not load, `load()` raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librokoko_b200.so")

RK_OK = 0
RK_PRECISION_FP32 = 0
RK_PRECISION_FP16 = 1
RK_ERR_WORKSPACE = -2
RK_ERR_DEVICE_TIMEOUT = -7
RK_CONV_STATIC_SCRATCH_BYTES = 32 * 1024 * 1024

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_lib = None


class RkError(RuntimeError):
    def __init__(self, status: int, what: str):
        L = load()
        super().__init__(f"{what}: {L.rk_status_string(status).decode()} ({status}): {L.rk_last_error().decode()}")
        self.status = status


class rk_options(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_int), ("max_tokens", ctypes.c_int), ("l_bucket", ctypes.c_int)]


# rk_pcm_fn: int (*)(void* user, int index, const float* pcm, size_t n_samples)
PCM_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t)

# (name, restype, argtypes) for every entry point of include/rk_b200.h
SIGNATURES = [
    ("rk_status_string", ctypes.c_char_p, [ctypes.c_int]),
    ("rk_last_error", ctypes.c_char_p, []),
    ("rk_conv1d_workspace_size", ctypes.c_size_t, [ctypes.c_int] * 8),
    ("rk_conv1d_fprop", ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 8 + [ctypes.c_void_p]),
    ("rk_conv1d_check", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ("rk_conv1d_fprop_static", ctypes.c_int, [ctypes.c_void_p] * 5 + [ctypes.c_int] * 8 + [ctypes.c_void_p]),
    ("rk_conv1d_static_check", ctypes.c_int, [ctypes.c_void_p]),
    ("rk_conv1d_fprop_f32", ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 7 + [ctypes.c_void_p]),
    ("rk_conv1d_fprop_f16", ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 7 + [ctypes.c_void_p]),
    ("rk_conv1d_workspace_bytes", ctypes.c_size_t, [ctypes.c_int] * 7),
    ("rk_create", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(rk_options), ctypes.POINTER(ctypes.c_void_p)]),
    ("rk_destroy", None, [ctypes.c_void_p]),
    ("rk_load_weights_koko", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]),
    ("rk_convert_koko_b200", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
      ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_decode_features", ctypes.c_int, [ctypes.c_void_p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int, _f32p]),
    ("rk_decode_features_device", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
      ctypes.c_void_p]),
    ("rk_infer", ctypes.c_int,
     [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p, _i32p, _i32p, ctypes.POINTER(ctypes.c_int), _f32p,
      ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_encode", ctypes.c_int,
     [ctypes.c_void_p, _i32p, _i32p, ctypes.c_int, _f32p, _i32p, _i32p, _i32p]),
    ("rk_synthesize_stream", ctypes.c_int,
     [ctypes.c_void_p, _i32p, _i32p, ctypes.c_int, _f32p, _i32p, ctypes.c_int, PCM_FN, ctypes.c_void_p]),
    ("rk_decode", ctypes.c_int,
     [ctypes.c_void_p, _f32p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int)]),
    ("rk_get_stage", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_char_p, _f32p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_record_stages", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    ("rk_kernel_count", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_longlong), ctypes.c_int]),
    ("rk_stream", ctypes.c_void_p, [ctypes.c_void_p]),
    ("rk_compute_decode_bytes", ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ("rk_g2p_load", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]),
    ("rk_g2p_infer", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int,
      ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_g2p_frames", ctypes.c_int,
     [ctypes.c_void_p, _i32p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_g2p_param_bytes", ctypes.c_size_t, [ctypes.c_void_p]),
    ("rk_g2p_free", None, [ctypes.c_void_p]),
    ("rk_ipa_to_tokens", ctypes.c_int,
     [ctypes.c_char_p, ctypes.c_size_t, _i32p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_ipa_chunks", ctypes.c_int,
     [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.c_size_t,
      ctypes.POINTER(ctypes.c_size_t)]),
    ("rk_profile", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    ("rk_profile_read", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
      ctypes.POINTER(ctypes.c_longlong)]),
    ("rk_profile_timeline", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
]


def load():
    """Load the in-tree shared library (raises if it is missing).  The
    environment variable RK_B200_LIBRARY may name another build of it."""
    global _lib
    if _lib is None:
        path = os.environ.get("RK_B200_LIBRARY") or LIB_PATH
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `python -m rokoko_b200.build` (no fallback path exists)")
        L = ctypes.CDLL(path)
        for name, res, args in SIGNATURES:
            try:
                fn = getattr(L, name)
            except AttributeError:
                continue  # reported by exported_symbols() / the export test
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    """Names from SIGNATURES that the loaded library exports."""
    L = load()
    out = []
    for name, _, _ in SIGNATURES:
        try:
            getattr(L, name)
            out.append(name)
        except AttributeError:
            pass
    return out


def check(status: int, what: str) -> None:
    if status != RK_OK:
        raise RkError(status, what)
