"""Python host front-end over the C ABI (include/rk_b200.h).

`Context` owns one rk_ctx (one CUDA device).  It mirrors the reference's
model-level entry points: `load_weights` (Weights::load +
precompute_weight_norms, src/weights.cpp:500-601, src/rokoko.cpp:1305),
`decode_features` (the decode phase of rokoko_infer, src/rokoko.cpp:915-1290)
and `infer` (rokoko_infer, src/rokoko.cpp:829-1297).  Every call goes through
librokoko_b200.so; there is no other implementation behind it.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib

FP32 = lib.RK_PRECISION_FP32
FP16 = lib.RK_PRECISION_FP16
# rk_profile mode bits (include/rk_b200.h)
RK_PROFILE_CONV = 1
RK_PROFILE_SERIAL = 2
RK_PROFILE_TIMELINE = 4

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


def _fp(a):
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data_as(_f32p)


def _ip(a):
    if a.dtype != np.int32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous int32 array")
    return a.ctypes.data_as(_i32p)


def _check_size(a, n: int, what: str) -> None:
    # the C ABI reads exactly n elements through the pointer
    if a.size != n:
        raise ValueError(f"{what}: expected {n} elements, got shape {a.shape}")


class Context:
    def __init__(self, device: int = 0, precision: int = FP32, l_bucket: int = 32, max_tokens: int = 512):
        self._L = lib.load()
        opts = lib.rk_options(precision, max_tokens, l_bucket)
        h = ctypes.c_void_p()
        lib.check(self._L.rk_create(device, ctypes.byref(opts), ctypes.byref(h)), "rk_create")
        self.h = h
        self.precision = precision
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self._L.rk_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self) -> int:
        return self._L.rk_stream(self.h) or 0

    def load_weights(self, blob: bytes) -> None:
        buf = (ctypes.c_char * len(blob)).from_buffer_copy(blob) if not isinstance(blob, bytearray) else \
            (ctypes.c_char * len(blob)).from_buffer(blob)
        lib.check(self._L.rk_load_weights_koko(self.h, buf, len(blob)), "rk_load_weights_koko")

    def record(self, on: bool = True) -> None:
        lib.check(self._L.rk_record_stages(self.h, int(on)), "rk_record_stages")

    def stage(self, name: str) -> np.ndarray | None:
        n = ctypes.c_size_t(0)
        lib.check(self._L.rk_get_stage(self.h, name.encode(), None, 0, ctypes.byref(n)), "rk_get_stage")
        if n.value == 0:
            return None
        out = np.empty(n.value, np.float32)
        lib.check(self._L.rk_get_stage(self.h, name.encode(), _fp(out), n.value, ctypes.byref(n)), "rk_get_stage")
        return out

    def decode_features(self, asr, f0, n, style128) -> np.ndarray:
        asr = np.ascontiguousarray(asr, np.float32)
        if asr.ndim != 2 or asr.shape[1] != 512 or asr.shape[0] < 1:
            raise ValueError(f"decode_features: asr must be [L, 512] with L >= 1, got shape {asr.shape}")
        L = asr.shape[0]
        f0 = np.ascontiguousarray(f0, np.float32)
        n = np.ascontiguousarray(n, np.float32)
        s = np.ascontiguousarray(style128, np.float32)
        _check_size(f0, 2 * L, "decode_features: f0")
        _check_size(n, 2 * L, "decode_features: n")
        _check_size(s, 128, "decode_features: style")
        pcm = np.empty(600 * L, np.float32)
        lib.check(self._L.rk_decode_features(self.h, _fp(asr), _fp(f0), _fp(n), _fp(s), L, _fp(pcm)),
                  "rk_decode_features")
        return pcm

    def decode_features_device(self, d_asr: int, d_f0: int, d_n: int, d_style: int, L: int, d_pcm: int) -> None:
        lib.check(self._L.rk_decode_features_device(self.h, d_asr, d_f0, d_n, d_style, L, d_pcm),
                  "rk_decode_features_device")

    def infer(self, tokens, style256, dur_override=None):
        tok = np.ascontiguousarray(tokens, np.int32)
        if tok.ndim != 1:
            raise ValueError(f"infer: tokens must be 1-D, got shape {tok.shape}")
        T = tok.shape[0]
        s = np.ascontiguousarray(style256, np.float32)
        _check_size(s, 256, "infer: style")
        dov = None if dur_override is None else np.ascontiguousarray(dur_override, np.int32)
        if dov is not None:
            _check_size(dov, T, "infer: dur_override")
        dur = np.empty(T, np.int32)
        L = ctypes.c_int(0)
        cap = 600 * (int(dov.sum()) if dov is not None else 64 * T)
        pcm = np.empty(max(cap, 1), np.float32)
        n = ctypes.c_size_t(0)
        lib.check(self._L.rk_infer(self.h, _ip(tok), T, _fp(s), _ip(dov) if dov is not None else None, _ip(dur),
                                   ctypes.byref(L), _fp(pcm), pcm.shape[0], ctypes.byref(n)), "rk_infer")
        return pcm[: n.value].copy(), dur, L.value

    def encode(self, utterances, overrides=True):
        """rk_encode over a batch: utterances have .tokens, .style (256) and
        .durations (used as overrides when `overrides`).  Returns (predicted
        durations per utterance, L per utterance)."""
        toks = [np.ascontiguousarray(u.tokens, np.int32).reshape(-1) for u in utterances]
        Ts = np.array([t.shape[0] for t in toks], np.int32)
        tok = np.ascontiguousarray(np.concatenate(toks), np.int32)
        styles = [np.asarray(u.style, np.float32).reshape(-1) for u in utterances]
        for st in styles:
            _check_size(st, 256, "encode: style")
        sty = np.ascontiguousarray(np.stack(styles), np.float32)
        dov = None
        if overrides:
            durs = [np.asarray(u.durations, np.int32).reshape(-1) for u in utterances]
            for d, t in zip(durs, Ts):
                _check_size(d, int(t), "encode: durations")
            dov = np.ascontiguousarray(np.concatenate(durs), np.int32)
        dur = np.empty(tok.shape[0], np.int32)
        Ls = np.empty(len(toks), np.int32)
        lib.check(self._L.rk_encode(self.h, _ip(tok), _ip(Ts), len(toks), _fp(sty),
                                    _ip(dov) if dov is not None else None, _ip(dur), _ip(Ls)), "rk_encode")
        offs = np.concatenate([[0], np.cumsum(Ts)])
        return [dur[offs[i]:offs[i + 1]].copy() for i in range(len(toks))], [int(x) for x in Ls]

    def decode(self, Ls):
        """rk_decode of every pending utterance; Ls from encode().  Returns PCM per utterance."""
        total = 600 * int(sum(Ls))
        pcm = np.empty(max(total, 1), np.float32)
        ns = (ctypes.c_size_t * max(len(Ls), 1))()
        B = ctypes.c_int(0)
        lib.check(self._L.rk_decode(self.h, _fp(pcm), pcm.shape[0], ns, ctypes.byref(B)), "rk_decode")
        out, off = [], 0
        for i in range(B.value):
            out.append(pcm[off:off + ns[i]].copy())
            off += ns[i]
        return out

    def synthesize_stream(self, utterances, on_pcm, chunk: int = 8, overrides: bool = True) -> None:
        """rk_synthesize_stream: the utterances (.tokens, .style, .durations as
        overrides when `overrides`) in chunks of `chunk`, the front half of
        chunk k + 1 overlapping the decode of chunk k.  on_pcm(index, pcm)
        receives each utterance's PCM (a copy) in order and returns False to
        stop."""
        toks = [np.ascontiguousarray(u.tokens, np.int32).reshape(-1) for u in utterances]
        Ts = np.array([t.shape[0] for t in toks], np.int32)
        tok = np.ascontiguousarray(np.concatenate(toks), np.int32)
        sty = np.ascontiguousarray(np.stack([np.asarray(u.style, np.float32).reshape(256) for u in utterances]))
        dov = None
        if overrides:
            dov = np.ascontiguousarray(np.concatenate([np.asarray(u.durations, np.int32).reshape(-1)
                                                       for u in utterances]), np.int32)
        errors = []

        def cb(_user, index, pcm, n):
            try:
                arr = np.ctypeslib.as_array(pcm, shape=(n,)).copy() if n else np.zeros(0, np.float32)
                return 0 if on_pcm(index, arr) is False else 1
            except BaseException as e:  # surfaced after the call
                errors.append(e)
                return 0

        fn = lib.PCM_FN(cb)
        lib.check(self._L.rk_synthesize_stream(self.h, _ip(tok), _ip(Ts), len(toks), _fp(sty),
                                               _ip(dov) if dov is not None else None, int(chunk), fn, None),
                  "rk_synthesize_stream")
        if errors:
            raise errors[0]

    def profile(self, on=True) -> None:
        """on: False / True (conv events) or a set of RK_PROFILE_* bits (CONV 1, SERIAL 2, TIMELINE 4)."""
        lib.check(self._L.rk_profile(self.h, int(on)), "rk_profile")

    def profile_timeline(self):
        """[(stream, name, end_ms)] of every launch since the last call (RK_PROFILE_TIMELINE)."""
        n = ctypes.c_size_t(0)
        lib.check(self._L.rk_profile_timeline(self.h, None, 0, ctypes.byref(n)), "rk_profile_timeline")
        buf = ctypes.create_string_buffer(max(n.value, 1))
        lib.check(self._L.rk_profile_timeline(self.h, buf, len(buf), ctypes.byref(n)), "rk_profile_timeline")
        out = []
        for line in buf.value.decode().splitlines():
            sid, name, t = line.split("\t")
            out.append((int(sid), name, float(t)))
        return out

    def profile_read(self):
        """(conv device ms, conv algorithmic FLOPs, conv launches) since profile(True)."""
        ms, fl, n = ctypes.c_double(0), ctypes.c_double(0), ctypes.c_longlong(0)
        lib.check(self._L.rk_profile_read(self.h, ctypes.byref(ms), ctypes.byref(fl), ctypes.byref(n)),
                  "rk_profile_read")
        return ms.value, fl.value, n.value

    def kernel_count(self, reset: bool = False) -> int:
        c = ctypes.c_longlong(0)
        lib.check(self._L.rk_kernel_count(self.h, ctypes.byref(c), int(reset)), "rk_kernel_count")
        return c.value
