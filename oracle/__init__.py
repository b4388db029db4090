"""ctypes front-end of the CPU parity oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py.  The product package
(rokoko_b200) never imports this module.

The oracle restates rokoko's inference (src/rokoko.cpp:829-1297 and the kernel
semantics of src/kernels.cu) in FP32 C++; see oracle/oracle.cpp for the
function-by-function citations.  Parity status: per-kernel semantics pinned
against fixtures produced by the reference's own CUDA kernels (tests/golden/);
the model-level composition is unpinned (the reference ships no golden
vectors).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)


def _has_g2p(path: str) -> bool:
    with open(path, "rb") as f:
        return b"og2p_forward" in f.read()


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or not _has_g2p(_LIB_PATH):
            build(force=True)
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_load.restype = ctypes.c_void_p
        L.orc_load.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
        L.orc_free.argtypes = [ctypes.c_void_p]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_get_threads.restype = ctypes.c_int
        L.orc_record_stages.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_get_stage.restype = ctypes.c_long
        L.orc_get_stage.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _f32p, ctypes.c_long]
        L.orc_decode_features.restype = ctypes.c_int
        L.orc_decode_features.argtypes = [ctypes.c_void_p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int, _f32p]
        L.orc_infer.restype = ctypes.c_int
        L.orc_infer.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p, _i32p, ctypes.c_int,
                                _i32p, _i32p, _i32p, _f32p, ctypes.c_long]
        L.orc_sinegen.argtypes = [_f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p]
        L.orc_stft.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_int]
        L.orc_istft.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_int]
        L.orc_rand_ini.argtypes = [_f32p]
        c_int, c_long, c_float = ctypes.c_int, ctypes.c_long, ctypes.c_float
        L.orc_adain.argtypes = [_f32p, c_int, c_int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
        L.orc_layer_norm.argtypes = [_f32p, c_int, c_int, _f32p, _f32p, c_float, c_int, _f32p]
        L.orc_durations_alignment.restype = c_int
        L.orc_durations_alignment.argtypes = [_f32p, c_int, _i32p, _f32p, c_int]
        L.orc_sigmoid_sum.argtypes = [_f32p, c_int, c_int, _f32p]
        L.orc_lstm_gates.argtypes = [_f32p, _f32p, c_int, _f32p, _f32p]
        L.orc_conv1d.argtypes = [_f32p, _f32p, _f32p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, _f32p]
        L.orc_convT_depthwise_k3s2.argtypes = [_f32p, _f32p, _f32p, c_int, c_int, _f32p]
        L.orc_weight_norm.argtypes = [_f32p, _f32p, c_int, c_long, _f32p]
        L.orc_gelu.argtypes = [_f32p, c_long, _f32p]
        L.orc_softmax.argtypes = [_f32p, c_int, c_int, _f32p]
        L.og2p_load.restype = ctypes.c_void_p
        L.og2p_load.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        L.og2p_free.argtypes = [ctypes.c_void_p]
        L.og2p_dims.argtypes = [ctypes.c_void_p, _i32p]
        L.og2p_ids.restype = c_int
        L.og2p_ids.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, _i32p, ctypes.c_size_t]
        L.og2p_forward.restype = c_long
        L.og2p_forward.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, _f32p, ctypes.c_size_t,
                                   _i32p, ctypes.c_size_t]
        L.og2p_ctc.restype = c_long
        L.og2p_ctc.argtypes = [ctypes.c_void_p, _i32p, c_long, ctypes.c_char_p, ctypes.c_size_t]
        _lib = L
    return _lib


def _fp(a: np.ndarray):
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data_as(_f32p)


def _ip(a: np.ndarray):
    if a.dtype != np.int32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous int32 array")
    return a.ctypes.data_as(_i32p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


class Oracle:
    """One loaded model (KOKO v1 blob).  fp16=True restates the FP16-weights
    variant (src/rokoko_f16.cpp): FP16 weights and FP16-rounded GEMM inputs."""

    def __init__(self, blob: bytes, fp16: bool = False):
        err = ctypes.create_string_buffer(256)
        self._buf = ctypes.create_string_buffer(blob, len(blob))
        self._h = lib().orc_load(self._buf, len(blob), int(fp16), err, 256)
        del self._buf
        if not self._h:
            raise RuntimeError("oracle load failed: " + err.value.decode())
        self.fp16 = fp16

    def close(self):
        if self._h:
            lib().orc_free(self._h)
            self._h = None

    __del__ = close

    def record(self, on: bool = True):
        lib().orc_record_stages(self._h, int(on))

    def stage(self, name: str) -> np.ndarray | None:
        n = lib().orc_get_stage(self._h, name.encode(), None, 0)
        if n == 0:
            return None
        out = np.empty(n, np.float32)
        lib().orc_get_stage(self._h, name.encode(), _fp(out), n)
        return out

    def decode_features(self, asr, f0, n, style128) -> np.ndarray:
        asr = np.ascontiguousarray(asr, np.float32)
        L = asr.shape[0]
        f0 = np.ascontiguousarray(f0, np.float32)
        n = np.ascontiguousarray(n, np.float32)
        s = np.ascontiguousarray(style128, np.float32)
        out = np.empty(600 * L, np.float32)
        rc = lib().orc_decode_features(self._h, _fp(asr), _fp(f0), _fp(n), _fp(s), L, _fp(out))
        if rc:
            raise RuntimeError("oracle decode failed")
        return out

    def infer(self, tokens, style256, dur_override=None, bucket: int = 32):
        tok = np.ascontiguousarray(tokens, np.int32)
        T = tok.shape[0]
        s = np.ascontiguousarray(style256, np.float32)
        dov = None if dur_override is None else np.ascontiguousarray(dur_override, np.int32)
        dur = np.empty(T, np.int32)
        L = ctypes.c_int(0)
        Lb = ctypes.c_int(0)
        cap = 600 * (int(dov.sum()) if dov is not None else 64 * T) + 1
        pcm = np.empty(cap, np.float32)
        rc = lib().orc_infer(self._h, _ip(tok), T, _fp(s), _ip(dov) if dov is not None else None, bucket,
                             _ip(dur), ctypes.byref(L), ctypes.byref(Lb), _fp(pcm), cap)
        if rc:
            raise RuntimeError("oracle infer failed")
        return pcm[: 600 * L.value].copy(), dur, L.value, Lb.value


def sinegen(f0, lw, lb):
    f0 = np.ascontiguousarray(f0, np.float32)
    L2 = f0.shape[0]
    ph = np.empty(L2 * 9, np.float32)
    src = np.empty(L2 * 300, np.float32)
    lib().orc_sinegen(_fp(f0), L2, _fp(np.ascontiguousarray(lw, np.float32)),
                      _fp(np.ascontiguousarray(lb, np.float32)), _fp(ph), _fp(src))
    return ph.reshape(L2, 9), src


def stft(x):
    x = np.ascontiguousarray(x, np.float32)
    T2 = x.shape[0] // 5 + 1
    har = np.empty((T2, 22), np.float32)
    lib().orc_stft(_fp(x), x.shape[0], _fp(har), T2)
    return har


def istft(c, T_audio):
    c = np.ascontiguousarray(c, np.float32)
    y = np.empty(T_audio, np.float32)
    lib().orc_istft(_fp(c), c.shape[0], _fp(y), T_audio)
    return y


def rand_ini():
    r = np.empty(9, np.float32)
    lib().orc_rand_ini(_fp(r))
    return r


# ---- single-op restatements (pinned against the reference's own kernels by
# tests/test_golden.py)

def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype)


def _fpn(a):
    return None if a is None else _fp(a)


def adain(x, norm_w, norm_b, gamma, beta, alpha=None):
    """InstanceNorm + style affine (+ Snake) on x [T, C]."""
    x, norm_w, norm_b, gamma, beta = map(_c, (x, norm_w, norm_b, gamma, beta))
    alpha = None if alpha is None else _c(alpha)
    T, C = x.shape
    y = np.empty_like(x)
    lib().orc_adain(_fp(x), T, C, _fp(norm_w), _fp(norm_b), _fp(gamma), _fp(beta), _fpn(alpha), _fp(y))
    return y


def layer_norm(x, gamma, beta, eps, ada=False):
    x, gamma, beta = map(_c, (x, gamma, beta))
    N, D = x.shape
    y = np.empty_like(x)
    lib().orc_layer_norm(_fp(x), N, D, _fp(gamma), _fp(beta), float(eps), int(bool(ada)), _fp(y))
    return y


def durations_alignment(dur, max_L=1 << 16):
    """float durations [T] -> (int durations [T], L, alignment [T, L])."""
    dur = _c(dur)
    T = dur.shape[0]
    idur = np.empty(T, np.int32)
    L = lib().orc_durations_alignment(_fp(dur), T, _ip(idur), None, 0)
    align = np.empty((T, L), np.float32)
    lib().orc_durations_alignment(_fp(dur), T, _ip(idur), _fp(align), L)
    return idur, L, align


def sigmoid_sum(x):
    x = _c(x)
    y = np.empty(x.shape[0], np.float32)
    lib().orc_sigmoid_sum(_fp(x), x.shape[0], x.shape[1], _fp(y))
    return y


def lstm_gates(gates, c_prev):
    gates, c_prev = _c(gates), _c(c_prev)
    H = c_prev.shape[0]
    c = np.empty(H, np.float32)
    h = np.empty(H, np.float32)
    lib().orc_lstm_gates(_fp(gates), _fp(c_prev), H, _fp(c), _fp(h))
    return c, h


def conv1d(x, w, bias, stride=1, pad=0, dil=1):
    """x [T_in, Ci], w [Co, Ci, K] -> y [T_out, Co]."""
    x, w = _c(x), _c(w)
    bias = None if bias is None else _c(bias)
    T_in, Ci = x.shape
    Co, _, K = w.shape
    T_out = (T_in + 2 * pad - dil * (K - 1) - 1) // stride + 1
    y = np.empty((T_out, Co), np.float32)
    lib().orc_conv1d(_fp(x), _fp(w), _fpn(bias), Ci, Co, T_in, K, stride, pad, dil, _fp(y))
    return y


def conv_transpose_depthwise_k3s2(x, w, b):
    x, w, b = map(_c, (x, w, b))
    T, C = x.shape
    y = np.empty((2 * T, C), np.float32)
    lib().orc_convT_depthwise_k3s2(_fp(x), _fp(w), _fp(b), C, T, _fp(y))
    return y


def weight_norm(g, v):
    g, v = _c(g), _c(v)
    w = np.empty_like(v)
    lib().orc_weight_norm(_fp(g), _fp(v), v.shape[0], v.size // v.shape[0], _fp(w))
    return w


def gelu(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_gelu(_fp(x), x.size, _fp(y))
    return y


def softmax(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_softmax(_fp(x), x.shape[0], x.shape[1], _fp(y))
    return y


class G2POracle:
    """The CPU restatement of rokoko's G2P3 phonemizer (oracle/g2p.cpp) for one
    G2P3 blob: ids, logits, per-frame argmax and the CTC string of a text."""

    def __init__(self, blob: bytes):
        err = ctypes.create_string_buffer(256)
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._h = lib().og2p_load(buf, len(blob), err, 256)
        if not self._h:
            raise RuntimeError("G2P oracle load failed: " + err.value.decode())
        dims = np.zeros(7, np.int32)
        lib().og2p_dims(self._h, _ip(dims))
        self.d, self.heads, self.n_layers, self.ff, self.up, self.n_chars, self.n_phones = (int(x) for x in dims)

    def close(self):
        if self._h:
            lib().og2p_free(self._h)
            self._h = None

    __del__ = close

    def ids(self, text: str) -> np.ndarray:
        b = text.encode("utf-8")
        out = np.zeros(len(b) + 1, np.int32)
        n = lib().og2p_ids(self._h, b, len(b), _ip(out), out.size)
        return out[:n]

    def forward(self, text: str) -> tuple[np.ndarray, np.ndarray]:
        """(logits [T*up][n_phones], argmax ids [T*up]); empty for "" or > 2048 characters."""
        b = text.encode("utf-8")
        rows = (len(b) + 1) * self.up
        logits = np.zeros(rows * self.n_phones, np.float32)
        best = np.zeros(rows, np.int32)
        n = lib().og2p_forward(self._h, b, len(b), _fp(logits), logits.size, _ip(best), best.size)
        if n < 0:
            raise RuntimeError("og2p_forward: buffer too small")
        return logits[: n * self.n_phones].reshape(n, self.n_phones), best[:n]

    def ctc(self, best: np.ndarray) -> str:
        best = np.ascontiguousarray(best, np.int32)
        cap = 4 * best.size + 4
        out = ctypes.create_string_buffer(cap)
        n = lib().og2p_ctc(self._h, _ip(best), best.size, out, cap)
        return out.raw[:n].decode("utf-8")

    def infer(self, text: str) -> str:
        return self.ctc(self.forward(text)[1])
