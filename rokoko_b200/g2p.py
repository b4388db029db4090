"""Neural phonemizer: the host side of rokoko::G2PModelCuda (src/g2p.h:374-430).

    m = G2PModel()                      # its own rk_ctx on device 0, or G2PModel(ctx=...)
    m.load("g2p.bin")                   # a G2P3 file (or m.load_bytes(blob))
    m.infer("hello world")              # -> IPA string, as the reference's infer()
    m.infer_batch(["hello", "world"])   # many texts in one device pass
    m.loaded(), m.param_bytes(), m.free()

Method names, arguments and results follow the reference class: load() returns
False on an unreadable or unsupported file (the reason in rk_last_error),
infer() returns "" when nothing is loaded, for an empty text and for texts
longer than 2048 characters.  The model runs on the tcgen05 kernels of
librokoko_b200.so (rk_g2p_* entry points); there is no other path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib
from .context import FP32, Context


class G2PModel:
    def __init__(self, device: int = 0, ctx: Context | None = None):
        self._own = ctx is None
        self.ctx = ctx if ctx is not None else Context(device, FP32)
        self._L = lib.load()
        self._loaded = False

    # ---- the reference's interface
    def load(self, path: str) -> bool:
        try:
            with open(path, "rb") as f:
                blob = f.read()
        except OSError:
            return False
        return self.load_bytes(blob)

    def load_bytes(self, blob: bytes) -> bool:
        buf = ctypes.create_string_buffer(blob, len(blob))
        st = self._L.rk_g2p_load(self.ctx.h, buf, len(blob))
        if st == lib.RK_OK:  # a failed load leaves the model loaded before in place
            self._loaded = True
        return st == lib.RK_OK

    def loaded(self) -> bool:
        return self._loaded

    def param_bytes(self) -> int:
        return int(self._L.rk_g2p_param_bytes(self.ctx.h))

    def free(self) -> None:
        if self.ctx.h:
            self._L.rk_g2p_free(self.ctx.h)
        self._loaded = False

    def infer(self, text: str) -> str:
        if not self._loaded:
            return ""
        return self.infer_batch([text])[0]

    # ---- batched form
    def infer_batch(self, texts: list[str]) -> list[str]:
        if not self._loaded:
            return [""] * len(texts)
        n = len(texts)
        if n == 0:
            return []
        enc = [t.encode("utf-8") for t in texts]
        arr = (ctypes.c_char_p * n)(*enc)
        lens = (ctypes.c_size_t * n)(*[len(b) for b in enc])
        out_len = (ctypes.c_size_t * n)()
        cap = sum(12 * len(b) + 16 for b in enc)  # up to 3 phones of <= 4 bytes per character
        out = ctypes.create_string_buffer(cap)
        st = self._L.rk_g2p_infer(self.ctx.h, arr, lens, n, out, cap, out_len)
        if st == lib.RK_ERR_WORKSPACE:
            cap = sum(out_len) + 16
            out = ctypes.create_string_buffer(cap)
            st = self._L.rk_g2p_infer(self.ctx.h, arr, lens, n, out, cap, out_len)
        lib.check(st, "rk_g2p_infer")
        res, off = [], 0
        raw = out.raw
        for i in range(n):
            res.append(raw[off:off + out_len[i]].decode("utf-8"))
            off += out_len[i]
        return res

    def frames(self) -> np.ndarray:
        """Per-frame CTC ids of the last infer call (texts in order)."""
        n = ctypes.c_size_t(0)
        lib.check(self._L.rk_g2p_frames(self.ctx.h, None, 0, ctypes.byref(n)), "rk_g2p_frames")
        out = np.zeros(max(n.value, 1), np.int32)
        lib.check(self._L.rk_g2p_frames(self.ctx.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        out.size, ctypes.byref(n)), "rk_g2p_frames")
        return out[: n.value]

    def close(self) -> None:
        self.free()
        if self._own:
            self.ctx.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
