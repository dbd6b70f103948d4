"""Engine: the whole-model API of include/qe_engine.h from Python, in the shape of the reference front end's own
ctypes class (engine/cli/qchat.py:34-76: forward, prefill, reset, position, max_len, set_threads, stats).

The routed MoE block of every layer runs on the GPU; the rest of each layer runs on the host
(moe-stream-mac_b200/csrc/engine.cu)."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from .lib import LIB_PATH


class ContextFull(Exception):
    pass


class Engine:
    def __init__(self, model_dir: str | Path, ctx: int, lib_path: str | Path = LIB_PATH):
        L = self.lib = C.CDLL(str(lib_path))
        L.qe_load.restype = C.c_void_p
        L.qe_load.argtypes = [C.c_char_p, C.c_int]
        for name in ("qe_reset", "qe_free"):
            getattr(L, name).argtypes = [C.c_void_p]
        L.qe_forward.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_float)]
        for name in ("qe_vocab", "qe_position", "qe_max_len"):
            getattr(L, name).argtypes = [C.c_void_p]
        L.qe_set_threads.argtypes = [C.c_int]
        for name in ("qe_expert_gb_read", "qe_expert_read_seconds", "qe_peak_rss_gb"):
            getattr(L, name).restype = C.c_double
        self.handle = L.qe_load(str(model_dir).encode(), int(ctx))
        if not self.handle:
            raise RuntimeError(f"engine could not load {model_dir} (see the message above)")
        self.vocab = L.qe_vocab(self.handle)
        self.logits = np.zeros(self.vocab, dtype=np.float32)
        self._ptr = self.logits.ctypes.data_as(C.POINTER(C.c_float))

    def forward(self, token: int) -> np.ndarray:
        rc = self.lib.qe_forward(self.handle, int(token), self._ptr)
        if rc == -2:
            raise ContextFull()
        if rc != 0:
            raise RuntimeError("engine forward failed")
        return self.logits

    def prefill(self, tokens: list[int]) -> np.ndarray:
        logits = self.logits
        for tok in tokens:
            logits = self.forward(tok)
        return logits

    def reset(self) -> None:
        self.lib.qe_reset(self.handle)

    def position(self) -> int:
        return self.lib.qe_position(self.handle)

    def max_len(self) -> int:
        return self.lib.qe_max_len(self.handle)

    def set_threads(self, n: int) -> int:
        return self.lib.qe_set_threads(n)

    def stats(self) -> dict:
        L = self.lib
        return {"peak_rss_gb": L.qe_peak_rss_gb(), "expert_gb_read": L.qe_expert_gb_read(),
                "expert_read_s": L.qe_expert_read_seconds(), "position": self.position(), "max_len": self.max_len()}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.qe_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
