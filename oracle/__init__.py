"""CPU checker for the routed MoE block (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may import this module.
It loads two shared libraries built by oracle/Makefile:

* ``liboracle.so``: the restatement of the reference's MoE block in moe_oracle.c;
* ``_ref/libqref.so``: the reference's own engine sources (hatim-mlf/moe-stream-mac engine/src) plus
  ref_harness.c, built only where the reference checkout exists; absent elsewhere.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libqref.so"


class OrQMat(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("rows", C.c_int), ("cols", C.c_int), ("bits", C.c_int), ("group_size", C.c_int)]


class OrBlock(C.Structure):
    _fields_ = [("hidden", C.c_int), ("E", C.c_int), ("top_k", C.c_int), ("inter", C.c_int),
                ("sh_inter", C.c_int), ("router_f32", C.c_void_p), ("router_bias", C.c_void_p),
                ("router_q", OrQMat), ("gate", OrQMat), ("up", OrQMat), ("down", OrQMat),
                ("sh_gate", OrQMat), ("sh_up", OrQMat), ("sh_down", OrQMat),
                ("sh_gate_f32", C.c_void_p), ("sh_router_q", OrQMat)]


class OrSynthCfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("E", C.c_int), ("top_k", C.c_int), ("inter", C.c_int),
                ("sh_inter", C.c_int), ("bits", C.c_int), ("group_size", C.c_int), ("quant_router", C.c_int)]


def build() -> None:
    """Compile liboracle.so (and _ref/libqref.so where the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        fp, ip, vp = C.POINTER(C.c_float), C.POINTER(C.c_int), C.c_void_p
        L.or_bf16_to_f32.restype = C.c_float; L.or_bf16_to_f32.argtypes = [C.c_uint16]
        L.or_qgroup_dot.restype = C.c_float; L.or_qgroup_dot.argtypes = [vp, fp, C.c_int, C.c_int]
        L.or_qmat_matvec.argtypes = [C.POINTER(OrQMat), fp, fp]
        L.or_softmax.argtypes = [fp, fp, C.c_int]
        L.or_topk.argtypes = [ip, fp, C.c_int, C.c_int]
        L.or_silu_mul.argtypes = [fp, fp, fp, C.c_int]
        L.or_sigmoid.argtypes = [fp, fp, C.c_int]
        L.or_expf.restype = C.c_float; L.or_expf.argtypes = [C.c_float]
        L.or_expf_bits.argtypes = [C.c_uint32, C.c_longlong, fp]
        L.or_dot_f32.restype = C.c_float; L.or_dot_f32.argtypes = [fp, fp, C.c_int]
        L.or_router_logits.argtypes = [C.POINTER(OrBlock), fp, fp]
        L.or_route_from_logits.argtypes = [fp, C.c_int, C.c_int, fp, ip, fp]
        L.or_moe_step.argtypes = [C.POINTER(OrBlock), fp, fp, ip, fp]
        L.or_moe_forward.argtypes = [C.POINTER(OrBlock), C.c_int, fp, fp, ip, fp]
        L.or_expert_mlp.argtypes = [C.POINTER(OrBlock), C.c_int, fp, fp]
        L.or_shared_gate_logit.argtypes = [C.POINTER(OrBlock), fp, fp]
        L.or_synth_block.restype = C.POINTER(OrBlock)
        L.or_synth_block.argtypes = [C.POINTER(OrSynthCfg), C.c_uint64, C.c_uint32, fp]
        L.or_free_block.argtypes = [C.POINTER(OrBlock)]
        L.or_synth_x.argtypes = [fp, C.c_int, C.c_int, C.c_uint64, C.c_uint32]
        L.or_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_PATH.exists()


def ref() -> C.CDLL:
    """The reference's own engine code (oracle/_ref/libqref.so)."""
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise FileNotFoundError(f"{REF_PATH} not built (needs the reference checkout)")
        L = C.CDLL(str(REF_PATH))
        fp, ip, vp = C.POINTER(C.c_float), C.POINTER(C.c_int), C.c_void_p
        L.qmat_matvec.argtypes = [vp, fp, fp]
        L.qgroup_dot.restype = C.c_float; L.qgroup_dot.argtypes = [vp, fp, C.c_int, C.c_int]
        L.bf16_to_f32.restype = C.c_float; L.bf16_to_f32.argtypes = [C.c_uint16]
        L.op_softmax.argtypes = [fp, fp, C.c_int]
        L.op_topk.argtypes = [ip, fp, C.c_int, C.c_int]
        L.op_silu_mul.argtypes = [fp, fp, fp, C.c_int]
        L.op_sigmoid.argtypes = [fp, fp, C.c_int]
        L.ref_b_forward.argtypes = [C.POINTER(OrBlock), C.c_int, fp, fp, ip, fp]
        L.ref_r_open.restype = vp
        L.ref_r_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_r_step.argtypes = [vp, fp, fp]
        L.ref_r_step_with_topk.argtypes = [vp, C.c_int, fp, fp]
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_expert_gb_read.restype = C.c_double
        _ref = L
    return _ref


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


def iptr(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_int))


def qmat_struct(w: np.ndarray, s: np.ndarray, b: np.ndarray, rows: int, cols: int, bits: int, gs: int) -> OrQMat:
    return OrQMat(w.ctypes.data, s.ctypes.data, b.ctypes.data, rows, cols, bits, gs)


@dataclass(frozen=True)
class BlockCfg:
    """Shape of one routed MoE block (engine/include/moe_layer.h:19 fields plus the quantization)."""
    hidden: int
    E: int
    top_k: int
    inter: int
    sh_inter: int
    bits: int
    group_size: int = 64
    quant_router: bool = False

    def synth(self) -> OrSynthCfg:
        return OrSynthCfg(self.hidden, self.E, self.top_k, self.inter, self.sh_inter, self.bits,
                          self.group_size, int(self.quant_router))


class SynthBlock:
    """A synthetic block generated in host RAM by the oracle (same bits as the GPU generator)."""

    def __init__(self, cfg: BlockCfg, seed: int, block: int = 0, router_bias: np.ndarray | None = None):
        self.cfg, self.seed, self.block = cfg, seed, block
        sc = cfg.synth()
        self._bias = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)
        self.ptr = lib().or_synth_block(C.byref(sc), seed, block, None if self._bias is None else fptr(self._bias))
        if not self.ptr:
            raise MemoryError("or_synth_block failed")

    def close(self) -> None:
        if self.ptr:
            lib().or_free_block(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def x(self, T: int, seed: int | None = None) -> np.ndarray:
        x = np.empty((T, self.cfg.hidden), np.float32)
        lib().or_synth_x(fptr(x), T, self.cfg.hidden, self.seed if seed is None else seed, self.block)
        return x

    def forward(self, x: np.ndarray):
        """Oracle restatement: (out[T,hidden], idx[T,k], score[T,k])."""
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.cfg.top_k), np.int32)
        score = np.empty((T, self.cfg.top_k), np.float32)
        if lib().or_moe_forward(self.ptr, T, fptr(np.ascontiguousarray(x)), fptr(out), iptr(idx), fptr(score)):
            raise RuntimeError("or_moe_forward failed")
        return out, idx, score

    def forward_ref(self, x: np.ndarray):
        """The reference's own qmat_matvec/op_* under the Mode B harness: (out, idx, score)."""
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.cfg.top_k), np.int32)
        score = np.empty((T, self.cfg.top_k), np.float32)
        if ref().ref_b_forward(self.ptr, T, fptr(np.ascontiguousarray(x)), fptr(out), iptr(idx), fptr(score)):
            raise RuntimeError("ref_b_forward failed")
        return out, idx, score

    def expert(self, e: int, x: np.ndarray) -> np.ndarray:
        """One expert's MLP on one token (e = -1: the shared expert), moe_layer.c:20-26."""
        y = np.empty(self.cfg.hidden, np.float32)
        if lib().or_expert_mlp(self.ptr, e, fptr(np.ascontiguousarray(x, np.float32)), fptr(y)):
            raise RuntimeError("or_expert_mlp failed")
        return y

    def shared_gate_logit(self, x: np.ndarray) -> np.float32:
        g = np.empty(1, np.float32)
        if lib().or_shared_gate_logit(self.ptr, fptr(np.ascontiguousarray(x, np.float32)), fptr(g)):
            raise RuntimeError("or_shared_gate_logit failed")
        return g[0]

    def router_logits(self, x: np.ndarray) -> np.ndarray:
        T = x.shape[0]
        lg = np.empty((T, self.cfg.E), np.float32)
        for t in range(T):
            row = np.ascontiguousarray(x[t])
            out = lg[t]
            if lib().or_router_logits(self.ptr, fptr(row), out.ctypes.data_as(C.POINTER(C.c_float))):
                raise RuntimeError("router failed")
        return lg

    def arrays(self) -> dict:
        """numpy views of the generated tensors (MLX layout), for writing checkpoints and GPU upload."""
        b = self.ptr.contents
        cfg = self.cfg

        def q(m: OrQMat, n: int):
            wpr, ng = m.cols * m.bits // 32, m.cols // m.group_size
            w = np.ctypeslib.as_array(C.cast(m.w, C.POINTER(C.c_uint32)), (n * m.rows * wpr,))
            s = np.ctypeslib.as_array(C.cast(m.scales, C.POINTER(C.c_uint16)), (n * m.rows * ng,))
            bb = np.ctypeslib.as_array(C.cast(m.biases, C.POINTER(C.c_uint16)), (n * m.rows * ng,))
            shp = (n, m.rows) if n > 1 else (m.rows,)
            return w.reshape(*shp, wpr), s.reshape(*shp, ng), bb.reshape(*shp, ng)

        out = {"gate": q(b.gate, cfg.E), "up": q(b.up, cfg.E), "down": q(b.down, cfg.E),
               "sh_gate": q(b.sh_gate, 1), "sh_up": q(b.sh_up, 1), "sh_down": q(b.sh_down, 1)}
        if cfg.quant_router:
            out["router_q"] = q(b.router_q, 1)
            out["sh_router_q"] = q(b.sh_router_q, 1)
        else:
            out["router_f32"] = np.ctypeslib.as_array(C.cast(b.router_f32, C.POINTER(C.c_float)),
                                                      (cfg.E * cfg.hidden,)).reshape(cfg.E, cfg.hidden)
            out["sh_gate_f32"] = np.ctypeslib.as_array(C.cast(b.sh_gate_f32, C.POINTER(C.c_float)),
                                                       (cfg.hidden,))
        return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().or_softmax(fptr(out), fptr(x), x.size)
    return out


def topk(x: np.ndarray, k: int, guard: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    idx = np.full(k + guard, -7, np.int32)
    lib().or_topk(iptr(idx), fptr(x), x.size, k)
    return idx


def expf_bits(lo: int, n: int) -> np.ndarray:
    """Host C-library expf of the n floats whose bit patterns start at lo."""
    y = np.empty(n, np.float32)
    lib().or_expf_bits(lo, n, fptr(y))
    return y


def route_from_logits(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, np.float32)
    E = logits.size
    probs = np.empty(E, np.float32); idx = np.empty(k, np.int32); score = np.empty(k, np.float32)
    if lib().or_route_from_logits(fptr(logits), E, k, fptr(probs), iptr(idx), fptr(score)):
        raise ValueError("bad top_k")
    return probs, idx, score


def qmat_matvec(w, s, b, rows, cols, bits, gs, x) -> tuple[int, np.ndarray]:
    m = qmat_struct(w, s, b, rows, cols, bits, gs)
    y = np.full(rows, 42.0, np.float32)
    rc = lib().or_qmat_matvec(C.byref(m), fptr(np.ascontiguousarray(x, np.float32)), fptr(y))
    return rc, y


os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
