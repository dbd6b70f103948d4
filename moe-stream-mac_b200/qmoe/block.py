"""MoeBlock: one routed MoE block resident on a B200 (the GPU counterpart of MoeWeights + moe_layer_step)."""
from __future__ import annotations

import ctypes as C
from typing import Mapping

import numpy as np

from .lib import QE_ROUTER_F32, QE_ROUTER_QMAT, QeMoeConfig, QeMoeWeights, QeQTensor, fptr, iptr, lib


class EngineError(RuntimeError):
    pass


def _qt(triple) -> QeQTensor:
    if triple is None:
        return QeQTensor(None, None, None)
    w, s, b = triple
    return QeQTensor(w.ctypes.data, s.ctypes.data, b.ctypes.data)


class MoeBlock:
    """Handle around qe_moe_create/qe_moe_forward (include/qe_moe.h).

    Construct with host weights (MLX layout, as a checkpoint stores them) or synthetically in HBM.
    forward() takes host float32 arrays x[T][hidden] and returns out[T][hidden]; forward_device() takes
    device pointers (e.g. torch tensors' data_ptr()) and a stream, without host synchronisation.
    """

    def __init__(self, hidden: int, E: int, top_k: int, inter: int, sh_inter: int, bits: int, group_size: int = 64,
                 *, router_mode: int = QE_ROUTER_F32, router_bits: int = 8, max_tokens: int = 4096, device: int = 0,
                 layer: int = 0, weights: Mapping | None = None, seed: int | None = None, block: int = 0,
                 router_bias: np.ndarray | None = None, ep_rank: int = 0, ep_size: int = 1, placement=None):
        self.cfg = QeMoeConfig(hidden, E, top_k, inter, sh_inter, bits, group_size, router_mode, router_bits,
                               max_tokens, device, layer, ep_rank, ep_size)
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self.hidden, self.top_k, self.E = hidden, top_k, E
        L = lib()
        self._keep = []
        self._set_placement(placement)
        if weights is not None:
            w = QeMoeWeights()
            if router_mode == QE_ROUTER_F32:
                rf = np.ascontiguousarray(weights["router_f32"], np.float32)
                sg = np.ascontiguousarray(weights["sh_gate_f32"], np.float32)
                self._keep += [rf, sg]
                w.router_f32, w.sh_gate_f32 = rf.ctypes.data, sg.ctypes.data
                rb = weights.get("router_bias") if router_bias is None else router_bias
                if rb is not None:
                    rb = np.ascontiguousarray(rb, np.float32)
                    self._keep.append(rb)
                    w.router_bias = rb.ctypes.data
            else:
                w.router_q, w.sh_router_q = _qt(weights["router_q"]), _qt(weights["sh_router_q"])
            for name in ("gate", "up", "down", "sh_gate", "sh_up", "sh_down"):
                setattr(w, name, _qt(weights[name]))
            self.handle = L.qe_moe_create(C.byref(self.cfg), C.byref(w))
        else:
            rb = None
            if router_bias is not None:
                rb = np.ascontiguousarray(router_bias, np.float32)
                self._keep.append(rb)
            self.handle = L.qe_moe_create_synthetic(C.byref(self.cfg), int(seed or 0), block,
                                                    None if rb is None else fptr(rb))
        if not self.handle:
            raise EngineError("qe_moe_create failed (see the message above)")

    @classmethod
    def from_safetensors(cls, directory: str, prefix: str, top_k: int, group_size: int = 64, *, max_tokens: int = 4096,
                         device: int = 0, layer: int = 0, ep_rank: int = 0, ep_size: int = 1,
                         placement=None) -> "MoeBlock":
        """One layer's block from an MLX checkpoint directory (qe_moe_open_safetensors): the shapes come
        from the tensors, e.g. prefix="language_model.model.layers.3.mlp"."""
        self = cls.__new__(cls)
        self.cfg = QeMoeConfig(0, 0, top_k, 0, 0, 0, group_size, QE_ROUTER_QMAT, 0, max_tokens, device, layer,
                               ep_rank, ep_size)
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self._keep = []
        self._set_placement(placement)
        self.handle = lib().qe_moe_open_safetensors(str(directory).encode(), prefix.encode(), C.byref(self.cfg))
        if not self.handle:
            raise EngineError("qe_moe_open_safetensors failed (see the message above)")
        L = lib()
        self.hidden, self.top_k = L.qe_moe_hidden(self.handle), top_k
        self.E = None
        return self

    def _set_placement(self, placement) -> None:
        """cfg.placement from a qmoe.placement.Placement or an int32 [ep_size][slots] table (None: contiguous)."""
        if placement is None:
            return
        table = np.ascontiguousarray(getattr(placement, "table", placement), np.int32)
        if table.ndim != 2:
            raise ValueError("placement must be a [ep_size][slots] table")
        self._keep.append(table)
        self.cfg.placement, self.cfg.slots = table.ctypes.data, table.shape[1]

    def held_experts(self) -> np.ndarray:
        """Global ids of the routed experts this handle holds, in slot order (qe_moe_ep_experts)."""
        n = lib().qe_moe_ep_experts(self.handle, None)
        ids = np.empty(max(n, 0), np.int32)
        lib().qe_moe_ep_experts(self.handle, iptr(ids))
        return ids

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().qe_moe_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = x.shape[0]
        if out is None:
            out = np.empty_like(x)
        if lib().qe_moe_forward(self.handle, T, fptr(x), fptr(out)):
            raise EngineError("qe_moe_forward failed")
        return out

    def forward_async(self, x: np.ndarray, out: np.ndarray) -> None:
        """qe_moe_forward_async: enqueue the forward of host x[T][hidden] into host out (both C-contiguous
        float32; pinned memory, e.g. torch's pin_memory().numpy(), for the copies to overlap the kernels).
        out is written by the time wait() returns; both arrays are kept alive until then."""
        if x.dtype != np.float32 or out.dtype != np.float32 or not x.flags.c_contiguous or not out.flags.c_contiguous \
                or x.shape != out.shape or x.ndim != 2:
            raise ValueError("x and out must be C-contiguous float32 [T][hidden] arrays of one shape")
        self._inflight = getattr(self, "_inflight", [])
        self._inflight.append((x, out))
        if lib().qe_moe_forward_async(self.handle, x.shape[0], fptr(x), fptr(out)):
            raise EngineError("qe_moe_forward_async failed")

    def wait(self) -> None:
        """qe_moe_forward_wait: every forward_async call on this block's device has written its out."""
        rc = lib().qe_moe_forward_wait(self.handle)
        self._inflight = []
        if rc:
            raise EngineError("qe_moe_forward_wait failed")

    def forward_device(self, T: int, x_ptr: int, out_ptr: int, stream: int = 0) -> None:
        if lib().qe_moe_forward_device(self.handle, T, C.c_void_p(x_ptr), C.c_void_p(out_ptr), C.c_void_p(stream)):
            raise EngineError("qe_moe_forward_device failed")

    def graph(self, T: int, x_ptr: int, out_ptr: int) -> "ForwardGraph":
        """forward_device of T tokens on fixed device buffers, captured into a CUDA graph (qe_moe_graph_create)."""
        return ForwardGraph(self, T, x_ptr, out_ptr)

    def route(self, x: np.ndarray):
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = x.shape[0]
        idx = np.empty((T, self.top_k), np.int32)
        score = np.empty((T, self.top_k), np.float32)
        if lib().qe_moe_route(self.handle, T, fptr(x), iptr(idx), fptr(score)):
            raise EngineError("qe_moe_route failed")
        return idx, score

    @property
    def weight_bytes(self) -> int:
        return lib().qe_moe_weight_bytes(self.handle)


class ForwardGraph:
    """A captured forward (include/qe_moe.h qe_moe_graph_*); launch() replays it on a stream."""

    def __init__(self, block: MoeBlock, T: int, x_ptr: int, out_ptr: int):
        self.block = block   # keeps the weights alive
        self.handle = lib().qe_moe_graph_create(block.handle, T, C.c_void_p(x_ptr), C.c_void_p(out_ptr))
        if not self.handle:
            raise EngineError("qe_moe_graph_create failed")

    def launch(self, stream: int = 0) -> None:
        if lib().qe_moe_graph_launch(self.handle, C.c_void_p(stream)):
            raise EngineError("qe_moe_graph_launch failed")

    def _set_placement(self, placement) -> None:
        """cfg.placement from a qmoe.placement.Placement or an int32 [ep_size][slots] table (None: contiguous)."""
        if placement is None:
            return
        table = np.ascontiguousarray(getattr(placement, "table", placement), np.int32)
        if table.ndim != 2:
            raise ValueError("placement must be a [ep_size][slots] table")
        self._keep.append(table)
        self.cfg.placement, self.cfg.slots = table.ctypes.data, table.shape[1]

    def held_experts(self) -> np.ndarray:
        """Global ids of the routed experts this handle holds, in slot order (qe_moe_ep_experts)."""
        n = lib().qe_moe_ep_experts(self.handle, None)
        ids = np.empty(max(n, 0), np.int32)
        lib().qe_moe_ep_experts(self.handle, iptr(ids))
        return ids

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().qe_moe_graph_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
