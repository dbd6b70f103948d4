"""ctypes binding of include/qe_moe.h (argtypes/restype set once, as engine/cli/qchat.py:40-48 does)."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = PKG / "lib" / "libqengine_b200.so"

QE_ROUTER_F32 = 0
QE_ROUTER_QMAT = 1
QE_EP_ROUTED = 0x40000000   # tag of the slot ids routed to the destination rank in packed slot lists


class QeMoeConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("E", C.c_int), ("top_k", C.c_int), ("inter", C.c_int), ("sh_inter", C.c_int),
                ("bits", C.c_int), ("group_size", C.c_int), ("router_mode", C.c_int), ("router_bits", C.c_int),
                ("max_tokens", C.c_int), ("device", C.c_int), ("layer", C.c_int), ("ep_rank", C.c_int),
                ("ep_size", C.c_int), ("placement", C.c_void_p), ("slots", C.c_int)]


class QeQTensor(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class QeMoeWeights(C.Structure):
    _fields_ = [("router_f32", C.c_void_p), ("router_bias", C.c_void_p), ("sh_gate_f32", C.c_void_p),
                ("router_q", QeQTensor), ("sh_router_q", QeQTensor),
                ("gate", QeQTensor), ("up", QeQTensor), ("down", QeQTensor),
                ("sh_gate", QeQTensor), ("sh_up", QeQTensor), ("sh_down", QeQTensor)]


def build() -> None:
    """Compile libqengine_b200.so in-tree (nvcc -gencode arch=compute_100a,code=sm_100a)."""
    subprocess.run(["make", "-s", "-C", str(PKG)], check=True)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `make -C {PKG}` (no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        vp, fp, ip = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32)
        L.qe_moe_create.restype = vp
        L.qe_moe_create.argtypes = [C.POINTER(QeMoeConfig), C.POINTER(QeMoeWeights)]
        L.qe_moe_create_synthetic.restype = vp
        L.qe_moe_create_synthetic.argtypes = [C.POINTER(QeMoeConfig), C.c_uint64, C.c_uint32, fp]
        L.qe_moe_free.argtypes = [vp]
        L.qe_moe_forward.argtypes = [vp, C.c_int, fp, fp]
        L.qe_moe_forward_device.argtypes = [vp, C.c_int, vp, vp, vp]
        L.qe_moe_route.argtypes = [vp, C.c_int, fp, ip, fp]
        for name in ("qe_moe_hidden", "qe_moe_top_k"):
            getattr(L, name).argtypes = [vp]
        L.qe_moe_weight_bytes.restype = C.c_size_t
        L.qe_moe_weight_bytes.argtypes = [vp]
        L.qe_qmat_matvec.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, fp, fp]
        L.qe_route_logits.argtypes = [C.c_int, C.c_int, C.c_int, fp, fp, ip, fp]
        L.qe_op_silu_mul.argtypes = [fp, fp, fp, C.c_int]
        L.qe_op_sigmoid.argtypes = [fp, fp, C.c_int]
        L.qe_op_expf.argtypes = [fp, fp, C.c_int]
        for name in ("qe_expert_gb_read", "qe_expert_read_seconds", "qe_peak_rss_gb"):
            getattr(L, name).restype = C.c_double
        L.qe_set_threads.argtypes = [C.c_int]
        L.qe_set_threads.restype = C.c_int
        L.qe_profile_begin.argtypes = [C.c_int]
        L.qe_profile_end.argtypes = [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int)]
        L.qe_kernel_launches.restype = C.c_ulonglong
        L.qe_graph_captures.restype = C.c_ulonglong
        L.qe_device_error.restype = C.c_int
        L.qe_device_error_on.argtypes = [C.c_int]
        L.qe_device_error_reset.argtypes = [C.c_int]
        L.qe_ep_xchg_set_timeout_ms.argtypes = [vp, C.c_int]
        L.qe_route_f32_noalloc.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp]
        L.qe_moe_ep_route_device.argtypes = [vp, C.c_int, vp, vp, vp, vp]
        L.qe_moe_forward_async.argtypes = [vp, C.c_int, vp, vp]
        L.qe_moe_forward_wait.argtypes = [vp]
        L.qe_moe_ep_pack_device.argtypes = [vp, C.c_int, vp, vp, vp, vp, vp, vp, vp]
        L.qe_moe_ep_experts_device.argtypes = [vp, C.c_int, vp, vp, vp, vp]
        L.qe_moe_ep_combine_device.argtypes = [vp, C.c_int, vp, vp, vp, vp, vp]
        L.qe_moe_ep_size.argtypes = [vp]
        L.qe_moe_ep_experts.argtypes = [vp, ip]
        L.qe_ep_xchg_create.restype = vp
        L.qe_ep_xchg_create.argtypes = [vp, C.c_int, vp]
        L.qe_ep_xchg_handle_bytes.restype = C.c_int
        L.qe_ep_xchg_connect.argtypes = [vp, vp]
        L.qe_ep_xchg_connect_local.argtypes = [vp, C.c_int]
        L.qe_ep_xchg_free.argtypes = [vp]
        L.qe_moe_ep_dispatch_p2p.argtypes = [vp, vp, C.c_int, vp, vp, vp, vp, vp]
        L.qe_moe_ep_route_p2p.argtypes = [vp, vp, C.c_int, vp, vp, vp]
        L.qe_ep_xchg_barrier.argtypes = [vp, vp]
        L.qe_moe_ep_experts_p2p.argtypes = [vp, vp, C.c_int, vp]
        L.qe_moe_ep_combine_p2p.argtypes = [vp, vp, C.c_int, vp, vp, vp, vp]
        L.qe_moe_graph_create.restype = vp
        L.qe_moe_graph_create.argtypes = [vp, C.c_int, vp, vp]
        L.qe_moe_graph_launch.argtypes = [vp, vp]
        L.qe_moe_graph_free.argtypes = [vp]
        L.qe_moe_open_safetensors.restype = vp
        L.qe_moe_open_safetensors.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(QeMoeConfig)]
        L.qe_safetensors_tensor_info.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.POINTER(C.c_int64),
                                                 C.POINTER(C.c_int)]
        _lib = L
    return _lib


def fptr(a: np.ndarray):
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data_as(C.POINTER(C.c_float))


def iptr(a: np.ndarray):
    if a.dtype != np.int32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous int32 array")
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def qmat_matvec(w: np.ndarray, scales: np.ndarray, biases: np.ndarray, rows: int, cols: int, bits: int, gs: int,
                x: np.ndarray, y: np.ndarray) -> int:
    """GPU qmat_matvec (engine/include/qmat.h:32): fills y, returns 0 or -1 (y untouched)."""
    return lib().qe_qmat_matvec(w.ctypes.data, scales.ctypes.data, biases.ctypes.data, rows, cols, bits, gs,
                                fptr(np.ascontiguousarray(x, np.float32)), fptr(y))


def route_logits(logits: np.ndarray, k: int):
    """GPU softmax + top-k + renormalisation on logits[T][E] -> (probs, idx, score)."""
    logits = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
    T, E = logits.shape
    probs = np.empty((T, E), np.float32)
    idx = np.empty((T, k), np.int32)
    score = np.empty((T, k), np.float32)
    if lib().qe_route_logits(T, E, k, fptr(logits), fptr(probs), iptr(idx), fptr(score)):
        raise ValueError("qe_route_logits failed")
    return probs, idx, score


def _op(name: str, *arrays: np.ndarray) -> np.ndarray:
    arrays = [np.ascontiguousarray(a, np.float32) for a in arrays]
    out = np.empty_like(arrays[0])
    if getattr(lib(), name)(fptr(out), *[fptr(a) for a in arrays], out.size):
        raise RuntimeError(f"{name} failed")
    return out


def op_silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    return _op("qe_op_silu_mul", gate, up)


def op_sigmoid(x: np.ndarray) -> np.ndarray:
    return _op("qe_op_sigmoid", x)


def op_expf(x: np.ndarray) -> np.ndarray:
    return _op("qe_op_expf", x)


def expert_gb_read() -> float:
    return lib().qe_expert_gb_read()


def expert_read_seconds() -> float:
    return lib().qe_expert_read_seconds()


STAGES = ("router", "topk", "bucket", "gateup", "down", "combine")


def profile_begin(device: int = 0) -> None:
    if lib().qe_profile_begin(device):
        raise RuntimeError("qe_profile_begin failed")


def profile_end(device: int = 0) -> tuple[dict, int]:
    """Summed GPU milliseconds per pipeline stage since profile_begin, and the number of passes."""
    ms = (C.c_double * len(STAGES))()
    passes = C.c_int(0)
    if lib().qe_profile_end(device, ms, C.byref(passes)):
        raise RuntimeError("qe_profile_end failed")
    return {name: ms[i] for i, name in enumerate(STAGES)}, passes.value


def kernel_launches() -> int:
    return lib().qe_kernel_launches()


def graph_captures() -> int:
    """Forwards the library has captured into CUDA graphs since the process started."""
    return lib().qe_graph_captures()


def device_count() -> int:
    return lib().qe_device_count()


def safetensors_tensor_info(directory: str, name: str):
    """(dtype, shape) of one tensor of a checkpoint directory, parsed by the library (no GPU needed)."""
    dt = C.create_string_buffer(8)
    shape = (C.c_int64 * 8)()
    nd = C.c_int(0)
    if lib().qe_safetensors_tensor_info(str(directory).encode(), name.encode(), dt, shape, C.byref(nd)):
        raise KeyError(name)
    return dt.value.decode(), tuple(shape[i] for i in range(nd.value))
