"""qmoe: Python host side of libqengine_b200, the B200 routed-MoE block.

The reference drives its C engine from Python through ctypes (engine/cli/qchat.py:34-76, class Engine:
argtypes/restype set once, opaque handle, numpy buffers passed by pointer, return codes checked). This
package does the same for include/qe_moe.h. The library is the product path: there is no CPU fallback,
and loading fails loudly if libqengine_b200.so is missing.
"""
from .lib import (QeMoeConfig, QeMoeWeights, QeQTensor, QE_ROUTER_F32, QE_ROUTER_QMAT, QE_EP_ROUTED, LIB_PATH, build, lib,
                  qmat_matvec, route_logits, op_silu_mul, op_sigmoid, op_expf, expert_gb_read,
                  expert_read_seconds, device_count, profile_begin, profile_end, kernel_launches, graph_captures,
                  STAGES, safetensors_tensor_info)
from .block import MoeBlock, EngineError
from .synth import CONFIGS, MoeConfig, zipf_router_bias
from .placement import Placement, histogram, histogram_from_trace, read_trace
from .engine import Engine, ContextFull

__all__ = ["QeMoeConfig", "QeMoeWeights", "QeQTensor", "QE_ROUTER_F32", "QE_ROUTER_QMAT", "LIB_PATH", "build", "lib",
           "qmat_matvec", "route_logits", "op_silu_mul", "op_sigmoid", "op_expf", "expert_gb_read",
           "expert_read_seconds", "device_count", "profile_begin", "profile_end",
           "kernel_launches", "graph_captures", "STAGES", "MoeBlock", "EngineError", "CONFIGS", "MoeConfig",
           "zipf_router_bias", "safetensors_tensor_info", "QE_EP_ROUTED", "Placement", "histogram",
           "histogram_from_trace", "read_trace", "Engine", "ContextFull"]
