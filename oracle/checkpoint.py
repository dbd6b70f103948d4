"""Checkpoint writer for the CPU checker (TEST INFRASTRUCTURE ONLY): one layer's MoE block in the MLX
safetensors layout the reference engine reads (engine/src/io/k3_st.c, tensor names of engine/src/model.c:52-64).
Used by the tests (Mode R goldens, the loader tests) and by bench.py's CPU baseline (Mode R timing)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np


def write_safetensors(path: Path, tensors: dict) -> None:
    """Minimal safetensors writer: 8-byte LE header length, JSON header, contiguous data.
    tensors: name -> (dtype string, array)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with Path(path).open("wb") as f:
        f.write(len(hb).to_bytes(8, "little"))
        f.write(hb)
        for b in blobs:
            f.write(b)


def checkpoint_tensors(prefix: str, arrays: dict) -> dict:
    """MLX checkpoint names for one layer's MoE block (engine/src/model.c:52-64)."""
    t = {}
    for key, name in (("gate", "switch_mlp.gate_proj"), ("up", "switch_mlp.up_proj"), ("down", "switch_mlp.down_proj"),
                      ("sh_gate", "shared_expert.gate_proj"), ("sh_up", "shared_expert.up_proj"),
                      ("sh_down", "shared_expert.down_proj"), ("router_q", "gate"),
                      ("sh_router_q", "shared_expert_gate")):
        w, s, b = arrays[key]
        if key == "sh_router_q":
            w, s, b = w.reshape(1, -1), s.reshape(1, -1), b.reshape(1, -1)
        t[f"{prefix}.{name}.weight"] = ("U32", w)
        t[f"{prefix}.{name}.scales"] = ("BF16", s)
        t[f"{prefix}.{name}.biases"] = ("BF16", b)
    return t
