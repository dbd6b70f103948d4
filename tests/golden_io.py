"""Readers for tests/golden: the reference's fixtures and the reference-generated MoE goldens."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
REF_FIX = GOLDEN / "ref_fixtures"


def qmat_fixtures() -> list[Path]:
    return sorted(REF_FIX.glob("qmat_*.bin"))


def read_qmat_fixture(path: Path):
    """tools/gen_qmat_fixture.py:3-4: int32 rows, cols, bits, gs | u32 w | u16 scales | u16 biases |
    f32 x[cols] | f32 y[rows]."""
    raw = path.read_bytes()
    rows, cols, bits, gs = np.frombuffer(raw, "<i4", 4)
    o = 16
    nw, ng = rows * cols * bits // 32, rows * (cols // gs)
    w = np.frombuffer(raw, "<u4", nw, o).copy(); o += 4 * nw
    s = np.frombuffer(raw, "<u2", ng, o).copy(); o += 2 * ng
    b = np.frombuffer(raw, "<u2", ng, o).copy(); o += 2 * ng
    x = np.frombuffer(raw, "<f4", cols, o).copy(); o += 4 * cols
    y = np.frombuffer(raw, "<f4", rows, o).copy(); o += 4 * rows
    assert o == len(raw)
    return int(rows), int(cols), int(bits), int(gs), w, s, b, x, y


def read_ops_fixture(name: str) -> list[np.ndarray]:
    """tools/gen_ops_fixture.py:3: int32 n_arrays; per array int32 len, f32[len]."""
    raw = (REF_FIX / f"ops_{name}.bin").read_bytes()
    n = int(np.frombuffer(raw, "<i4", 1)[0])
    o, out = 4, []
    for _ in range(n):
        ln = int(np.frombuffer(raw, "<i4", 1, o)[0]); o += 4
        out.append(np.frombuffer(raw, "<f4", ln, o).copy()); o += 4 * ln
    return out


def moe_goldens() -> list[Path]:
    return sorted(GOLDEN.glob("moe_*.npz"))


def read_moe_golden(path: Path) -> dict:
    z = np.load(path)
    d = {k: z[k] for k in z.files}
    d["cfg"] = json.loads(str(d["cfg"]))
    d["seed"] = int(d["seed"]); d["T"] = int(d["T"]); d["mode"] = str(d["mode"])
    d["bias"] = None if d["bias"].size == 0 else d["bias"]
    d["name"] = path.stem
    return d


def rel_l2(got: np.ndarray, want: np.ndarray) -> np.ndarray:
    """Per-row relative L2 error (engine/tests/test_moe_layer.c:45-50)."""
    got = np.asarray(got, np.float64); want = np.asarray(want, np.float64)
    num = ((got - want) ** 2).sum(-1)
    den = (want ** 2).sum(-1) + 1e-30
    return np.sqrt(num / den)


from oracle.checkpoint import write_safetensors, checkpoint_tensors  # noqa: E402,F401
