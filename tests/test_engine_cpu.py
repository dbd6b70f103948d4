"""CPU: the whole-model ABI (include/qe_engine.h) -- its host trunk ops against the reference's own fixtures
(engine/tests/test_ops.c, test_gdn.c: MLX ground truth, tolerance 2e-5 absolute + relative), the binding with
the reference front end's exact ctypes declarations (engine/cli/qchat.py:37-48), and config.json strictness
(engine/src/config.c:46-81). Loading a model needs a GPU for its MoE blocks; that path is tests/test_gpu_engine.py.
"""
import ctypes as C
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import qmoe

FIX = Path(__file__).resolve().parent / "golden" / "ref_fixtures"
REPO = Path(__file__).resolve().parents[1]
fp = C.POINTER(C.c_float)


def _fixture(name):
    """int32 n, then n x (int32 len, float32[len]) (the reference's fixture layout)."""
    raw = (FIX / name).read_bytes()
    n = int(np.frombuffer(raw[:4], np.int32)[0])
    out, o = [], 4
    for _ in range(n):
        ln = int(np.frombuffer(raw[o:o + 4], np.int32)[0])
        out.append(np.frombuffer(raw[o + 4:o + 4 + 4 * ln], np.float32).copy())
        o += 4 + 4 * ln
    return out


def _close(got, want, tol=2e-5):
    err = np.abs(got - want)
    assert np.all(err <= tol + tol * np.abs(want)), float(err.max())


def _p(a):
    return a.ctypes.data_as(fp)


@pytest.fixture(scope="module")
def L():
    lib = C.CDLL(str(qmoe.LIB_PATH))
    lib.qe_trunk_rmsnorm.argtypes = [fp, fp, fp, C.c_int, C.c_float]
    lib.qe_trunk_rope.argtypes = [fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
    lib.qe_trunk_conv_step.argtypes = [fp, fp, fp, fp, C.c_int, C.c_int]
    lib.qe_trunk_l2norm.argtypes = [fp, C.c_int, C.c_float, C.c_float]
    lib.qe_trunk_gates.argtypes = [fp, fp, fp, fp, fp, fp, C.c_int]
    lib.qe_trunk_recurrent_step.argtypes = [fp, fp, fp, fp, fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int]
    return lib


def test_rmsnorm_fixture(L):
    x, w, want = _fixture("ops_rmsnorm.bin")
    out = np.empty_like(x)
    L.qe_trunk_rmsnorm(_p(out), _p(x), _p(w), x.size, 1e-6)
    _close(out, want)


@pytest.mark.parametrize("name", ["ops_rope_p0.bin", "ops_rope_p7.bin", "ops_rope_p3001.bin"])
def test_rope_fixture(L, name):
    p, x, want = _fixture(name)
    v = x.copy()
    L.qe_trunk_rope(_p(v), int(p[0]), int(p[1]), int(p[2]), int(p[3]), float(p[4]))
    _close(v, want)


def test_conv_fixture(L):
    a = _fixture("gdn_conv.bin")
    Cc, K, T = int(a[0][0]), int(a[0][1]), int(a[0][2])
    state = np.zeros((K - 1) * Cc, np.float32)
    out = np.empty(Cc, np.float32)
    for t in range(T):
        x = np.ascontiguousarray(a[2][t * Cc:(t + 1) * Cc])
        L.qe_trunk_conv_step(_p(out), _p(state), _p(x), _p(a[1]), Cc, K)
        _close(out, a[3][t * Cc:(t + 1) * Cc])


def test_l2norm_and_gates_fixtures(L):
    a = _fixture("gdn_l2norm.bin")
    H, Dk = int(a[0][0]), int(a[0][1])
    for src, want, scale in ((a[1], a[2], 1.0 / np.sqrt(np.float32(Dk))), (a[3], a[4], 1.0)):
        v = src.copy()
        for h in range(H):
            seg = v[h * Dk:(h + 1) * Dk]
            L.qe_trunk_l2norm(_p(seg), Dk, 1e-6, float(scale))
        _close(v, want)
    g = _fixture("gdn_gates.bin")
    Hv = int(g[0][0])
    gg, beta = np.empty(Hv, np.float32), np.empty(Hv, np.float32)
    L.qe_trunk_gates(_p(gg), _p(beta), _p(g[1]), _p(g[2]), _p(g[3]), _p(g[4]), Hv)
    _close(gg, g[5])
    _close(beta, g[6])


def test_recurrence_fixture(L):
    a = _fixture("gdn_recurrence.bin")
    Hk, Hv, Dk, Dv, T = (int(v) for v in a[0][:5])
    state = np.zeros(Hv * Dv * Dk, np.float32)
    y = np.empty(Hv * Dv, np.float32)
    for t in range(T):
        q, k, v, g, beta, want = a[1 + 6 * t:7 + 6 * t]
        L.qe_trunk_recurrent_step(_p(y), _p(state), _p(q), _p(k), _p(v), _p(g), _p(beta), Hk, Hv, Dk, Dv)
        _close(y, want)
    _close(state, a[1 + 6 * T])


def _qchat_bind(path):
    """The reference front end's declarations, verbatim in effect (engine/cli/qchat.py:39-48)."""
    lib = C.CDLL(str(path))
    lib.qe_load.restype = C.c_void_p
    lib.qe_load.argtypes = [C.c_char_p, C.c_int]
    for name in ("qe_reset", "qe_free"):
        getattr(lib, name).argtypes = [C.c_void_p]
    lib.qe_forward.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_float)]
    for name in ("qe_vocab", "qe_position", "qe_max_len"):
        getattr(lib, name).argtypes = [C.c_void_p]
    lib.qe_set_threads.argtypes = [C.c_int]
    for name in ("qe_expert_gb_read", "qe_expert_read_seconds", "qe_peak_rss_gb"):
        getattr(lib, name).restype = C.c_double
    return lib


def test_engine_binds_as_the_reference_front_end(tmp_path):
    lib = _qchat_bind(qmoe.LIB_PATH)
    assert not lib.qe_load(str(tmp_path / "missing").encode(), 16)   # no config.json
    assert not lib.qe_load(str(tmp_path).encode(), 0)                 # max_len < 1
    assert lib.qe_set_threads(0) >= 1
    assert lib.qe_peak_rss_gb() > 0


CHILD = r"""
import ctypes as C, sys
lib = C.CDLL(sys.argv[1]); lib.qe_load.restype = C.c_void_p; lib.qe_load.argtypes = [C.c_char_p, C.c_int]
sys.exit(0 if not lib.qe_load(sys.argv[2].encode(), 8) else 3)
"""


@pytest.mark.parametrize("edit,message", [
    (lambda c: c["text_config"].pop("head_dim"), 'missing or non-numeric "head_dim"'),
    (lambda c: c["text_config"].update(model_type="llama"), "model_type must be qwen3_5_moe"),
    (lambda c: c.pop("quantization"), 'no "quantization"'),
    (lambda c: c["quantization"].update(mode="mxfp4"), "only affine quantization"),
    (lambda c: c["text_config"]["rope_parameters"].update(rope_type="yarn"), 'only rope_type "default"'),
    (lambda c: c["text_config"].update(norm_topk_prob=False), "norm_topk_prob=false"),
])
def test_config_is_read_strictly(tmp_path, edit, message):
    from model_synth import TinyModel
    cfg = TinyModel().config()
    edit(cfg)
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    r = subprocess.run([sys.executable, "-c", CHILD, str(qmoe.LIB_PATH), str(tmp_path)], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert message in r.stderr, r.stderr


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_load_without_gpu_fails_at_the_moe_blocks(tmp_path):
    from model_synth import write_tiny_model
    write_tiny_model(tmp_path, seed=1)
    r = subprocess.run([sys.executable, "-c", CHILD, str(qmoe.LIB_PATH), str(tmp_path)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "MoE block not loaded" in r.stderr
