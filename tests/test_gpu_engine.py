"""GPU: the whole-model ABI (include/qe_engine.h) against the reference's own engine on the same checkpoint.

A tiny synthetic qwen3_5_moe checkpoint (tests/model_synth.py: Gated DeltaNet and full-attention layers, routed
MoE blocks with an 8-bit quantized router) is run token by token through the reference's unmodified qe_load /
qe_forward (engine/src/qengine.c, compiled from its sources into oracle/_ref/libqengine_ref.so, in a child
process) and through libqengine_b200's (trunk on the GPU by default, or on the host with QE_TRUNK=host; MoE
blocks on the GPU), both bound with the reference front end's
ctypes declarations (engine/cli/qchat.py:39-48). The logits must agree within fp32 reordering at every
position, with the same arg-max token; the position, reset and context-full (-2) conventions must match.
"""
import ctypes as C
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import qmoe
from model_synth import TinyModel, write_tiny_model
from test_engine_cpu import _qchat_bind

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
REF_LIB = REPO / "oracle" / "_ref" / "libqengine_ref.so"
TOKENS = [5, 17, 200, 3, 3, 99, 250, 1, 64, 17]

CHILD = r"""
import ctypes as C, json, sys
import numpy as np
a = json.loads(sys.argv[2])
lib = C.CDLL(a["lib"])          # bound as engine/cli/qchat.py:39-48 binds it
lib.qe_load.restype = C.c_void_p
lib.qe_load.argtypes = [C.c_char_p, C.c_int]
lib.qe_forward.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_float)]
lib.qe_vocab.argtypes = [C.c_void_p]
h = lib.qe_load(a["dir"].encode(), a["max_len"])
assert h, "reference qe_load failed"
V = lib.qe_vocab(h)
out = np.zeros((len(a["tokens"]), V), np.float32)
lg = np.zeros(V, np.float32)
for i, t in enumerate(a["tokens"]):
    assert lib.qe_forward(h, t, lg.ctypes.data_as(C.POINTER(C.c_float))) == 0
    out[i] = lg
np.save(a["out"], out)
"""


def _reference_logits(d: Path, tokens, max_len, tmp_path) -> np.ndarray:
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libqengine_ref.so was not built (no reference sources when the oracle was made)")
    out = tmp_path / "ref_logits.npy"
    args = {"lib": str(REF_LIB), "dir": str(d), "max_len": max_len, "tokens": tokens, "out": str(out)}
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO / "tests"), json.dumps(args)], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return np.load(out)


def _ours(lib, h, tokens, V):
    lg = np.zeros(V, np.float32)
    out = np.zeros((len(tokens), V), np.float32)
    for i, t in enumerate(tokens):
        assert lib.qe_forward(h, t, lg.ctypes.data_as(C.POINTER(C.c_float))) == 0
        out[i] = lg
    return out


@pytest.mark.parametrize("trunk", ["gpu", "host"])
@pytest.mark.parametrize("bits,interval", [(4, 4), (8, 2)])
def test_engine_matches_reference_engine(tmp_path, monkeypatch, bits, interval, trunk):
    monkeypatch.setenv("QE_TRUNK", trunk)                     # read by qe_load
    m = TinyModel(bits=bits, full_attention_interval=interval)
    d = tmp_path / "model"
    write_tiny_model(d, m, seed=bits)
    max_len = 16
    want = _reference_logits(d, TOKENS, max_len, tmp_path)
    lib = _qchat_bind(qmoe.LIB_PATH)
    h = lib.qe_load(str(d).encode(), max_len)
    assert h
    try:
        V = lib.qe_vocab(h)
        assert V == m.vocab and lib.qe_max_len(h) == max_len and lib.qe_position(h) == 0
        got = _ours(lib, h, TOKENS, V)
        assert lib.qe_position(h) == len(TOKENS)
        for i in range(len(TOKENS)):
            rel = np.linalg.norm(got[i] - want[i]) / np.linalg.norm(want[i])
            assert rel <= 2e-5, (i, rel)
            assert int(got[i].argmax()) == int(want[i].argmax()), i
        # reset: the same sequence gives the same logits again (states and KV caches cleared)
        lib.qe_reset(h)
        assert lib.qe_position(h) == 0
        again = _ours(lib, h, TOKENS[:3], V)
        assert np.array_equal(again, got[:3])
        assert lib.qe_expert_gb_read() > 0
    finally:
        lib.qe_free(h)


def test_engine_context_full_and_bad_token(tmp_path):
    d = tmp_path / "model"
    m = write_tiny_model(d, TinyModel(), seed=7)
    lib = _qchat_bind(qmoe.LIB_PATH)
    h = lib.qe_load(str(d).encode(), 3)
    assert h
    try:
        lg = np.zeros(m.vocab, np.float32)
        p = lg.ctypes.data_as(C.POINTER(C.c_float))
        assert lib.qe_forward(h, m.vocab, p) == -1          # token id outside the vocabulary
        assert lib.qe_position(h) == 0
        for t in (1, 2, 3):
            assert lib.qe_forward(h, t, p) == 0
        assert lib.qe_forward(h, 4, p) == -2                 # context full (qengine.h:13)
        assert lib.qe_position(h) == 3
        lib.qe_reset(h)
        assert lib.qe_forward(h, 4, p) == 0
    finally:
        lib.qe_free(h)


def test_engine_trace_records_every_layer(tmp_path):
    """QE_TRACE through the whole-model API (moe_layer.c:57-64: int32 layer id, then the top-k expert ids, per token and
    layer): the GPU trunk's steps write one record per MoE block and token, layers in order, ids valid and distinct."""
    d = tmp_path / "model"
    m = write_tiny_model(d, TinyModel(), seed=11)
    trace = tmp_path / "trace.bin"
    code = r"""
import ctypes as C, os, sys
import numpy as np
sys.path[:0] = sys.argv[3:]
import qmoe
from test_engine_cpu import _qchat_bind
lib = _qchat_bind(qmoe.LIB_PATH)
h = lib.qe_load(sys.argv[1].encode(), 8)
assert h
lg = np.zeros(int(sys.argv[2]), np.float32)
for t in (3, 9, 27, 81):
    assert lib.qe_forward(h, t, lg.ctypes.data_as(C.POINTER(C.c_float))) == 0
lib.qe_free(h)
"""
    env = dict(__import__("os").environ, QE_TRACE=str(trace), QE_TRUNK="gpu")
    r = subprocess.run([sys.executable, "-c", code, str(d), str(m.vocab), str(REPO / "tests"),
                        str(REPO / "moe-stream-mac_b200"), str(REPO)], capture_output=True, text=True, env=env,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    rec = np.fromfile(trace, np.int32).reshape(-1, 1 + m.top_k)
    assert rec.shape[0] == 4 * m.n_layers
    assert np.array_equal(rec[:, 0], np.tile(np.arange(m.n_layers), 4))
    ids = rec[:, 1:]
    assert ids.min() >= 0 and ids.max() < m.E
    assert all(len(set(row)) == m.top_k for row in ids.tolist())
