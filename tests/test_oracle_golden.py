"""CPU: pin the oracle (oracle/moe_oracle.c) before trusting it.

1. Against the reference's own committed fixtures and known-answer tests for this path
   (engine/tests/test_qmat.c, test_ops.c, test_qgroup.c: same tolerances).
2. Against the reference's C sources compiled here (oracle/_ref/libqref.so): bit-exact.
3. Against goldens produced by the reference's code (tests/golden/moe_*.npz, make_golden.py): bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from golden_io import qmat_fixtures, read_qmat_fixture, read_ops_fixture, moe_goldens, read_moe_golden

QMAT_REL, QMAT_ABS = 1e-4, 1e-4           # engine/tests/test_qmat.c:8-9
OPS_TOL = 1e-5                            # engine/tests/test_ops.c:10
SOFTMAX_TOL = 1e-6                        # engine/tests/test_ops.c:47


@pytest.mark.parametrize("path", qmat_fixtures(), ids=lambda p: p.name)
def test_qmat_fixture(path):
    rows, cols, bits, gs, w, s, b, x, y = read_qmat_fixture(path)
    rc, got = O.qmat_matvec(w, s, b, rows, cols, bits, gs, x)
    assert rc == 0
    err = np.abs(got - y)
    assert (err <= QMAT_ABS + QMAT_REL * np.abs(y)).all(), f"max abs err {err.max():.3e}"


def test_qmat_validation_and_bf16():
    # engine/tests/test_qmat.c:64-82: bad shapes rejected and y untouched; bf16 known answers
    w = np.zeros(8, np.uint32); s = np.zeros(2, np.uint16); b = np.zeros(2, np.uint16); x = np.zeros(64, np.float32)
    for rows, cols, bits, gs in [(1, 64, 3, 64), (1, 64, 4, 48), (1, 100, 4, 64)]:
        rc, y = O.qmat_matvec(w, s, b, rows, cols, bits, gs, x)
        assert rc == -1 and y[0] == 42.0
    assert O.lib().or_bf16_to_f32(0x3F80) == 1.0 and O.lib().or_bf16_to_f32(0xC000) == -2.0


def test_ops_fixtures():
    g, u, want = read_ops_fixture("silu_mul")
    out = np.empty_like(g)
    O.lib().or_silu_mul(O.fptr(out), O.fptr(g), O.fptr(u), g.size)
    assert (np.abs(out - want) <= OPS_TOL + OPS_TOL * np.abs(want)).all()
    x, want = read_ops_fixture("sigmoid")
    out = np.empty_like(x)
    O.lib().or_sigmoid(O.fptr(out), O.fptr(x), x.size)
    assert (np.abs(out - want) <= OPS_TOL + OPS_TOL * np.abs(want)).all()
    x, want = read_ops_fixture("softmax")
    out = O.softmax(x)
    assert (np.abs(out - want) <= SOFTMAX_TOL + SOFTMAX_TOL * np.abs(want)).all()
    x, k, want = read_ops_fixture("topk")
    assert np.array_equal(O.topk(x, int(k[0])), want.astype(np.int32))


def test_topk_known_answers():
    # engine/tests/test_ops.c:55-73
    x = np.array([1, 5, 3, 5, 2, 5, 0, 4, -1, 3], np.float32)
    idx = O.topk(x, 4, guard=1)
    assert idx.tolist() == [1, 3, 5, 7, -7]
    idx = O.topk(np.array([5, 4, 4], np.float32), 2, guard=1)
    assert idx.tolist() == [0, 1, -7]


def test_qgroup_random_and_edges():
    # engine/tests/test_qgroup.c: 1800 cases vs a double reference, tol 1e-5*(|want|+1)*n
    rng = np.random.default_rng(42)
    for trial in range(300):
        for n in (32, 64, 128):
            for bits in (4, 8):
                w = (np.zeros(32, np.uint32) if trial == 0 else np.full(32, 0xFFFFFFFF, np.uint32) if trial == 1
                     else rng.integers(0, 2**32, 32, dtype=np.uint64).astype(np.uint32))
                x = rng.uniform(-2, 2, 128).astype(np.float32)
                per, mask = 32 // bits, (1 << bits) - 1
                q = np.array([(int(w[j // per]) >> ((j % per) * bits)) & mask for j in range(n)], np.float64)
                want = float((q * x[:n].astype(np.float64)).sum())
                got = O.lib().or_qgroup_dot(w.ctypes.data, O.fptr(x), n, bits)
                assert abs(got - want) <= 1e-5 * (abs(want) + 1.0) * n


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
def test_oracle_bit_exact_with_reference_kernels():
    R, L = O.ref(), O.lib()
    rng = np.random.default_rng(5)
    for rows, cols, bits, gs in [(64, 256, 4, 64), (33, 384, 8, 32), (17, 512, 4, 128), (256, 2048, 8, 64)]:
        w = rng.integers(0, 2**32, rows * cols * bits // 32, dtype=np.uint64).astype(np.uint32)
        s = rng.integers(0x3800, 0x3c00, rows * cols // gs).astype(np.uint16)
        b = rng.integers(0xb800, 0xbc00, rows * cols // gs).astype(np.uint16)
        x = rng.normal(size=cols).astype(np.float32)
        m = O.qmat_struct(w, s, b, rows, cols, bits, gs)
        y1 = np.empty(rows, np.float32); y2 = np.empty(rows, np.float32)
        assert L.or_qmat_matvec(C.byref(m), O.fptr(x), O.fptr(y1)) == 0
        assert R.qmat_matvec(C.cast(C.pointer(m), C.c_void_p), O.fptr(x), O.fptr(y2)) == 0
        assert np.array_equal(y1, y2)
    for scale in (0.1, 1.0, 6.0, 40.0):
        x = (rng.normal(size=256) * scale + 40).astype(np.float32)
        a = np.empty_like(x); b_ = np.empty_like(x)
        L.or_softmax(O.fptr(a), O.fptr(x), 256); R.op_softmax(O.fptr(b_), O.fptr(x), 256)
        assert np.array_equal(a, b_)
        i1 = np.empty(8, np.int32); i2 = np.empty(8, np.int32)
        L.or_topk(O.iptr(i1), O.fptr(a), 256, 8); R.op_topk(O.iptr(i2), O.fptr(a), 256, 8)
        assert np.array_equal(i1, i2)
        g = (rng.normal(size=512) * scale).astype(np.float32); u = rng.normal(size=512).astype(np.float32)
        o1 = np.empty_like(g); o2 = np.empty_like(g)
        L.or_silu_mul(O.fptr(o1), O.fptr(g), O.fptr(u), 512); R.op_silu_mul(O.fptr(o2), O.fptr(g), O.fptr(u), 512)
        assert np.array_equal(o1, o2)


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("cfg", [dict(hidden=256, E=16, top_k=4, inter=64, sh_inter=64, bits=4),
                                 dict(hidden=384, E=40, top_k=8, inter=128, sh_inter=64, bits=8),
                                 dict(hidden=256, E=16, top_k=16, inter=64, sh_inter=64, bits=4, group_size=32)])
def test_oracle_block_bit_exact_with_reference_harness(cfg):
    blk = O.SynthBlock(O.BlockCfg(**cfg), seed=77)
    x = blk.x(9)
    o1, i1, s1 = blk.forward(x)
    o2, i2, s2 = blk.forward_ref(x)
    assert np.array_equal(i1, i2) and np.array_equal(s1, s2) and np.array_equal(o1, o2)


@pytest.mark.parametrize("path", moe_goldens(), ids=lambda p: p.stem)
def test_oracle_reproduces_reference_goldens(path):
    """The goldens were produced by the reference's own code; the oracle must reproduce them exactly."""
    g = read_moe_golden(path)
    blk = O.SynthBlock(O.BlockCfg(**g["cfg"]), g["seed"], 0, g["bias"])
    x = blk.x(g["T"])
    out, idx, score = blk.forward(x)
    assert np.array_equal(idx, g["idx"])
    if g["mode"] == "B":
        assert np.array_equal(score, g["score"])
    assert np.array_equal(out, g["out"])


def test_expf_bits_matches_python_reference_points():
    # expf(0) = 1, expf(-inf) = 0, expf(-104) underflows to 0; spot values within 1 ulp of double exp
    y = O.expf_bits(0x80000000, 1)  # -0.0
    assert y[0] == 1.0
    xs = np.array([-1.0, -0.5, -20.0, -87.0, -103.0], np.float32)
    for x in xs:
        u = int(x.view(np.uint32))
        got = O.expf_bits(u, 1)[0]
        want = np.float32(np.exp(np.float64(x)))
        assert abs(int(got.view(np.int32)) - int(want.view(np.int32))) <= 1
