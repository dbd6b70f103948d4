"""GPU parity of the kernel-level entry points against the reference's fixtures and the CPU oracle.

Tolerances: qmat fixtures 1e-4 + 1e-4|y| (engine/tests/test_qmat.c:8-9), ops 1e-5 (test_ops.c:10),
softmax 1e-6 (test_ops.c:47); routing (softmax probabilities, top-k ids, renormalised scores) BIT-EXACT
against the oracle; silu_mul/sigmoid bit-exact too (same expf, same IEEE operation order).
"""
import numpy as np
import pytest

import oracle as O
import qmoe
from golden_io import qmat_fixtures, read_qmat_fixture, read_ops_fixture

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", qmat_fixtures(), ids=lambda p: p.name)
def test_qmat_fixture_gpu(path):
    rows, cols, bits, gs, w, s, b, x, y = read_qmat_fixture(path)
    got = np.full(rows, 42.0, np.float32)
    assert qmoe.qmat_matvec(w, s, b, rows, cols, bits, gs, x, got) == 0
    err = np.abs(got - y)
    assert (err <= 1e-4 + 1e-4 * np.abs(y)).all(), f"max abs err {err.max():.3e}"
    rc, want = O.qmat_matvec(w, s, b, rows, cols, bits, gs, x)
    scale = np.sqrt((want.astype(np.float64) ** 2).mean())
    assert np.abs(got - want).max() / scale < 1e-5, "GPU vs oracle differ beyond 1e-5 of the output RMS"


def test_qmat_validation_gpu():
    w = np.zeros(8, np.uint32); s = np.zeros(2, np.uint16); x = np.zeros(64, np.float32)
    for rows, cols, bits, gs in [(1, 64, 3, 64), (1, 64, 4, 48), (1, 100, 4, 64)]:
        y = np.full(1, 42.0, np.float32)
        assert qmoe.qmat_matvec(w, s, s, rows, cols, bits, gs, x, y) == -1 and y[0] == 42.0


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
@pytest.mark.parametrize("rows,cols", [(1, 128), (96, 384), (300, 1024), (2048, 512)])
def test_qmat_random_shapes_vs_oracle(bits, gs, rows, cols):
    if cols % gs:
        pytest.skip("cols must be a multiple of group_size")
    rng = np.random.default_rng(rows * 7 + cols + bits + gs)
    w = rng.integers(0, 2**32, rows * cols * bits // 32, dtype=np.uint64).astype(np.uint32)
    sc = np.array([np.float32(v).view(np.uint32) >> 16 for v in np.abs(rng.normal(0, 0.02, rows * cols // gs))],
                  np.uint16)
    bi = np.array([np.float32(v).view(np.uint32) >> 16 for v in rng.normal(0, 0.1, rows * cols // gs)], np.uint16)
    x = rng.normal(size=cols).astype(np.float32)
    got = np.empty(rows, np.float32)
    assert qmoe.qmat_matvec(w, sc, bi, rows, cols, bits, gs, x, got) == 0
    rc, want = O.qmat_matvec(w, sc, bi, rows, cols, bits, gs, x)
    scale = np.sqrt((want.astype(np.float64) ** 2).mean()) + 1e-30
    assert np.abs(got - want).max() / scale < 1e-5


def test_softmax_and_topk_fixtures_gpu():
    x, want = read_ops_fixture("softmax")
    probs, idx, score = qmoe.route_logits(x[None], 8)
    assert (np.abs(probs[0] - want) <= 1e-6 + 1e-6 * np.abs(want)).all()
    assert np.array_equal(probs[0], O.softmax(x)), "softmax not bit-exact with the reference op_softmax"
    x, k, want = read_ops_fixture("topk")
    _, idx, _ = qmoe.route_logits(x[None], int(k[0]))
    assert np.array_equal(idx[0], want.astype(np.int32))


def test_topk_known_answers_gpu():
    # engine/tests/test_ops.c:55-73 (ties keep the lower index; a tie with the k-th value stays out)
    _, idx, _ = qmoe.route_logits(np.array([[1, 5, 3, 5, 2, 5, 0, 4, -1, 3]], np.float32), 4)
    assert idx[0].tolist() == [1, 3, 5, 7]
    _, idx, _ = qmoe.route_logits(np.array([[5, 4, 4]], np.float32), 2)
    assert idx[0].tolist() == [0, 1]


def _oracle_route(logits: np.ndarray, k: int):
    T, E = logits.shape
    P = np.empty((T, E), np.float32); I = np.empty((T, k), np.int32); S = np.empty((T, k), np.float32)
    for t in range(T):
        P[t], I[t], S[t] = O.route_from_logits(logits[t], k)
    return P, I, S


@pytest.mark.parametrize("E,k", [(256, 8), (16, 4), (512, 16), (100, 1), (33, 7)])
def test_routing_bit_exact_random(E, k):
    rng = np.random.default_rng(E * 31 + k)
    T = 2048
    scales = rng.choice([0.01, 0.3, 1.0, 3.0, 20.0, 200.0], T)
    logits = (rng.normal(size=(T, E)) * scales[:, None]).astype(np.float32)
    # ties: duplicate values inside rows; coarse quantisation creates many equal probabilities
    logits[::7, : E // 2] = logits[::7, E // 2: 2 * (E // 2)]
    logits[1::11] = np.round(logits[1::11] * 2) / 2
    logits[2::13] = 0.0                               # all equal
    logits[3::17, 0] = -np.inf                        # -inf entries
    logits[4::19, :3] = np.float32(3e38)              # huge
    P, I, S = qmoe.route_logits(logits, k)
    Po, Io, So = _oracle_route(logits, k)
    assert np.array_equal(I, Io)
    assert np.array_equal(S.view(np.uint32), So.view(np.uint32))
    assert np.array_equal(P.view(np.uint32), Po.view(np.uint32))


def test_routing_with_nan_follows_the_reference_sequence():
    rng = np.random.default_rng(3)
    logits = rng.normal(size=(64, 256)).astype(np.float32)
    logits[0, 0] = np.nan        # NaN at index 0 propagates through max (ops.c:30-33)
    logits[1, 100] = np.nan      # NaN elsewhere is skipped by the max
    logits[2, :] = np.nan
    P, I, S = qmoe.route_logits(logits, 8)
    Po, Io, So = _oracle_route(logits, 8)
    assert np.array_equal(I, Io)
    # NaN payloads are not reproduced (x86 propagates the input payload, the GPU returns a canonical NaN):
    # NaN must appear in the same places, every other value bit for bit.
    for got, want in ((S, So), (P, Po)):
        assert np.array_equal(np.isnan(got), np.isnan(want))
        ok = ~np.isnan(want)
        assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


def test_silu_sigmoid_fixtures_gpu():
    g, u, want = read_ops_fixture("silu_mul")
    got = qmoe.op_silu_mul(g, u)
    assert (np.abs(got - want) <= 1e-5 + 1e-5 * np.abs(want)).all()
    ref = np.empty_like(g)
    O.lib().or_silu_mul(O.fptr(ref), O.fptr(g), O.fptr(u), g.size)
    assert np.array_equal(got, ref)
    x, want = read_ops_fixture("sigmoid")
    got = qmoe.op_sigmoid(x)
    assert (np.abs(got - want) <= 1e-5 + 1e-5 * np.abs(want)).all()
    ref = np.empty_like(x)
    O.lib().or_sigmoid(O.fptr(ref), O.fptr(x), x.size)
    assert np.array_equal(got, ref)


def test_device_expf_equals_host_expf_exhaustively():
    """Every negative float (the softmax domain: x - max <= 0) and every float in [0, 88.72]."""
    ranges = [(0x80000000, 0xFF800000 - 0x80000000 + 1), (0x00000000, 0x42B17218)]
    chunk = 1 << 26
    for lo, n in ranges:
        for start in range(0, n, chunk):
            m = min(chunk, n - start)
            bits = np.arange(lo + start, lo + start + m, dtype=np.uint64).astype(np.uint32)
            got = qmoe.op_expf(bits.view(np.float32))
            want = O.expf_bits(lo + start, m)
            bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
            assert bad.size == 0, f"{bad.size} mismatches, first x bits {int(bits[bad[0]]):#010x}"
