"""CPU: the C-ABI library loads, exports every function include/*.h declares, and refuses to run without a
GPU (no CPU fallback). Also the host-side configuration logic."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import qmoe
from qmoe.synth import CONFIGS, zipf_router_bias

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def declared_functions() -> list[str]:
    names = []
    for h in sorted(INCLUDE.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(qe_\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_the_block_api():
    names = declared_functions()
    for required in ("qe_moe_create", "qe_moe_forward", "qe_moe_forward_device", "qe_moe_route", "qe_moe_free",
                     "qe_qmat_matvec", "qe_route_logits"):
        assert required in names


def test_library_exports_every_declared_symbol():
    L = C.CDLL(str(qmoe.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_gpu():
    L = qmoe.lib()
    cfg = qmoe.QeMoeConfig(256, 16, 4, 64, 64, 4, 64, qmoe.QE_ROUTER_F32, 8, 64, 0, 0)
    assert not L.qe_moe_create_synthetic(C.byref(cfg), 1, 0, None)
    x = np.zeros(64, np.float32); y = np.full(4, 42.0, np.float32)
    w = np.zeros(32, np.uint32); s = np.zeros(4, np.uint16)
    assert qmoe.qmat_matvec(w, s, s, 4, 64, 4, 64, x, y) == -1 and (y == 42.0).all()


def test_qmat_validation_rejects_before_touching_the_gpu():
    # engine/src/qmat.c:16-22 checks, evaluated on the host: no device needed to refuse
    x = np.zeros(128, np.float32); y = np.full(1, 42.0, np.float32)
    w = np.zeros(64, np.uint32); s = np.zeros(4, np.uint16)
    for rows, cols, bits, gs in [(1, 64, 3, 64), (1, 64, 4, 48), (1, 100, 4, 64), (0, 64, 4, 64)]:
        assert qmoe.qmat_matvec(w, s, s, rows, cols, bits, gs, x, y) == -1
        assert y[0] == 42.0


def test_config_byte_and_flop_counts():
    c1 = CONFIGS["c1"]
    assert c1.expert_bytes == 1_769_472
    assert c1.decode_bytes_per_token() == 18_046_976
    assert c1.flops_per_token() == 57_675_776
    c3 = CONFIGS["c3_decode"]
    assert c3.expert_bytes == 10_027_008
    assert c3.decode_bytes_per_token() == 93_425_664
    assert c3.flops_per_token() == 171_448_320


def test_zipf_bias_is_a_seeded_permutation_of_a_zipf_law():
    b = zipf_router_bias(256, 1.1, seed=3)
    assert b.dtype == np.float32 and b.shape == (256,)
    assert b.max() == 0.0 and np.isclose(b.min(), -0.75 * 1.1 * np.log(256), rtol=1e-6)
    assert np.array_equal(b, zipf_router_bias(256, 1.1, seed=3))
    assert not np.array_equal(b, zipf_router_bias(256, 1.1, seed=4))


def test_engine_thread_and_rss_calls_bind_as_qchat_does():
    """qe_set_threads / qe_peak_rss_gb / the read statistics, bound with the argtypes and restypes of the
    reference's terminal chat (engine/cli/qchat.py:46-48) on a fresh CDLL handle; no GPU needed."""
    L = C.CDLL(str(qmoe.LIB_PATH))
    L.qe_set_threads.argtypes = [C.c_int]
    for name in ("qe_expert_gb_read", "qe_expert_read_seconds", "qe_peak_rss_gb"):
        getattr(L, name).restype = C.c_double
    default = L.qe_set_threads(0)          # n <= 0: keep, report the effective count
    assert default >= 1
    assert L.qe_set_threads(3) == 3
    assert L.qe_set_threads(-1) == 3
    assert L.qe_set_threads(default) == default
    import resource
    rss = L.qe_peak_rss_gb()
    want = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 2**20   # KiB -> GiB (Linux)
    assert 0 < rss and abs(rss - want) <= 0.05 * want + 1e-3
    assert L.qe_expert_gb_read() >= 0 and L.qe_expert_read_seconds() >= 0
