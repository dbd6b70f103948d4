"""GPU: qe_route_f32_noalloc, the routing entry point that allocates no device memory.

Callers whose device memory is owned by another allocator, or whose decode loop cannot take the
synchronisation of a cudaMalloc, use it instead of qe_moe_route; its only scratch (the logits) is a fixed
4 MiB device array inside the library. Here it must return exactly the routing of the existing entry point
qe_moe_route (bit for bit, the tolerance every routing test uses) on two calls in a row that reuse that
array, and refuse a batch too large for it.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import qmoe
from qmoe.synth import zipf_router_bias

pytestmark = pytest.mark.gpu

CFG = dict(hidden=2048, E=256, top_k=8, inter=512, sh_inter=512, bits=4)


def _noalloc_route(router_rows: torch.Tensor, bias, x: np.ndarray, k: int):
    T, H = x.shape
    E = router_rows.shape[0] - 1
    dx = torch.from_numpy(x).cuda()
    idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    score = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    rc = qmoe.lib().qe_route_f32_noalloc(C.c_void_p(router_rows.data_ptr()),
                                         C.c_void_p(bias.data_ptr() if bias is not None else None),
                                         C.c_void_p(dx.data_ptr()), T, H, E, k, C.c_void_p(idx.data_ptr()),
                                         C.c_void_p(score.data_ptr()), C.c_void_p(stream.cuda_stream))
    stream.synchronize()
    return rc, idx.cpu().numpy(), score.cpu().numpy()


def test_noalloc_routing_matches_qe_moe_route_on_two_calls_in_a_row():
    bias = zipf_router_bias(CFG["E"], 1.1, seed=31)
    checker = O.SynthBlock(O.BlockCfg(**CFG), 31, 0, bias)
    a = checker.arrays()
    rows = torch.from_numpy(np.concatenate([a["router_f32"], a["sh_gate_f32"][None]], 0)).cuda()
    dbias = torch.from_numpy(bias).cuda()
    block = qmoe.MoeBlock(**CFG, seed=31, router_bias=bias)
    for call, T in enumerate((300, 9)):
        x = checker.x(T, seed=500 + call)
        want_idx, want_score = block.route(x)
        rc, idx, score = _noalloc_route(rows, dbias, x, CFG["top_k"])
        assert rc == 0
        assert np.array_equal(idx, want_idx), f"call {call}: routing indices differ"
        assert np.array_equal(score.view(np.uint32), want_score.view(np.uint32)), f"call {call}: weights differ"
    block.close()


def test_noalloc_refuses_a_batch_beyond_its_fixed_scratch():
    rows = torch.zeros((257, 64), dtype=torch.float32, device="cuda")
    x = np.zeros((4081, 64), np.float32)                 # 4081 * 257 > 2^20 logits
    rc, idx, score = _noalloc_route(rows, None, x, 8)
    assert rc == -1
    assert (idx == -1).all() and (score == 0).all()
