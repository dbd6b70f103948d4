"""Expert-parallel exchange on CPU ranks (gloo, world_size 2): qmoe.ep.ExpertParallelMoe with the oracle engine.

Checks the host logic that the GPU run shares: packing per destination rank, the equal-block all_to_all with
padding rows, the return exchange, and the rank-order combine; both step shapes (token-sharded, replicated)
against the oracle's single-process block (moe_layer.c:66-89)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from ep_cpu import OracleEngine
from qmoe.placement import Placement, histogram
from qmoe.synth import zipf_router_bias

CFG = oracle.BlockCfg(hidden=256, E=16, top_k=4, inter=128, sh_inter=128, bits=4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, T: int, q, slots: int = 0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qmoe.ep import ExpertParallelMoe
        placement = None
        if slots:
            # skewed routing and a placement planned from a calibration batch's histogram (same on every rank)
            blk = oracle.SynthBlock(CFG, seed=11, router_bias=zipf_router_bias(CFG.E, 1.1, seed=3))
            placement = Placement.from_load(histogram(blk.forward(blk.x(64, seed=99))[1], CFG.E), world, slots)
        else:
            blk = oracle.SynthBlock(CFG, seed=11)
        # sharded: each rank its own tokens; replicated: the same tokens everywhere
        x = blk.x(T, seed=200 + (rank if mode == "sharded" else 0))
        ep = ExpertParallelMoe(OracleEngine(blk, rank, world, placement), rank, world, device="cpu")
        out = ep.forward(torch.from_numpy(x), mode=mode).numpy()
        want, _, _ = blk.forward(x)
        rel = np.linalg.norm(out - want, axis=1) / np.linalg.norm(want, axis=1)
        counts = None if ep.last_counts is None else ep.last_counts.tolist()
        q.put((rank, float(rel.max()), float(np.abs(out - want).max()), counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,T,slots", [("sharded", 7, 0), ("sharded", 1, 0), ("replicated", 5, 0),
                                          ("sharded", 7, 10), ("replicated", 5, 10)])
def test_ep_two_ranks(mode, T, slots):
    """slots > 0: a planned placement with replicated hot experts (10 slots per rank for E = 16)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, T, q, slots)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes
    res = [q.get(timeout=10) for _ in procs]
    for rank, rel, mx, counts in res:
        # the only difference from the single-process block is the fp32 grouping of the sum by rank
        assert rel <= 1e-6, (rank, rel)
        assert mx <= 1e-5, (rank, mx)
        if mode == "sharded":
            assert len(counts) == 2 and all(0 <= c <= T for c in counts)


def test_placement_balances_skewed_routing():
    """The planner on C4-style Zipf(1.1) routing over 8 ranks: hot experts replicated into one spare slot per
    rank cut the busiest rank's assignments against the contiguous ranges, and every assignment still lands on
    a rank that holds its expert."""
    cfg = oracle.BlockCfg(hidden=256, E=64, top_k=8, inter=128, sh_inter=128, bits=4)
    blk = oracle.SynthBlock(cfg, seed=21, router_bias=zipf_router_bias(cfg.E, 1.1, seed=4))
    G = 8
    calib = blk.forward(blk.x(256, seed=1))[1]
    steps = [blk.forward(blk.x(64, seed=10 + s))[1] for s in range(G)]   # one batch per source rank
    plain = Placement.contiguous(cfg.E, G)
    placed = Placement.from_load(histogram(calib, cfg.E), G, slots=cfg.E // G + 1)
    a, b = plain.rank_loads(steps), placed.rank_loads(steps)
    assert a.sum() == b.sum() == sum(s.size for s in steps)
    assert b.max() / b.mean() < 0.6 * a.max() / a.mean(), (a, b)
    for s, idx in enumerate(steps):
        d = placed.dest(idx, s)
        for t in range(idx.shape[0]):
            for j in range(cfg.top_k):
                assert idx[t, j] in placed.table[d[t, j]]


def test_placement_tables():
    p = Placement(np.array([[0, 1, 2, -1], [2, 3, 1, -1]], np.int32), 4)
    assert p.nrep.tolist() == [1, 2, 2, 1]
    assert p.reps[1, :2].tolist() == [0, 1] and p.reps[0, 0] == 0
    idx = np.array([[1, 2], [1, 3], [0, -1]])
    # replica (t + src) % nrep
    assert p.dest(idx, 0).tolist() == [[0, 0], [1, 1], [0, -1]]
    assert p.dest(idx, 1).tolist() == [[1, 1], [0, 1], [0, -1]]
    for bad in ([[0, 0], [1, 2]], [[0, 1], [1, -1]], [[0, 1], [-1, -1]], [[0, 5], [1, 2]]):
        with pytest.raises(ValueError):
            Placement(np.array(bad, np.int32), 4 if bad != [[0, 1], [1, -1]] else 3)
