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

CFG = oracle.BlockCfg(hidden=256, E=16, top_k=4, inter=128, sh_inter=128, bits=4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, T: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qmoe.ep import ExpertParallelMoe
        blk = oracle.SynthBlock(CFG, seed=11)
        # sharded: each rank its own tokens; replicated: the same tokens everywhere
        x = blk.x(T, seed=200 + (rank if mode == "sharded" else 0))
        ep = ExpertParallelMoe(OracleEngine(blk, rank, world), rank, world, device="cpu")
        out = ep.forward(torch.from_numpy(x), mode=mode).numpy()
        want, _, _ = blk.forward(x)
        rel = np.linalg.norm(out - want, axis=1) / np.linalg.norm(want, axis=1)
        counts = None if ep.last_counts is None else ep.last_counts.tolist()
        q.put((rank, float(rel.max()), float(np.abs(out - want).max()), counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,T", [("sharded", 7), ("sharded", 1), ("replicated", 5)])
def test_ep_two_ranks(mode, T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, T, q)) for r in range(2)]
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
