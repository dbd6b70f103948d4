"""Expert parallelism on the GPU: the qe_moe_ep_* entry points of include/qe_moe.h.

On one GPU the ranks are emulated: G handles, each holding E/G experts, run the token-sharded step with the
all_to_all done by tensor slicing (every launch completes before the next; nothing waits on another rank).
Results are compared with the single-handle forward (routing bit-identical; outputs within the fp32 regrouping
of the sum by rank) and with the oracle. With two or more GPUs, the same step runs over NCCL in one process per
GPU (qmoe.ep.ExpertParallelMoe)."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
import qmoe

pytestmark = pytest.mark.gpu

CFG = qmoe.MoeConfig("ep_small", hidden=512, inter=256, sh_inter=256, bits=4, tokens=64, E=32, top_k=4)


def _blocks(cfg, G, seed=5, router_bias=None, placement=None):
    return [qmoe.MoeBlock(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, seed=seed,
                          router_bias=router_bias, ep_rank=r, ep_size=G, placement=placement) for r in range(G)]


def _emulated_sharded_step(blocks, xs):
    """The token-sharded step of qmoe.ep with G emulated ranks on one GPU; xs[r] = rank r's tokens [T][H]."""
    from qmoe.ep import DeviceEngine
    G, T, H = len(blocks), xs[0].shape[0], xs[0].shape[1]
    eng = [DeviceEngine(b) for b in blocks]
    k = blocks[0].top_k
    dev = xs[0].device
    meta = [torch.empty(T, 2 * k, dtype=torch.int32, device=dev) for _ in range(G)]
    shared = [torch.empty(T, H, device=dev) for _ in range(G)]
    send_x = [torch.empty(G, T, H, device=dev) for _ in range(G)]
    send_m = [torch.empty(G, T, 2 * k, dtype=torch.int32, device=dev) for _ in range(G)]
    home = [torch.empty(G, T, dtype=torch.int32, device=dev) for _ in range(G)]
    counts = [torch.empty(G, dtype=torch.int32, device=dev) for _ in range(G)]
    for r in range(G):
        eng[r].route(xs[r], meta[r], shared[r])
        eng[r].pack(xs[r], meta[r], send_x[r], send_m[r], home[r], counts[r])
    # all_to_all: rank d receives block d of every source s, stacked by s
    recv_x = [torch.stack([send_x[s][d] for s in range(G)]) for d in range(G)]
    recv_m = [torch.stack([send_m[s][d] for s in range(G)]) for d in range(G)]
    partial = [torch.empty(G, T, H, device=dev) for _ in range(G)]
    for d in range(G):
        eng[d].experts(recv_x[d].view(G * T, H), recv_m[d].view(G * T, 2 * k), partial[d].view(G * T, H))
    back = [torch.stack([partial[d][s] for d in range(G)]) for s in range(G)]
    outs = []
    for r in range(G):
        out = torch.empty(T, H, device=dev)
        eng[r].combine(back[r], home[r], shared[r], out)
        outs.append(out)
    torch.cuda.synchronize()
    return outs, [m.cpu().numpy() for m in meta], [c.cpu().numpy() for c in counts]


def _emulated_p2p_step(blocks, xs, fold=False):
    """The peer-memory step with G emulated ranks on one GPU (contexts connected with plain pointers); fold:
    routed by qe_moe_ep_route_p2p, the shared expert running in the expert stage's launches."""
    import ctypes as C
    from qmoe.ep import DeviceEngine
    from qmoe.lib import lib
    G, T, H = len(blocks), xs[0].shape[0], xs[0].shape[1]
    k = blocks[0].top_k
    dev = xs[0].device
    eng = [DeviceEngine(b) for b in blocks]
    for e in eng:
        e.xchg_create(T)
    arr = (C.c_void_p * G)(*[e.xchg for e in eng])
    assert lib().qe_ep_xchg_connect_local(arr, G) == 0
    meta = [torch.empty(T, 2 * k, dtype=torch.int32, device=dev) for _ in range(G)]
    shared = [torch.empty(T, H, device=dev) for _ in range(G)]
    home = [torch.empty(G, T, dtype=torch.int32, device=dev) for _ in range(G)]
    counts = [torch.empty(G, dtype=torch.int32, device=dev) for _ in range(G)]
    for r in range(G):
        if fold:
            eng[r].route_p2p(xs[r], meta[r])
        else:
            eng[r].route(xs[r], meta[r], shared[r])
        eng[r].dispatch_p2p(xs[r], meta[r], home[r], counts[r])
    for d in range(G):
        eng[d].experts_p2p(T)
    outs = []
    for r in range(G):
        out = torch.empty(T, H, device=dev)
        eng[r].combine_p2p(T, home[r], None if fold else shared[r], out)
        outs.append(out)
    torch.cuda.synchronize()
    res = [o.cpu().numpy() for o in outs]
    for e in eng:
        e.xchg_free()
    return res


@pytest.mark.parametrize("fold", [False, True])
@pytest.mark.parametrize("G,T", [(1, 16), (2, 64), (4, 24), (8, 5)])
def test_ep_p2p_emulated_equals_all_to_all(G, T, fold):
    """Bit-identical to the all_to_all step, also with the shared expert folded into the expert stage (the
    same tcgen05 kernels and token tile width run it in both batches here, and every token is an independent
    MMA column)."""
    blocks = _blocks(CFG, G)
    gen = torch.Generator().manual_seed(500 + G + T)
    xs = [torch.randn(T, CFG.hidden, generator=gen).cuda() for _ in range(G)]
    want, _, _ = _emulated_sharded_step(blocks, xs)
    got = _emulated_p2p_step(blocks, xs, fold)
    for r in range(G):
        assert np.array_equal(got[r].view(np.uint32), want[r].cpu().numpy().view(np.uint32)), f"rank {r}"
    for b in blocks:
        b.close()


def _rel(a, b):
    return np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-30)


@pytest.mark.parametrize("G,T", [(1, 64), (1, 8), (2, 64), (4, 32), (8, 16), (8, 3)])
def test_ep_emulated_vs_single(G, T):
    ref = qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5)
    blocks = _blocks(CFG, G)
    gen = torch.Generator().manual_seed(100 + G * 7 + T)
    xs = [torch.randn(T, CFG.hidden, generator=gen).cuda() for _ in range(G)]
    outs, metas, counts = _emulated_sharded_step(blocks, xs)
    k = CFG.top_k
    for r in range(G):
        want = torch.empty_like(xs[r])
        ref.forward_device(T, xs[r].data_ptr(), want.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        idx, score = ref.route(xs[r].cpu().numpy())
        assert np.array_equal(metas[r][:, :k], idx)
        assert np.array_equal(metas[r][:, k:].view(np.float32).view(np.uint32), score.view(np.uint32))
        got, w = outs[r].cpu().numpy(), want.cpu().numpy()
        # each rank's destinations: tokens with an expert on d
        dests = (idx // (CFG.E // G))
        for d in range(G):
            assert counts[r][d] == int(np.any(dests == d, axis=1).sum())
        if G == 1:
            # one rank: same expert path (the experts call sees the same T rows), bit-identical
            assert np.array_equal(got.view(np.uint32), w.view(np.uint32)), "ep_size 1 differs from forward"
        else:
            # regrouped fp32 sum, and the experts call may take the other expert path (G*T rows)
            assert _rel(got, w).max() <= 5e-6
    for b in blocks + [ref]:
        b.close()


def test_ep_vs_oracle():
    G, T = 4, 24
    cfg = oracle.BlockCfg(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits)
    ob = oracle.SynthBlock(cfg, seed=9)
    blocks = _blocks(CFG, G, seed=9)
    xs_np = [ob.x(T, seed=300 + r) for r in range(G)]
    outs, _, _ = _emulated_sharded_step(blocks, [torch.from_numpy(x).cuda() for x in xs_np])
    for r in range(G):
        want, _, _ = ob.forward(xs_np[r])
        got = outs[r].cpu().numpy()
        assert _rel(got, want).max() <= 1e-5
        assert np.abs(got - want).max() <= 1e-4
    for b in blocks:
        b.close()


@pytest.mark.parametrize("G,T,extra", [(2, 40, 4), (4, 24, 2), (8, 16, 1), (8, 3, 2)])
def test_ep_placement_emulated(G, T, extra):
    """A placement planned from a Zipf-skewed calibration batch (qmoe.placement), `extra` spare slots per rank
    holding replicas of the hot experts: each handle holds its row of the table, the rows sent to each rank are
    those the host rule (replica (t + src) mod n) predicts, the sharded and peer-memory steps agree bit for bit,
    and both steps and the replicated step match the single-handle forward."""
    from qmoe.placement import Placement, histogram
    bias = qmoe.zipf_router_bias(CFG.E, 1.1, seed=7)
    ref = qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, router_bias=bias)
    gen = torch.Generator().manual_seed(900 + G + T)
    calib = torch.randn(256, CFG.hidden, generator=gen).numpy()
    pl = Placement.from_load(histogram(ref.route(calib)[0], CFG.E), G, CFG.E // G + extra)
    assert pl.nrep.max() > 1
    blocks = _blocks(CFG, G, router_bias=bias, placement=pl)
    for r, b in enumerate(blocks):
        assert b.held_experts().tolist() == [int(e) for e in pl.table[r] if e >= 0]
    xs = [torch.randn(T, CFG.hidden, generator=gen).cuda() for _ in range(G)]
    outs, metas, counts = _emulated_sharded_step(blocks, xs)
    # folded shared expert only where its batch takes the same kernels as the separate pass (T >= 5 rows: at
    # T <= 4 the separate pass runs the decode GEMVs, the folded one the tensor-core kernels)
    p2p = _emulated_p2p_step(blocks, xs, fold=T > 4)
    k = CFG.top_k
    for r in range(G):
        want = ref.forward(xs[r].cpu().numpy())
        idx = metas[r][:, :k]
        dest = pl.dest(idx, r)
        for d in range(G):
            assert counts[r][d] == int(np.any(dest == d, axis=1).sum())
        got = outs[r].cpu().numpy()
        assert _rel(got, want).max() <= 5e-6
        assert np.array_equal(p2p[r].view(np.uint32), got.view(np.uint32)), f"rank {r}"
    # replicated step: the same tokens on every rank, the partials summed in rank order
    from qmoe.ep import DeviceEngine
    x = xs[0]
    eng = [DeviceEngine(b) for b in blocks]
    parts = torch.empty(G, T, CFG.hidden, device="cuda")
    shared = torch.empty(T, CFG.hidden, device="cuda")
    for r in range(G):
        meta = torch.empty(T, 2 * k, dtype=torch.int32, device="cuda")
        eng[r].route(x, meta, shared)
        eng[r].experts(x, meta, parts[r])
    out = torch.empty(T, CFG.hidden, device="cuda")
    eng[0].combine(parts, None, shared, out)
    torch.cuda.synchronize()
    assert _rel(out.cpu().numpy(), ref.forward(x.cpu().numpy())).max() <= 5e-6
    for b in blocks + [ref]:
        b.close()


def test_ep_refusals():
    b = qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, ep_rank=1, ep_size=2)
    x = np.zeros((2, CFG.hidden), np.float32)
    with pytest.raises(qmoe.EngineError):
        b.forward(x)   # a handle with half the experts has no whole-block forward
    b.close()
    with pytest.raises(qmoe.EngineError):
        qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, ep_rank=0, ep_size=3)
    with pytest.raises(qmoe.EngineError):
        qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, ep_rank=2, ep_size=2)
    E = CFG.E
    full = np.arange(E, dtype=np.int32).reshape(2, E // 2)
    for bad in (full[:, :-1],                                   # an expert held by no rank
                np.concatenate([full, full[:, :1]], axis=1),    # rank 0 lists expert 0 twice
                np.where(full == 3, E, full)):                  # an id outside [0, E)
        with pytest.raises(qmoe.EngineError):
            qmoe.MoeBlock(CFG.hidden, E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, ep_rank=0, ep_size=2,
                          placement=bad)
    with pytest.raises(qmoe.EngineError):   # a placement needs ep_size > 1
        qmoe.MoeBlock(CFG.hidden, E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, placement=full[:1])


def _nccl_worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from qmoe.ep import ExpertParallelMoe
        ep = ExpertParallelMoe.on_gpu(CFG, rank, world, rank, seed=5)
        if mode.startswith("p2p"):
            ep.enable_p2p(64, barrier="nccl" if mode == "p2p_unfolded" else "device")
        ref = qmoe.MoeBlock(CFG.hidden, CFG.E, CFG.top_k, CFG.inter, CFG.sh_inter, CFG.bits, seed=5, device=rank)
        T = 48
        gen = torch.Generator().manual_seed(1000 + (rank if mode != "replicated" else 0))
        x = torch.randn(T, CFG.hidden, generator=gen).cuda(rank)

        def reference(xv):
            want = torch.empty_like(xv)
            ref.forward_device(T, xv.data_ptr(), want.data_ptr(), torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            return want.cpu().numpy()

        if mode == "p2p_graph":
            # the peer-memory step with device barriers, captured once and replayed on new inputs
            for _ in range(2):
                ep.forward(x, mode="p2p")
            torch.cuda.synchronize()
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                g_out = ep.forward(x, mode="p2p")
            worst = 0.0
            for _ in range(3):
                x.copy_(torch.randn(T, CFG.hidden, generator=gen).cuda(rank))
                g.replay()
                torch.cuda.synchronize()
                worst = max(worst, float(_rel(g_out.cpu().numpy(), reference(x)).max()))
            del g, g_out
            torch.cuda.synchronize()
            q.put((rank, worst, qmoe.lib().qe_device_error()))
        else:
            out = ep.forward(x, mode="p2p", fold=False) if mode == "p2p_unfolded" else ep.forward(x, mode=mode)
            torch.cuda.synchronize()
            q.put((rank, float(_rel(out.cpu().numpy(), reference(x)).max()), qmoe.lib().qe_device_error()))
        ep.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["sharded", "replicated", "p2p", "p2p_unfolded", "p2p_graph"])
def test_ep_nccl_two_gpus(mode):
    """One process per GPU over NCCL against the single-handle forward. p2p: peer-memory exchange with the
    library's device barriers; p2p_unfolded: the separate shared-expert pass and NCCL barriers; p2p_graph: the
    device-barrier step captured in a CUDA graph and replayed on new inputs."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes
    for _ in procs:
        rank, rel, err = q.get(timeout=10)
        assert err == 0, (rank, err)
        assert rel <= 5e-6, (rank, rel)


def test_exchange_barrier_timeout_is_reported_and_cleared():
    """qe_ep_xchg_barrier's bounded wait: with two contexts of one GPU connected and only one of them entering
    the barrier (the other's flag is never written), the wait gives up after the 20 ms bound set here, the kernel
    returns, qe_device_error_on reports 201 for that device, and qe_device_error_reset clears it. No kernel waits
    on another kernel: the peer never launches anything."""
    import ctypes as C
    from qmoe.ep import DeviceEngine
    from qmoe.lib import lib
    cfg = dict(hidden=256, E=16, top_k=4, inter=128, sh_inter=128, bits=4)
    blocks = [qmoe.MoeBlock(**cfg, seed=3, ep_rank=r, ep_size=2, max_tokens=16) for r in range(2)]
    eng = [DeviceEngine(b) for b in blocks]
    for e in eng:
        e.xchg_create(16)
    arr = (C.c_void_p * 2)(*[e.xchg for e in eng])
    assert lib().qe_ep_xchg_connect_local(arr, 2) == 0
    assert lib().qe_device_error_reset(0) == 0
    assert lib().qe_ep_xchg_set_timeout_ms(C.c_void_p(eng[0].xchg), 20) == 0
    assert lib().qe_ep_xchg_set_timeout_ms(C.c_void_p(eng[0].xchg), 0) == -1
    eng[0].xchg_barrier()
    torch.cuda.synchronize()
    assert lib().qe_device_error_on(0) == 201
    assert lib().qe_device_error_reset(0) == 0
    assert lib().qe_device_error_on(0) == 0
    for e in eng:
        e.xchg_free()
    for b in blocks:
        b.close()
