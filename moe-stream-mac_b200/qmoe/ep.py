"""Expert parallelism: one routed MoE block sharded by expert over the ranks of a torch.distributed group.

The reference runs the block in one process (engine/src/moe_layer.c:66-89). Here expert e lives on rank
e // (E / world), or where a placement table puts it (qmoe.placement: hot experts replicated on several
ranks, each token served by one replica); the router and the shared expert are replicated. Step shapes:

* token-sharded (prefill batches): every rank routes its own tokens, packs for each destination rank the rows
  of its tokens that have at least one expert there (token order, padded to T rows per destination so the
  exchange is one all_to_all with equal blocks and needs no host round trip for the counts), exchanges rows
  and slot lists, computes the partial sums of the slots it owns, sends them back, and sums the partials in
  rank order plus the gated shared expert;
* replicated (decode): every rank holds the same tokens, computes the partial sums of its own experts, and
  the partials are all-gathered and summed in rank order (deterministic, unlike a reduction whose order
  depends on the collective's algorithm);
* p2p: the token-sharded step with the exchange done by the library's kernels through peer memory: the
  packing kernel stores each row straight into its destination rank's receive buffer (NVLink, CUDA IPC
  mappings), and the expert stage's combine stores each partial row straight into its home rank's return
  buffer; NCCL only provides the two barriers (one-element all_reduce). Same arithmetic, bit-identical.

The arithmetic runs in an engine: `DeviceEngine` calls libqengine_b200's qe_moe_ep_* entry points on the
rank's GPU (the product path). Tests substitute a CPU engine with the same contract to check the exchange
logic under the gloo backend.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .block import EngineError, MoeBlock
from .lib import lib


class DeviceEngine:
    """The qe_moe_ep_* calls of include/qe_moe.h on one handle (device tensors, torch's current stream)."""

    def __init__(self, block: MoeBlock):
        self.block = block
        self.hidden, self.top_k = block.hidden, block.top_k

    def _s(self) -> C.c_void_p:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    @staticmethod
    def _p(t: torch.Tensor | None) -> C.c_void_p:
        return C.c_void_p(t.data_ptr() if t is not None else None)

    def route(self, x, meta, shared):
        if lib().qe_moe_ep_route_device(self.block.handle, x.shape[0], self._p(x), self._p(meta), self._p(shared),
                                        self._s()):
            raise EngineError("qe_moe_ep_route_device failed")

    def pack(self, x, meta, send_x, send_meta, home, counts):
        if lib().qe_moe_ep_pack_device(self.block.handle, x.shape[0], self._p(x), self._p(meta), self._p(send_x),
                                       self._p(send_meta), self._p(home), self._p(counts), self._s()):
            raise EngineError("qe_moe_ep_pack_device failed")

    def experts(self, x, meta, partial):
        if lib().qe_moe_ep_experts_device(self.block.handle, x.shape[0], self._p(x), self._p(meta),
                                          self._p(partial), self._s()):
            raise EngineError("qe_moe_ep_experts_device failed")

    def combine(self, part, home, shared, out):
        if lib().qe_moe_ep_combine_device(self.block.handle, out.shape[0], self._p(part), self._p(home),
                                          self._p(shared), self._p(out), self._s()):
            raise EngineError("qe_moe_ep_combine_device failed")

    # ---- exchange through peer memory
    xchg = None

    def xchg_create(self, t_max: int) -> bytes:
        nb = lib().qe_ep_xchg_handle_bytes()
        handle = (C.c_uint8 * nb)()
        self.xchg = lib().qe_ep_xchg_create(self.block.handle, t_max, handle)
        if not self.xchg:
            raise EngineError("qe_ep_xchg_create failed")
        return bytes(handle)

    def xchg_connect(self, handles: bytes) -> None:
        buf = (C.c_uint8 * len(handles)).from_buffer_copy(handles)
        if lib().qe_ep_xchg_connect(self.xchg, buf):
            raise EngineError("qe_ep_xchg_connect failed")

    def xchg_free(self) -> None:
        if self.xchg:
            lib().qe_ep_xchg_free(self.xchg)
            self.xchg = None

    def xchg_barrier(self):
        if lib().qe_ep_xchg_barrier(self.xchg, self._s()):
            raise EngineError("qe_ep_xchg_barrier failed")

    def route_p2p(self, x, meta):
        if lib().qe_moe_ep_route_p2p(self.block.handle, self.xchg, x.shape[0], self._p(x), self._p(meta), self._s()):
            raise EngineError("qe_moe_ep_route_p2p failed")

    def dispatch_p2p(self, x, meta, home, counts):
        if lib().qe_moe_ep_dispatch_p2p(self.block.handle, self.xchg, x.shape[0], self._p(x), self._p(meta),
                                        self._p(home), self._p(counts), self._s()):
            raise EngineError("qe_moe_ep_dispatch_p2p failed")

    def experts_p2p(self, T: int):
        if lib().qe_moe_ep_experts_p2p(self.block.handle, self.xchg, T, self._s()):
            raise EngineError("qe_moe_ep_experts_p2p failed")

    def combine_p2p(self, T: int, home, shared, out):
        if lib().qe_moe_ep_combine_p2p(self.block.handle, self.xchg, T, self._p(home), self._p(shared), self._p(out),
                                       self._s()):
            raise EngineError("qe_moe_ep_combine_p2p failed")


class ExpertParallelMoe:
    """One routed MoE block, experts sharded over `group` (default: the world), one rank per GPU."""

    def __init__(self, engine, rank: int, world: int, group=None, device: torch.device | str = "cuda"):
        self.engine, self.rank, self.world, self.group = engine, rank, world, group
        self.device = torch.device(device)
        self.hidden, self.top_k = engine.hidden, engine.top_k
        self.last_counts: torch.Tensor | None = None   # rows sent to each rank by the last sharded step

    @classmethod
    def on_gpu(cls, cfg, rank: int, world: int, device: int, *, seed: int, block: int = 0, router_bias=None,
               max_tokens: int = 4096, group=None, placement=None) -> "ExpertParallelMoe":
        """A synthetic block (qmoe.synth.MoeConfig shape) holding experts [rank*E/world, (rank+1)*E/world), or
        row `rank` of a qmoe.placement.Placement."""
        blk = MoeBlock(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, max_tokens=max_tokens,
                       device=device, seed=seed, block=block, router_bias=router_bias, ep_rank=rank, ep_size=world,
                       placement=placement)
        return cls(DeviceEngine(blk), rank, world, group, torch.device("cuda", device))

    @staticmethod
    def plan_placement(cfg, rank: int, world: int, device: int, x: torch.Tensor, spare_slots: int, *, seed: int,
                       block: int = 0, router_bias=None, group=None):
        """Plan a placement with `spare_slots` replica slots per rank from the routing of every rank's calibration
        tokens x (collective): a contiguous handle routes x, the per-expert counts are summed over the ranks,
        and qmoe.placement.Placement.from_load places E/world + spare_slots experts per rank."""
        from .placement import Placement, histogram
        if cfg.E % world:
            raise ValueError("the calibration handle needs world to divide E")
        blk = MoeBlock(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, max_tokens=x.shape[0],
                       device=device, seed=seed, block=block, router_bias=router_bias, ep_rank=rank, ep_size=world)
        try:
            idx, _ = blk.route(x.cpu().numpy())
        finally:
            blk.close()
        h = torch.from_numpy(histogram(idx, cfg.E)).to(torch.device("cuda", device))
        dist.all_reduce(h, group=group)
        return Placement.from_load(h.cpu().numpy(), world, min(cfg.E, cfg.E // world + spare_slots))

    def _empty(self, *shape, dtype=torch.float32):
        return torch.empty(*shape, dtype=dtype, device=self.device)

    def enable_p2p(self, t_max: int, barrier: str = "device") -> None:
        """Create this rank's exchange buffers and map every other rank's (collective: all ranks call it).
        barrier: "device" (qe_ep_xchg_barrier through the exchange's flags; the step then holds no NCCL call and
        can be captured in a CUDA graph) or "nccl" (a one-element all_reduce)."""
        if barrier not in ("device", "nccl"):
            raise ValueError(f"barrier {barrier!r}")
        self.barrier_kind = barrier
        h = self.engine.xchg_create(t_max)
        mine = torch.tensor(list(h), dtype=torch.uint8, device=self.device)
        allh = torch.empty(self.world * len(h), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=self.group)
        self.engine.xchg_connect(bytes(allh.cpu().numpy().tobytes()))
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.t_max = t_max
        dist.barrier(group=self.group)

    def _barrier(self) -> None:
        """Stream-ordered: every rank's preceding kernels are done (and their peer stores visible)."""
        if getattr(self, "barrier_kind", "nccl") == "device":
            self.engine.xchg_barrier()
        else:
            dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        if getattr(self.engine, "xchg", None):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.engine.xchg_free()

    def forward(self, x: torch.Tensor, mode: str = "sharded", mark=None, fold: bool = True) -> torch.Tensor:
        """out[T][hidden] for this rank's x[T][hidden] (sharded), or for the tokens every rank holds
        (replicated). Every rank must call it with the same T and mode. mark(name), if given, is called
        after each phase (route, pack, dispatch, experts, return, combine), e.g. to record CUDA events.
        p2p with fold (the default when (world + 1) * T fits the handle's max_tokens): the shared expert runs
        on this rank's own rows inside the expert stage's launches (qe_moe_ep_route_p2p) instead of in a
        separate pass during routing."""
        if mode not in ("sharded", "replicated", "p2p"):
            raise ValueError(f"mode {mode!r}")
        mark = mark or (lambda name: None)
        T, H, k, G = x.shape[0], self.hidden, self.top_k, self.world
        meta = self._empty(T, 2 * k, dtype=torch.int32)
        out = self._empty(T, H)
        fold = fold and mode == "p2p" and (G + 1) * T <= self.engine.block.cfg.max_tokens
        if fold:
            shared = None
            self.engine.route_p2p(x, meta)
        else:
            shared = self._empty(T, H)
            self.engine.route(x, meta, shared)
        mark("route")
        if mode == "replicated":
            partial = self._empty(T, H)
            self.engine.experts(x, meta, partial)
            mark("experts")
            parts = self._empty(G, T, H)
            dist.all_gather_into_tensor(parts.view(G * T, H), partial, group=self.group)
            mark("return")
            self.engine.combine(parts, None, shared, out)
            mark("combine")
            return out
        if mode == "p2p":
            home, counts = self._empty(G, T, dtype=torch.int32), self._empty(G, dtype=torch.int32)
            self.engine.dispatch_p2p(x, meta, home, counts)
            mark("pack")
            self._barrier()
            mark("dispatch")
            self.engine.experts_p2p(T)
            mark("experts")
            self._barrier()
            mark("return")
            self.engine.combine_p2p(T, home, shared, out)
            mark("combine")
            self.last_counts = counts
            return out
        send_x, send_meta = self._empty(G, T, H), self._empty(G, T, 2 * k, dtype=torch.int32)
        home, counts = self._empty(G, T, dtype=torch.int32), self._empty(G, dtype=torch.int32)
        self.engine.pack(x, meta, send_x, send_meta, home, counts)
        mark("pack")
        recv_x, recv_meta = torch.empty_like(send_x), torch.empty_like(send_meta)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_meta, send_meta, group=self.group)
        mark("dispatch")
        partial = self._empty(G, T, H)
        self.engine.experts(recv_x.view(G * T, H), recv_meta.view(G * T, 2 * k), partial.view(G * T, H))
        mark("experts")
        back = torch.empty_like(partial)
        dist.all_to_all_single(back, partial, group=self.group)
        mark("return")
        self.engine.combine(back, home, shared, out)
        mark("combine")
        self.last_counts = counts
        return out
