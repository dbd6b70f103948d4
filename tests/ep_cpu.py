"""A CPU engine with the contract of qmoe.ep.DeviceEngine, built on the oracle (test infrastructure only).

It lets the expert-parallel exchange of qmoe.ep.ExpertParallelMoe run under the gloo backend without a GPU:
route/pack/experts/combine have the semantics of the qe_moe_ep_* entry points of include/qe_moe.h, computed
with the oracle's restatement of the reference (oracle.SynthBlock.expert / shared_gate_logit, moe_layer.c).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

import oracle
from qmoe.placement import Placement

ROUTED = 0x40000000   # QE_EP_ROUTED of include/qe_moe.h


def _sigmoid(g: np.float32) -> np.float32:
    x = np.array([g], np.float32)
    y = np.empty(1, np.float32)
    oracle.lib().or_sigmoid(oracle.fptr(y), oracle.fptr(x), 1)
    return y[0]


class OracleEngine:
    def __init__(self, blk: oracle.SynthBlock, rank: int, world: int, placement: Placement | None = None):
        self.blk = blk
        self.hidden, self.top_k, self.E = blk.cfg.hidden, blk.cfg.top_k, blk.cfg.E
        self.place = placement or Placement.contiguous(self.E, world)
        self.held = set(int(e) for e in self.place.table[rank] if e >= 0)
        self.rank, self.world = rank, world

    def route(self, x: torch.Tensor, meta: torch.Tensor, shared: torch.Tensor) -> None:
        xn, k = x.numpy(), self.top_k
        logits = self.blk.router_logits(xn)
        m = meta.numpy()
        sh = shared.numpy()
        for t in range(xn.shape[0]):
            _, idx, score = oracle.route_from_logits(logits[t], k)
            m[t, :k] = idx
            m[t, k:] = score.view(np.int32)
            sg = _sigmoid(self.blk.shared_gate_logit(xn[t]))
            sh[t] = np.float32(0.0) + sg * self.blk.expert(-1, xn[t])

    def pack(self, x, meta, send_x, send_meta, home, counts) -> None:
        T, k, G = x.shape[0], self.top_k, self.world
        xn, m = x.numpy(), meta.numpy()
        sx, sm, hm, cn = send_x.numpy(), send_meta.numpy(), home.numpy(), counts.numpy()
        dest = self.place.dest(m[:, :k], self.rank)   # the replica serving each slot (include/qe_moe.h rule)
        for d in range(G):
            n = 0
            for t in range(T):
                ids = m[t, :k]
                if np.any(dest[t] == d):
                    hm[d, t] = n
                    sx[d, n] = xn[t]
                    sm[d, n, :k] = np.where(dest[t] == d, ids | ROUTED, -1)
                    sm[d, n, k:] = m[t, k:]
                    n += 1
                else:
                    hm[d, t] = -1
            cn[d] = n
            sm[d, n:, :k] = -1
            sm[d, n:, k:] = 0

    def experts(self, x, meta, partial) -> None:
        xn, m, p, k = x.numpy(), meta.numpy(), partial.numpy(), self.top_k
        for r in range(xn.shape[0]):
            o = np.zeros(self.hidden, np.float32)
            for j in range(k):
                e = int(m[r, j])
                if e < 0:
                    continue
                if e & ROUTED:       # routed here by the sender
                    mine = (e & ~ROUTED) in self.held
                    e &= ~ROUTED
                else:                # the replicated step's own rows: row r is token r, source rank 0
                    mine = int(self.place.reps[e, r % self.place.nrep[e]]) == self.rank
                if mine:
                    s = m[r, k + j:k + j + 1].view(np.float32)[0]
                    o = o + s * self.blk.expert(e, xn[r])
            p[r] = o

    def combine(self, part, home, shared, out) -> None:
        pn, sh, o = part.numpy(), shared.numpy(), out.numpy()
        G, T = pn.shape[0], o.shape[0]
        hm = None if home is None else home.numpy()
        for t in range(T):
            acc = np.zeros(self.hidden, np.float32)
            for d in range(G):
                pos = t if hm is None else int(hm[d, t])
                if pos >= 0:
                    acc = acc + pn[d, pos]
            o[t] = acc + sh[t]
