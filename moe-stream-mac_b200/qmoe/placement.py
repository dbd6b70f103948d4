"""Expert placement over expert-parallel ranks, planned from the routing the model actually produces.

The reference serves one process and records its routing for offline analysis: with QE_TRACE set, every
moe_layer_step appends int32 layer followed by the token's top-k expert ids (engine/src/moe_layer.c:57-64),
and its analysis scripts count per-expert popularity from that file. Here the same records (written by
qe_moe_forward with QE_TRACE, in the same format) feed a placement planner: a per-expert load histogram is
turned into a table [ranks][slots] of expert ids where the hottest experts get extra replicas, and the
library splits each replicated expert's tokens over its replicas by the rule of include/qe_moe.h
(assignment (t, e) from source rank src goes to reps[e][(t + src) % nrep[e]]).

The planner is a greedy longest-processing-time assignment under a slot-count constraint: with G ranks of
`slots` slots each, the G*slots - E spare slots go one by one to the expert with the largest load per
replica, then replicas are placed, heaviest first, on the least-loaded rank that has a free slot and does
not already hold that expert.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


class Placement:
    """table[G][slots]: the global expert ids each rank holds (-1 = empty slot), the same on every rank."""

    def __init__(self, table, E: int):
        t = np.ascontiguousarray(table, np.int32)
        if t.ndim != 2 or t.shape[0] < 2 or t.shape[1] < 1:
            raise ValueError("placement table must be [ranks >= 2][slots >= 1]")
        seen = np.zeros(E, np.int64)
        for r, row in enumerate(t):
            ids = row[row >= 0]
            if np.any(row < -1) or np.any(ids >= E):
                raise ValueError(f"rank {r}: ids outside [0, {E})")
            if len(np.unique(ids)) != len(ids):
                raise ValueError(f"rank {r} lists an expert twice")
            if not len(ids):
                raise ValueError(f"rank {r} holds no expert")
            seen[ids] += 1
        if np.any(seen == 0):
            raise ValueError(f"experts held by no rank: {np.flatnonzero(seen == 0).tolist()}")
        self.table, self.E = t, E
        self.G, self.slots = t.shape
        self.nrep = seen.astype(np.int32)
        # reps[e][i]: the i-th rank holding e, ascending (-1 past nrep[e])
        self.reps = np.full((E, self.G), -1, np.int32)
        fill = np.zeros(E, np.int64)
        for r in range(self.G):
            for e in t[r][t[r] >= 0]:
                self.reps[e, fill[e]] = r
                fill[e] += 1

    @classmethod
    def contiguous(cls, E: int, G: int) -> "Placement":
        """Rank r holds [r*E/G, (r+1)*E/G): the layout a handle gets without a table."""
        if E % G:
            raise ValueError("G must divide E")
        return cls(np.arange(E, dtype=np.int32).reshape(G, E // G), E)

    @classmethod
    def from_load(cls, load, G: int, slots: int) -> "Placement":
        """Greedy plan for a per-expert load (assignment counts or any non-negative weights)."""
        load = np.asarray(load, np.float64)
        E = load.shape[0]
        if slots * G < E:
            raise ValueError(f"{G} ranks x {slots} slots cannot hold {E} experts")
        if slots > E:
            raise ValueError("more slots per rank than experts")
        nrep = np.ones(E, np.int64)
        for _ in range(slots * G - E):
            per = np.where(nrep < G, load / nrep, -1.0)
            e = int(np.argmax(per))
            if per[e] <= 0:
                break
            nrep[e] += 1
        # replicas, heaviest per-replica load first (ties: lower id first)
        order = sorted(((load[e] / nrep[e], e) for e in range(E) for _ in range(nrep[e])), key=lambda p: (-p[0], p[1]))
        rank_load = np.zeros(G)
        rows: list[list[int]] = [[] for _ in range(G)]
        for w, e in order:
            best = None
            for r in range(G):
                if len(rows[r]) < slots and e not in rows[r] and (best is None or rank_load[r] < rank_load[best]):
                    best = r
            if best is None:
                continue   # no rank can take another copy of e: fewer replicas, the slot stays empty
            rows[best].append(e)
            rank_load[best] += w
        table = np.full((G, slots), -1, np.int32)
        for r in range(G):
            table[r, :len(rows[r])] = sorted(rows[r])
        return cls(table, E)

    def dest(self, idx, src: int) -> np.ndarray:
        """Serving rank of each assignment idx[T][k] (global ids, -1 = empty slot -> -1) from source rank src."""
        idx = np.asarray(idx, np.int64)
        t = np.arange(idx.shape[0])[:, None]
        e = np.where(idx >= 0, idx, 0)
        n = self.nrep[e]
        d = self.reps[e, (t + src) % n]
        return np.where(idx >= 0, d, -1)

    def rank_loads(self, idx_by_src) -> np.ndarray:
        """Assignments each rank serves when source rank s routes idx_by_src[s][T][k]."""
        out = np.zeros(self.G, np.int64)
        for s, idx in enumerate(idx_by_src):
            d = self.dest(idx, s)
            out += np.bincount(d[d >= 0], minlength=self.G)
        return out


def histogram(idx, E: int) -> np.ndarray:
    """Per-expert assignment counts of routing results idx[..][k] (-1 entries ignored)."""
    a = np.asarray(idx).ravel()
    return np.bincount(a[a >= 0], minlength=E).astype(np.int64)


def read_trace(path, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """(layer[N], idx[N][top_k]) from a QE_TRACE file: per token int32 layer then int32 idx[top_k]."""
    raw = np.fromfile(Path(path), dtype=np.int32)
    if raw.size % (1 + top_k):
        raise ValueError(f"{path}: {raw.size} int32 values is not a whole number of {1 + top_k}-value records")
    rec = raw.reshape(-1, 1 + top_k)
    return rec[:, 0].copy(), rec[:, 1:].copy()


def histogram_from_trace(path, top_k: int, E: int, layer: int | None = None) -> np.ndarray:
    """Per-expert assignment counts of one layer (or all) of a QE_TRACE file."""
    layers, idx = read_trace(path, top_k)
    if layer is not None:
        idx = idx[layers == layer]
    return histogram(idx, E)
