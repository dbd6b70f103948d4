#!/usr/bin/env python
"""bench.py: MoE-layer tokens/s of the B200 routed-MoE block (libqengine_b200) vs the reference C engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

One step = one forward of one MoE block over the configuration's token batch (config c2: 512 tokens of the
4-bit hidden-2048 block, the configuration the benchmark metric is quoted on). Four blocks with distinct
weights (4 x 453 MB, far above the 126 MB L2) are used in rotation, so no step finds its weights in L2.
`value` is device-timed (CUDA events on the launching stream, inputs resident in HBM); `e2e` is the same
metric through the public host-buffer calls (pinned host x in, host out back, every step), with consecutive
steps pipelined by qe_moe_forward_async (each step's copies under its neighbours' kernels); `e2e.sync_value`
is the one-call-at-a-time figure of qe_moe_forward.
Under torchrun (N > 1) the block is expert-parallel (qmoe.ep): rank r holds experts [r*E/N, (r+1)*E/N) of
every block plus the replicated router and shared expert, routes its own 512 tokens, and exchanges rows and
partial sums through peer memory (the kernels store into the other GPUs' buffers; --ep-mode sharded: all_to_all
over NCCL), weak scaling (per-rank tokens fixed); value = tokens of all ranks / max rank time. With the
peer-memory exchange each block's step is replayed from a CUDA graph, as on one GPU.
--impl reference times the reference's own C engine (oracle/_ref, built from its sources) on the host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "moe-stream-mac_b200"))

import numpy as np  # noqa: E402
from qmoe.synth import CONFIGS  # noqa: E402

METRIC = "MoE-layer tokens/s"
PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def hbm_peak():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms from start to stop (warm-up, timed steps, e2e
    passes and sub-records alike); mark(name, start) brackets named phases, and stop() reports the samples inside
    any phase (median SM clock, reasons) plus a per-phase breakdown."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50", "-i", str(gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        self.phases = []   # [name, t0, t1]

    def mark(self, name: str, start: bool):
        if start:
            self.phases.append([name, time.time(), None])
        else:
            for ph in reversed(self.phases):
                if ph[0] == name and ph[2] is None:
                    ph[2] = time.time()
                    break

    def _summary(self, rows):
        sm = [float(r[2]) for r in rows]
        reasons = set()
        for r in rows:
            for n, v in zip(self.NAMES, r[6:10]):
                if v.strip() == "Active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][3]), "reasons": sorted(reasons),
                "samples": len(rows), "power_w_max": max(float(r[4]) for r in rows)}

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = [r.split(", ") for r in Path(self.f.name).read_text().splitlines() if r.count(",") >= 9]
        os.unlink(self.f.name)
        stamped = []
        for r in rows:
            try:
                ts = time.mktime(time.strptime(r[0].split(".")[0], "%Y/%m/%d %H:%M:%S")) + float("0." + r[0].split(".")[1])
            except Exception:
                continue
            stamped.append((ts, r))
        if not stamped:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        per_phase, inside = {}, []
        for name, t0, t1 in self.phases:
            sel = [r for ts, r in stamped if t0 - 0.06 <= ts <= (t1 or ts) + 0.06]
            if sel:
                per_phase.setdefault(name, []).extend(sel)
                inside.extend(sel)
        out = self._summary(inside or [r for _, r in stamped])
        out["scope"] = "samples inside the measured phases" if inside else "all samples (no phase overlapped one)"
        out["phases"] = {k: {kk: v for kk, v in self._summary(rs).items() if kk in ("sm_mhz", "reasons", "samples")}
                         for k, rs in per_phase.items()}
        return out


def router_bias(cfg, seed):
    """The configuration's skewed-popularity router bias (Zipf law over a seeded permutation), or None."""
    from qmoe.synth import zipf_router_bias
    return zipf_router_bias(cfg.E, cfg.zipf_s, seed=seed) if cfg.zipf_s else None


def reference_block(cfg, seed, threads):
    import oracle as O
    if not O.ref_available():
        return None, None
    O.ref().ref_set_threads(threads)
    blk = O.SynthBlock(O.BlockCfg(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, cfg.group_size),
                       seed, router_bias=router_bias(cfg, seed))
    return O, blk


def time_reference(cfg, seed, sample_tokens, steps, warmup, threads, budget_s=None):
    """Reference C engine (Mode B harness over the reference's own qmat_matvec/op_* from oracle/_ref):
    tokens one after the other, as the engine's prefill does; OpenMP inside qmat_matvec."""
    O, blk = reference_block(cfg, seed, threads)
    if blk is None:
        return None
    x = blk.x(sample_tokens)
    for _ in range(warmup):
        blk.forward_ref(x[:1])
    times, done = [], 0
    t_all = time.perf_counter()
    for _ in range(steps):
        t = time.perf_counter()
        blk.forward_ref(x)
        times.append(time.perf_counter() - t)
        done += 1
        if budget_s and time.perf_counter() - t_all > budget_s:
            break
    blk.close()
    sec = sum(times)
    return {"value": done * sample_tokens / sec, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{done} x {sample_tokens} tokens of {cfg.name} through the reference's moe_layer_step "
                      f"restated around its own qmat_matvec/op_softmax/op_topk/op_silu_mul (oracle/_ref), "
                      f"{threads} OpenMP threads, experts in RAM"}


def host_cpu() -> dict:
    """CPU model, physical cores and logical CPUs of this host (the reference's OpenMP threads use all logical
    CPUs)."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    phys = None
    try:
        import psutil
        phys = psutil.cpu_count(logical=False)
    except Exception:
        pass
    return {"cpu_model": model, "physical_cores": phys, "logical_cpus": os.cpu_count()}


def time_reference_mode_r(cfg, seed, sample_tokens, threads, budget_s=8.0):
    """The reference's UNMODIFIED moe_layer_step (Mode R): a synthetic checkpoint of the block (8-bit quantized
    router, as real checkpoints have) is written in the MLX safetensors layout to a temporary directory, opened
    with the reference's own k3_st_open / expert_tensor_open / load_qmat, and every token preads its 8 selected
    experts from that page-cache-warm file (engine/src/expert_store.c:54-61), as the engine does."""
    import shutil
    import oracle as O
    from oracle.checkpoint import checkpoint_tensors, write_safetensors
    if not O.ref_available():
        return None
    bc = O.BlockCfg(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, cfg.group_size, True)
    blk = O.SynthBlock(bc, seed)
    d = Path(tempfile.mkdtemp(prefix="qe_moder_"))
    try:
        prefix = "language_model.model.layers.0.mlp"
        write_safetensors(d / "model.safetensors", checkpoint_tensors(prefix, blk.arrays()))
        R = O.ref()
        R.ref_set_threads(threads)
        h = R.ref_r_open(str(d).encode(), prefix.encode(), cfg.hidden, cfg.top_k, cfg.inter, cfg.sh_inter,
                         cfg.group_size)
        if not h:
            return None
        x = blk.x(sample_tokens)
        out = np.empty(cfg.hidden, np.float32)
        for t in range(min(2, sample_tokens)):   # warm: the file is in the page cache after its first reads
            R.ref_r_step(h, O.fptr(np.ascontiguousarray(x[t])), O.fptr(out))
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            R.ref_r_step(h, O.fptr(np.ascontiguousarray(x[done % sample_tokens])), O.fptr(out))
            done += 1
        sec = time.perf_counter() - t0
        return {"value": done / sec, "unit": "tokens/s", "cores": threads, "kind": "reference",
                "sample": f"{done} tokens of {cfg.name} (8-bit quantized router) through the reference's unmodified "
                          f"moe_layer_step, experts pread from a page-cache-warm safetensors file, {threads} threads"}
    finally:
        blk.close()
        shutil.rmtree(d, ignore_errors=True)


def run_reference_arm(args, cfg):
    rank, _, world = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    res = time_reference(cfg, 1, args.ref_tokens, args.steps, min(args.warmup, 3), threads, budget_s=150)
    if res is not None and args.stack:   # one block timed; a token through the stack takes `blocks` passes
        res["value"] /= cfg.blocks
        res["sample"] += f"; one block timed, value divided by the stack's {cfg.blocks} blocks"
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqref.so (reference build) is missing"}))
        return
    res.update(host_cpu())
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * args.ref_tokens / res["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(cfg, world, cfg.blocks if args.stack else 4, stack=args.stack),
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def workload_config(cfg, world, blocks=4, ep_mode="rows and partial sums stored into peer memory by the kernels",
                    stack=False):
    mb = blocks * (cfg.E // world * cfg.expert_bytes + cfg.shared_bytes + 4 * cfg.E * cfg.hidden) / 1e6
    l2 = (f"the whole stack of {blocks} independent blocks runs every step, each fed the step's tokens ({mb:.0f} "
          f"MB of weights per GPU > 126 MB L2)" if stack else
          f"{blocks} blocks with distinct weights rotated per step ({mb:.0f} MB of weights per GPU > 126 MB L2)")
    return {"workload": f"{cfg.name}: {cfg.note}", "tokens_per_step": cfg.tokens, "hidden": cfg.hidden,
            "experts": cfg.E, "top_k": cfg.top_k, "inter": cfg.inter, "sh_inter": cfg.sh_inter, "bits": cfg.bits,
            "group_size": cfg.group_size, "router": "fp32", "parallelism": "1 GPU" if world == 1 else
            f"expert parallel over {world} GPUs ({cfg.E // world} experts each; router and shared expert "
            f"replicated; {cfg.tokens} tokens per GPU; exchange: {ep_mode})",
            "l2": l2, "stack_blocks": blocks if stack else None,
            "routing": (f"router logit bias -{0.75 * cfg.zipf_s:g} ln(popularity rank) (Zipf({cfg.zipf_s:g})-skewed)"
                        if cfg.zipf_s else "seeded random router, no bias")}


def profiled_traffic(kernel: str, config: str):
    """DRAM bytes per launch (read + write) of `kernel` on `config` from the committed ncu summaries
    (lines `dram_bytes_per_launch[<kernel>,<config>]: N` under profiles/), or None."""
    import re
    key = f"dram_bytes_per_launch[{kernel},{config}]:"
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            line = line.strip()
            if line.startswith(key):
                m = re.match(r".*:\s*(\d+)", line)
                if m:
                    return int(m.group(1)), f.name
    return None


def expert_kernel_name(cfg, stage: str, T: int) -> str:
    """The kernel the library runs for this stage: decode GEMVs for up to 4 tokens, the grouped GEMVs for larger
    batches of at most 4 routed assignments per expert on average (or when selected, QE_EXPERT_PATH=group), the
    tensor-core kernels for the rest (group size 64, every matrix a whole number of 128-row tiles), mma.sync
    kernels otherwise."""
    path = os.environ.get("QE_EXPERT_PATH", "auto")
    bh, bi = cfg.hidden * cfg.bits // 8, cfg.inter * cfg.bits // 8
    tc = (T >= 5 and cfg.group_size == 64 and all(d % 128 == 0 for d in (cfg.hidden, cfg.inter, cfg.sh_inter))
          and path in ("auto", "tc"))
    decode = (T <= 4 and cfg.group_size == 64 and cfg.inter == cfg.sh_inter and path in ("auto", "gemv")
              and bh % 128 == 0 and bh // 128 >= 8 and bi % 128 == 0)
    group = ((path == "group" or (path == "auto" and 4 < T and T * cfg.top_k <= 4 * cfg.E))
             and cfg.bits in (4, 8) and cfg.group_size == 64)
    if decode:
        def coalesced(K: int, slots: int, max_warps: int) -> bool:
            # the library's choice (decode.cu dg_supported): 16-byte lanes, a power of two (2..16) per row or
            # whole 512-byte slices, and the CTA's warps within its bound
            lanes = K * cfg.bits // 8 // 16
            ok = (lanes >= 32 and lanes % 32 == 0 and lanes // 32 <= 8) or (2 <= lanes < 32 and lanes & (lanes - 1) == 0)
            return (K % 64 == 0 and ok and slots * max(1, K * cfg.bits // 8 // 512) <= max_warps
                    and os.environ.get("QE_DECODE_V1", "0") in ("", "0"))
        if stage == "gateup":
            return (f"dg_gateup_kernel<{cfg.bits}>" if coalesced(cfg.hidden, 2, 12)
                    else f"decode_gateup_kernel<{cfg.bits}>")
        return (f"dg_down_kernel<{cfg.bits}>" if coalesced(cfg.inter, cfg.top_k + 1, 18)
                else f"decode_down_combine_kernel<{cfg.bits}>")
    if group:
        return f"gm_kernel<{cfg.bits},{'true' if stage == 'gateup' else 'false'}>"
    if tc:
        return f"tc_expert_kernel<{cfg.bits},{2 if stage == 'gateup' else 1}>"
    return f"expert_kernel<{cfg.bits},{cfg.group_size},{stage}>"


def fused_decode(cfg, T: int) -> bool:
    """Whether the library runs the decode step as one cooperative launch (decode_fused_kernel): with
    QE_DECODE_FUSED=1, for decode GEMV shapes, up to 4 tokens, fp32 router, top_k <= 15."""
    if os.environ.get("QE_DECODE_FUSED", "0") != "1" or os.environ.get("QE_EXPERT_PATH", "auto") not in ("auto", "gemv"):
        return False
    return expert_kernel_name(cfg, "gateup", T).startswith("decode_") and cfg.top_k <= 15


def stage_bytes(cfg, uniq: int, T: int) -> dict:
    """Algorithmic bytes per launch of each expert kernel: every active expert's weights once, plus the
    activations the kernel must read and write (fp32)."""
    def q(rows, cols):
        return rows * cols * cfg.bits // 8 + 4 * rows * (cols // cfg.group_size)
    npair = T * (cfg.top_k + 1)
    I = max(cfg.inter, cfg.sh_inter)
    gu = uniq * 2 * q(cfg.inter, cfg.hidden) + 2 * q(cfg.sh_inter, cfg.hidden) + 4 * T * cfg.hidden + 4 * npair * I
    dn = uniq * q(cfg.hidden, cfg.inter) + q(cfg.hidden, cfg.sh_inter) + 4 * npair * I + 4 * npair * cfg.hidden
    return {"gateup": gu, "down": dn}


def ep_roofline(cfg, models, x, stream, rank, world, peak, peak_source, mode, placement=None, spare=0, nprof=10):
    """Per-phase times of the expert-parallel step (CUDA events between phases, a separate run after the
    timed region) and the roofline of its expert stage: this rank's touched experts' weights once, plus the
    rows it receives and the partial sums it returns. With the assignments every rank serves under the
    placement used and under contiguous ranges (the busiest rank sets the step's time)."""
    import torch
    from qmoe.placement import Placement
    names = ("route", "pack", "dispatch", "experts", "return", "combine")
    acc = dict.fromkeys(names, 0.0)
    for i in range(nprof):
        evs = []
        e_start = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)

        def mark(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            evs.append((name, ev))
        models[i % len(models)].forward(x, mode=mode, mark=mark)
        torch.cuda.synchronize()
        prev = e_start
        for name, ev in evs:
            acc[name] += prev.elapsed_time(ev)
            prev = ev
    phase_ms = {k: v / nprof for k, v in acc.items()}
    # experts of this rank touched by any rank's tokens
    idx, _ = models[0].engine.block.route(x.cpu().numpy())
    allidx = torch.empty(world * idx.size, dtype=torch.int32, device="cuda")
    torch.distributed.all_gather_into_tensor(allidx, torch.from_numpy(idx.reshape(-1)).cuda())
    ids = allidx.cpu().numpy().reshape(-1, cfg.top_k)
    by_src = ids.reshape(world, -1, cfg.top_k)
    used = placement or Placement.contiguous(cfg.E, world)
    local = np.concatenate([used.dest(by_src[s], s) for s in range(world)]) == rank
    uniq = len(np.unique(ids[local]))
    loads = used.rank_loads(by_src)
    plain = Placement.contiguous(cfg.E, world).rank_loads(by_src)
    rows, pairs = int(local.any(axis=1).sum()), int(local.sum())   # rows received, (row, expert) pairs
    H, I = cfg.hidden, cfg.inter
    # weights of the touched experts once; x rows in, partial rows out; h3 written and read; y per pair
    nbytes = uniq * cfg.expert_bytes + 8 * rows * H + 8 * pairs * I + 4 * pairs * H
    G, T = world, cfg.tokens
    if mode == "p2p" and (G + 1) * T <= models[0].engine.block.cfg.max_tokens:
        # the shared expert on this rank's own T rows runs in the same launches (qe_moe_ep_route_p2p)
        nbytes += cfg.shared_bytes + 8 * T * H + 8 * T * cfg.sh_inter + 4 * T * H
    achieved = nbytes / (phase_ms["experts"] / 1e3) / 1e9
    xbytes = (G - 1) * T * (4 * H + 8 * cfg.top_k)   # rows + slot lists sent to the other ranks (padded blocks)
    return {"bound": "hbm", "kernel": f"expert stage (qe_moe_ep_experts_{'p2p' if mode == 'p2p' else 'device'}) on rank {rank}", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": None, "peak_source": peak_source,
            "algorithmic_bytes_per_launch": nbytes, "unique_local_experts": uniq,
            "rank_assignments": {"placement": "planned" if placement is not None else "contiguous",
                                 "spare_slots_per_rank": spare,
                                 "replicated_experts": int((used.nrep > 1).sum()),
                                 "per_rank": loads.tolist(), "max_over_mean": float(loads.max() / loads.mean()),
                                 "contiguous_per_rank": plain.tolist(),
                                 "contiguous_max_over_mean": float(plain.max() / plain.mean())},
            "phase_ms": {k: round(v, 5) for k, v in phase_ms.items()},
            "exchange": {"bytes_sent_per_rank_each_way": xbytes,
                         "dispatch_GBs": xbytes / (phase_ms["dispatch"] / 1e3) / 1e9 if phase_ms["dispatch"] else None,
                         "return_GBs": (G - 1) * T * 4 * H / (phase_ms["return"] / 1e3) / 1e9
                         if phase_ms["return"] else None}}


def sub_record(cfg, device, stream, args, nblocks=4, steps=None, warmup=5):
    """One configuration measured like the headline (1 GPU, CUDA-graph replay of one block's forward per step,
    nblocks blocks with distinct weights rotated, inputs in HBM, CUDA events on the launching stream), with the
    roofline of the whole step and of its dominant kernel: HBM bytes for decode batches, tensor flops for prefill.
    Stage times come from an eager, untimed repeat of the same forwards (qe_profile_begin/end)."""
    import torch
    import qmoe
    T = cfg.tokens
    steps = steps or (200 if T <= 64 else 40)
    blocks = [qmoe.MoeBlock(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, cfg.group_size,
                            max_tokens=T, device=device, seed=b + 1, block=b) for b in range(nblocks)]
    gen = torch.Generator(device="cuda").manual_seed(17)
    x = torch.randn(T, cfg.hidden, device="cuda", generator=gen, dtype=torch.float32)
    out = torch.empty_like(x)
    sptr = stream.cuda_stream
    graphs = [b.graph(T, x.data_ptr(), out.data_ptr()) for b in blocks]
    for i in range(max(warmup, 3)):
        graphs[i % nblocks].launch(sptr)
    torch.cuda.synchronize()
    l0 = qmoe.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        graphs[i % nblocks].launch(sptr)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = qmoe.kernel_launches() - l0
    ms = e0.elapsed_time(e1) / steps
    qmoe.profile_begin(device)
    for i in range(min(steps, 40)):
        blocks[i % nblocks].forward_device(T, x.data_ptr(), out.data_ptr(), sptr)
    torch.cuda.synchronize()
    stage_ms, passes = qmoe.profile_end(device)
    per_pass = {k: v / max(passes, 1) for k, v in stage_ms.items()}
    idx, _ = blocks[0].route(x.cpu().numpy())
    uniq = len(np.unique(idx))
    for g in graphs:
        g.close()
    for b in blocks:
        b.close()
    value = T / (ms / 1e3)
    top = max(("gateup", "down"), key=lambda k: per_pass[k])
    kname = expert_kernel_name(cfg, top, T)
    rec = {"config": cfg.name, "workload": cfg.note, "tokens_per_step": T, "value": value, "unit": "tokens/s",
           "ms_per_step": ms, "steps": steps, "blocks_rotated": nblocks, "cuda_graph": True,
           "gpu_launches": launches, "unique_experts": uniq,
           "stage_ms_per_pass": {k: round(v, 5) for k, v in per_pass.items()}}
    if T <= 64:   # decode batches: HBM-bound; compulsory bytes of the step and of the dominant kernel
        peak, kind = hbm_peak()
        step_bytes = (uniq * cfg.expert_bytes + cfg.shared_bytes + 4 * (cfg.E + 1) * cfg.hidden
                      + 8 * T * cfg.hidden)
        kb = stage_bytes(cfg, uniq, T)[top]
        kms = per_pass[top]
        rec["roofline"] = {"bound": "hbm", "unit": "GB/s", "peak": peak,
                           "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured"
                           else "fallback 6.65 TB/s",
                           "step": {"algorithmic_bytes": step_bytes, "achieved": step_bytes / (ms / 1e3) / 1e9,
                                    "frac": step_bytes / (ms / 1e3) / 1e9 / peak},
                           "kernel": kname, "kernel_ms": kms, "algorithmic_bytes_per_launch": kb,
                           "achieved": kb / (kms / 1e3) / 1e9, "frac": kb / (kms / 1e3) / 1e9 / peak}
    else:         # prefill: tensor-bound; algorithmic flops (the 2-term activation split is not counted)
        peak, kind = tensor_peak()
        step_flops = T * cfg.flops_per_token()
        npair = T * (cfg.top_k + 1)
        kf = (4 if top == "gateup" else 2) * npair * cfg.inter * cfg.hidden
        kms = per_pass[top]
        rec["roofline"] = {"bound": "tensor", "unit": "TFLOP/s", "peak": peak, "peak_source": kind,
                           "step": {"algorithmic_flops": step_flops, "achieved": step_flops / (ms / 1e3) / 1e12,
                                    "frac": step_flops / (ms / 1e3) / 1e12 / peak},
                           "kernel": kname, "kernel_ms": kms, "algorithmic_flops_per_launch": kf,
                           "achieved": kf / (kms / 1e3) / 1e12, "frac": kf / (kms / 1e3) / 1e12 / peak}
    return rec


def tensor_peak():
    """Dense bf16 tensor peak for a kernel timed inside a long step: the sustained figure of MEASURED_PEAKS.json,
    else the profiling recipe's fallback."""
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["bf16_tflops_sustained"]), "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    except Exception:
        return 1400.0, "fallback 1.4 PFLOP/s sustained"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--blocks", type=int, default=4)
    ap.add_argument("--stack", action="store_true",
                    help="one step = one forward of every block of the configuration's stack (c4: 40, c5: 48 "
                         "independent blocks, each fed the step's tokens); value = tokens through the stack per s")
    ap.add_argument("--ref-tokens", type=int, default=16)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="config c2 on 1 GPU: skip the decode and compute-bound prefill sub-records")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="1 GPU: replay each block's forward as a captured CUDA graph (qe_moe_graph_create; auto: "
                         "on) or launch its kernels one by one (off)")
    ap.add_argument("--ep-mode", default="p2p", choices=["p2p", "sharded"],
                    help="N > 1: exchange through peer memory (p2p) or NCCL all_to_all (sharded)")
    ap.add_argument("--placement", default="auto", choices=["auto", "contiguous", "planned"],
                    help="N > 1: experts in contiguous ranges per rank, or a placement planned from a calibration "
                         "batch's routing with hot experts replicated into spare slots (auto: planned when the "
                         "configuration's routing is skewed)")
    ap.add_argument("--spare-slots", type=int, default=-1,
                    help="planned placement: replica slots per rank beyond E/N (default E/N/8, at least 1)")
    args = ap.parse_args()

    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        run_reference_arm(args, cfg)
        return

    import torch
    import qmoe
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    T = cfg.tokens
    ep = world > 1
    if args.stack:
        args.blocks = cfg.blocks
    gen = torch.Generator(device="cuda").manual_seed(7 + rank)
    x = torch.randn(T, cfg.hidden, device="cuda", generator=gen, dtype=torch.float32)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    use_graph = False
    graph_launches = [0]   # kernels launched by replays of torch-captured graphs (not seen by the library)
    if ep:
        from qmoe.ep import ExpertParallelMoe
        planned = args.placement == "planned" or (args.placement == "auto" and cfg.zipf_s > 0)
        spare = args.spare_slots if args.spare_slots >= 0 else max(1, cfg.E // world // 8)
        placements = []
        for b in range(args.blocks):
            if planned:   # calibration tokens: a batch distinct from the timed one, on every rank
                xc = torch.randn(T, cfg.hidden, device="cuda", generator=torch.Generator(device="cuda").manual_seed(
                    1000 + 7 * b + rank))
                placements.append(ExpertParallelMoe.plan_placement(cfg, rank, world, local, xc, spare, seed=b + 1,
                                                                   block=b, router_bias=router_bias(cfg, b + 1)))
            else:
                placements.append(None)
        models = [ExpertParallelMoe.on_gpu(cfg, rank, world, local, seed=b + 1, block=b, max_tokens=(world + 1) * T,
                                           router_bias=router_bias(cfg, b + 1), placement=placements[b])
                  for b in range(args.blocks)]
        if args.ep_mode == "p2p":
            for mdl in models:
                mdl.enable_p2p(T)
        blocks = [m.engine.block for m in models]

        def step(i):
            if args.stack:
                for mdl in models:
                    mdl.forward(x, mode=args.ep_mode)
            else:
                models[i % len(models)].forward(x, mode=args.ep_mode)

        if args.ep_mode == "p2p" and args.graph in ("on", "auto"):
            # the peer-memory step holds only this library's kernels (the barriers are qe_ep_xchg_barrier): after
            # two eager passes (buffers and kernel attributes in place), each block's step is captured once and
            # replayed; the kernels a replay launches are counted from the capture
            for _ in range(2):
                for mdl in models:
                    mdl.forward(x, mode="p2p")
            torch.cuda.synchronize()
            torch.distributed.barrier()
            ep_graphs = []
            for mdl in models:
                l0 = qmoe.kernel_launches()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    g_out = mdl.forward(x, mode="p2p")
                ep_graphs.append((g, g_out, qmoe.kernel_launches() - l0))
            torch.cuda.synchronize()
            use_graph = True
            eager_step = step

            def step(i):
                for g, _, n in (ep_graphs if args.stack else [ep_graphs[i % len(ep_graphs)]]):
                    g.replay()
                    graph_launches[0] += n
    else:
        blocks = [qmoe.MoeBlock(cfg.hidden, cfg.E, cfg.top_k, cfg.inter, cfg.sh_inter, cfg.bits, cfg.group_size,
                                max_tokens=T, device=local, seed=b + 1, block=b, router_bias=router_bias(cfg, b + 1))
                  for b in range(args.blocks)]

        def step(i):
            if args.stack:
                for b in blocks:
                    b.forward_device(T, x.data_ptr(), out.data_ptr(), sptr)
            else:
                blocks[i % len(blocks)].forward_device(T, x.data_ptr(), out.data_ptr(), sptr)

        use_graph = args.graph in ("on", "auto")
        if use_graph:   # one captured forward per block, replayed (no per-kernel host launch cost)
            graphs = [b.graph(T, x.data_ptr(), out.data_ptr()) for b in blocks]
            eager_step = step

            def step(i):
                if args.stack:
                    for g in graphs:
                        g.launch(sptr)
                else:
                    graphs[i % len(graphs)].launch(sptr)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)   # sampled from here to the end: warm-up, timed steps, e2e and sub-records
    clocks.mark("warmup", True)
    for i in range(max(args.warmup, 3)):
        step(i)
    barrier()
    clocks.mark("warmup", False)
    launches0 = qmoe.kernel_launches() + graph_launches[0]
    qmoe.profile_begin(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark("timed", True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    barrier()
    clocks.mark("timed", False)
    launches = qmoe.kernel_launches() + graph_launches[0] - launches0
    stage_ms, passes = qmoe.profile_end(local)
    if not ep and use_graph:   # graphs carry no stage events: profile the same forwards eagerly, untimed
        qmoe.profile_begin(local)
        for i in range(min(args.steps, 50)):
            eager_step(i)
        torch.cuda.synchronize()
        stage_ms, passes = qmoe.profile_end(local)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * T * args.steps / (ms_max / 1e3)

    # end to end through the public host-buffer call: pinned host x in, host out back, every step
    xh = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(11 + rank)).pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xn, on = xh.numpy(), oh.numpy()
    ke = max(10, min(args.steps, 200)) if not args.stack else 5

    def e2e_step(i):
        sel = range(len(blocks)) if args.stack else [i % len(blocks)]
        for bi in sel:
            if ep:   # qmoe.ep.ExpertParallelMoe.forward with the copies in and out of pinned host memory
                xd = xh.to("cuda", non_blocking=True)
                oh.copy_(models[bi].forward(xd, mode=args.ep_mode), non_blocking=True)
                torch.cuda.current_stream().synchronize()
            else:    # qe_moe_forward: host buffers in and out
                blocks[bi].forward(xn, on)

    # pipelined: the same public calls with step i+1's input copy and step i-1's output copy running under step
    # i's kernels (1 GPU: qe_moe_forward_async; N GPUs: copy streams around qmoe.ep.ExpertParallelMoe.forward)
    copy_in, copy_out = torch.cuda.Stream(), torch.cuda.Stream()
    xd2 = [torch.empty(T, cfg.hidden, device="cuda") for _ in range(2)]
    ev_in, ev_comp = [torch.cuda.Event() for _ in range(2)], [torch.cuda.Event() for _ in range(2)]
    n_async = [0]
    e2e_graphs, ev_out, out_used = {}, {}, set()
    if ep and use_graph:   # the captured step per block and input slot (as the timed steps replay theirs)
        for bi, mdl in enumerate(models):
            for j in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    g_out = mdl.forward(xd2[j], mode="p2p")
                e2e_graphs[(bi, j)] = (g, g_out)
                ev_out[(bi, j)] = torch.cuda.Event()
        torch.cuda.synchronize()

    def e2e_async_step(i):
        sel = range(len(blocks)) if args.stack else [i % len(blocks)]
        for bi in sel:
            if ep:
                j = n_async[0] & 1
                cur = torch.cuda.current_stream()
                if n_async[0] >= 2:
                    copy_in.wait_event(ev_comp[j])     # slot j's input was read by its forward
                with torch.cuda.stream(copy_in):
                    xd2[j].copy_(xh, non_blocking=True)
                    ev_in[j].record(copy_in)
                cur.wait_event(ev_in[j])
                if e2e_graphs:
                    g, o = e2e_graphs[(bi, j)]
                    if (bi, j) in out_used:
                        cur.wait_event(ev_out[(bi, j)])   # the last copy of this graph's output has finished
                    g.replay()
                else:
                    o = models[bi].forward(xd2[j], mode=args.ep_mode)
                ev_comp[j].record(cur)
                copy_out.wait_event(ev_comp[j])
                with torch.cuda.stream(copy_out):
                    oh.copy_(o, non_blocking=True)
                    if e2e_graphs:
                        ev_out[(bi, j)].record(copy_out)
                        out_used.add((bi, j))
                if not e2e_graphs:
                    o.record_stream(copy_out)
                n_async[0] += 1
            else:
                blocks[bi].forward_async(xn, on)

    def e2e_async_wait():
        if ep:
            copy_out.synchronize()
            torch.cuda.current_stream().synchronize()
        else:
            blocks[0].wait()

    def timed_e2e(run, wait=None):
        # warm-up: every block at least twice (each block's first pipelined call captures its CUDA graph); a
        # --stack step already runs every block
        for i in range(3 if args.stack else max(3, 2 * len(blocks) + 1)):
            run(i)
        if wait:
            wait()
        barrier()
        t0 = time.perf_counter()
        for i in range(ke):
            run(i)
        if wait:
            wait()
        barrier()
        te = torch.tensor([time.perf_counter() - t0], device="cuda")
        if world > 1:
            torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        return world * T * ke / float(te.item())

    clocks.mark("e2e", True)
    e2e_sync_value = timed_e2e(e2e_step)
    e2e_value = timed_e2e(e2e_async_step, e2e_async_wait)
    clocks.mark("e2e", False)

    peak, peak_kind = hbm_peak()
    peak_source = (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s")
    if ep:
        roofline = ep_roofline(cfg, models, x, stream, rank, world, peak, peak_source, args.ep_mode, placements[0],
                               spare if planned else 0)
    else:
        # roofline of the dominant kernel (per-stage CUDA events recorded inside the timed region)
        idx, _ = blocks[0].route(x.cpu().numpy())
        uniq = len(np.unique(idx))
        sb = stage_bytes(cfg, uniq, T)
        total_stage = sum(stage_ms.values())
        if fused_decode(cfg, T):
            # fused decode step: one kernel (router, top-k, gate/up, down + combine); its compulsory bytes are
            # the router, every selected expert and the shared expert once, x in and out back
            top = "router"
            sb = {"router": 4 * (cfg.E + 1) * cfg.hidden + uniq * cfg.expert_bytes + cfg.shared_bytes
                  + 8 * T * cfg.hidden}
            kname, kdesc = f"decode_fused_kernel<{cfg.bits}>", " (whole decode step, one cooperative launch)"
        else:
            top = max(("gateup", "down"), key=lambda s: stage_ms[s])
            kname = expert_kernel_name(cfg, top, T)
            kdesc = " (gate/up + SwiGLU)" if top == "gateup" else " (down)"
        per_launch_ms = stage_ms[top] / max(passes, 1)
        achieved = sb[top] / (per_launch_ms / 1e3) / 1e9
        tr = profiled_traffic(kname, cfg.name)
        roofline = {"bound": "hbm", "kernel": kname + kdesc,
                    "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": tr[0] if tr else None,
                    "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/{tr[1]}" if tr
                    else "no ncu capture committed for this kernel and config",
                    "peak_source": peak_source, "algorithmic_bytes_per_launch": sb[top], "unique_experts": uniq,
                    "stage_share": {k: round(v / total_stage, 4) for k, v in stage_ms.items()},
                    "stage_ms_per_pass": {k: round(v / max(passes, 1), 5) for k, v in stage_ms.items()}}

    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(cfg, world, args.blocks, "rows and partial sums stored into peer memory by "
                                      "the kernels" if args.ep_mode == "p2p" else "all_to_all over NCCL", args.stack),
            "cuda_graph": use_graph,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 4 * T * cfg.hidden,
                    "d2h_bytes_per_step": 4 * T * cfg.hidden, "steps": ke,
                    "timing": "host clock, max over ranks; consecutive steps pipelined: each step's pinned-host "
                              "input copy and output copy run under its neighbours' kernels "
                              + ("(copy streams around ExpertParallelMoe.forward, replayed from CUDA graphs when the "
                                 "timed steps are)" if ep else "(qe_moe_forward_async)"),
                    "sync_value": e2e_sync_value,
                    "sync_timing": "one step at a time: copy in, forward, copy out, wait"
                                   + (" (ExpertParallelMoe.forward)" if ep else " (qe_moe_forward)")},
            "roofline": roofline, "gpu_launches": launches}
    if ep:
        line["config"]["placement"] = (f"planned per block from a calibration batch's routing (qmoe.placement): "
                                       f"{cfg.E // world + spare} expert slots per rank, hot experts replicated"
                                       if planned else f"contiguous: {cfg.E // world} experts per rank")
    if args.stack:   # every token passes through all blocks of the stack: block-level throughput for reference
        line["block_tokens_per_s"] = value * args.blocks
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = time_reference(cfg, 1, args.ref_tokens, 1000, 1, os.cpu_count() or 1, budget_s=args.cpu_budget)
        if cb and args.stack:   # one block timed; a token through the stack takes `blocks` such passes
            cb["value"] /= args.blocks
            cb["sample"] += f"; one block timed, value divided by the stack's {args.blocks} blocks"
        if cb:
            cb.update(host_cpu())
            if not args.stack:
                mr = time_reference_mode_r(cfg, 1, args.ref_tokens, os.cpu_count() or 1)
                if mr:
                    cb["mode_r"] = mr
        line["cpu_baseline"] = cb if cb else {"value": None, "unavailable": "oracle/_ref missing"}
    if world == 1 and not args.stack and args.config == "c2" and not args.no_sub_records:
        # the other headline measurements in the same run: decode (config 1 at one token, one config-5 block at 64
        # tokens) and compute-bound prefill (config 3 at 4096 tokens); each on its own rotated blocks
        for b in blocks:
            b.close()
        if use_graph:
            for g in graphs:
                g.close()
            use_graph = False
        blocks = []
        line["sub_records"] = {}
        for name, key in (("decode_c1", "c1"), ("decode_c5_block", "c5"), ("prefill_compute_c3", "c3_prefill")):
            clocks.mark(name, True)
            line["sub_records"][name] = sub_record(CONFIGS[key], local, stream, args)
            clocks.mark(name, False)
        line["gpu_launches"] += sum(r["gpu_launches"] for r in line["sub_records"].values())
    line["clocks"] = clocks.stop()
    if ep:
        if use_graph:   # the captured steps reference the exchange buffers: drop them before those are freed
            torch.cuda.synchronize()
            ep_graphs.clear()
            e2e_graphs.clear()
        for mdl in models:
            mdl.close()
    elif use_graph:
        for g in graphs:
            g.close()
    for b in blocks:
        b.close()
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
