#!/usr/bin/env python
"""Benchmark of the B200 sparse-KV decode path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3]
                  [--impl ours|reference] [--shard auto|heads|seqs]

A step is one decode step of the workload: for every (sequence, layer)
append the token's K/V, score + select blocks per KV head, attend over the
selected blocks plus the open tail, and seal the tail when it holds 32
tokens (rebuilding the sealed block's representative). The default workload
is the path's target configuration: Qwen3-8B shape (32 query / 8 KV heads,
head_dim 128, 36 layers), one sequence of 32K context (1024 blocks), 4096-token
budget (1 init + 4 local + 123 dynamic blocks). Every open tail starts with
the tokens that make the last timed step a seal step, so the timed window
always holds at least one seal and representative rebuild.

Multi-GPU (N > 1, one process per GPU): a single-sequence config is split by
KV head (rank r holds KH/N heads of every layer), and each step's per-head
outputs are gathered by the attention kernel's peer-memory stores over NVLink
(--gather nccl: an NCCL all-gather after the step): strong scaling, value =
steps/s of the one sequence. A batched config (cfg4) is split by sequence
(no data-path collective): weak scaling. With --shard heads at N > 1 the line
also carries `replicas`: every rank decoding its own whole sequence.

`value` is device-timed with inputs resident in HBM, the timed steps replayed
from one recorded CUDA graph (`--launch eager` issues one call per step); `e2e`
runs the same steps through the public host-buffer call (sa_ctx_step_host:
H2D of the step's query + new K/V, step, D2H of the output, synchronize).
`--impl reference` times the reference's own CPU implementation (its C++
selector, packed gather, attention and seal-time representative rebuild,
compiled from its sources into oracle/_ref) on the host's cores, on the same
seeded inputs (generated on GPU 0 with the same generator calls, then
copied to the host), over a bounded sample of the step's units.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "sparse decode attn steps/s + selected-KV HBM GB/s (% of peak) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
SEED = 1


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", default="cfg3", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--shard", default="auto", choices=["auto", "heads", "seqs"],
                    help="N > 1: split one sequence's KV heads over the ranks (heads; the "
                         "single-sequence configs' default) or give each rank its own "
                         "sequences (seqs; the batched config's default)")
    ap.add_argument("--kernel-iters", type=int, default=50)
    ap.add_argument("--launch", default="graph", choices=["graph", "eager"],
                    help="timed steps replayed from one recorded CUDA graph (sa_ctx_graph_*) "
                         "or launched one call at a time; the NCCL gather runs eager")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-replicas", action="store_true",
                    help="skip the per-rank whole-sequence replica run of a KV-head split")
    ap.add_argument("--cpu-seconds", type=float, default=8.0,
                    help="host time of each cpu_baseline timing (1 thread, all cores)")
    ap.add_argument("--ref-seconds", type=float, default=40.0,
                    help="--impl reference: host time budget of each of its two timings")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="KV-head split: gather the per-head outputs with peer-memory stores "
                         "from the attention kernel (p2p) or an NCCL all-gather after it")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the workload's layer count (small profiling cases)")
    ap.add_argument("--rank-share", type=int, default=1,
                    help="on one GPU, run rank 0's share of an N-GPU KV-head split (its KV "
                         "heads of every layer, no gather): the per-rank work of --gpus N")
    ap.add_argument("--probe-streaming", action="store_true",
                    help="instead of the decode step: stream random 16 KB pool entries into "
                         "shared memory with per-lane cp.async and with bulk copies "
                         "(sa_probe_stream) and print the GB/s of each")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(kernel: str, workload: str, bytes_per_launch: int | None = None):
    """DRAM bytes per launch from an ncu capture recorded in profiles/, or None.

    A profile line reads `traffic_per_launch[kernel@workload]: T` or
    `... : T per A algorithmic bytes`; with A given, T is scaled to
    bytes_per_launch (traffic grows in proportion to the blocks processed)."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        text = f.read_text()
        m = re.search(rf"traffic_per_launch\[{re.escape(kernel)}@{re.escape(workload)}\]:\s*([0-9.]+)"
                      rf"(?:\s+per\s+([0-9.]+)\s+algorithmic bytes)?", text)
        if m:
            traffic = float(m.group(1))
            if m.group(2) and bytes_per_launch:
                traffic *= bytes_per_launch / float(m.group(2))
            return traffic
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def wait_first(self, timeout: float = 10.0) -> None:
        """Block until nvidia-smi has printed its first row (its start-up can
        take longer than a short timed region)."""
        self.first = ""
        if self.proc is None or self.proc.stdout is None:
            return
        import select

        ready, _, _ = select.select([self.proc.stdout], [], [], timeout)
        if ready:
            self.first = self.proc.stdout.readline()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        out = getattr(self, "first", "") + (out or "")
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------ layout, config

def job_layout(args, w, world: int, rank: int):
    """(shard, kv_heads_slice, seq_offset) of this rank: 'single' at N = 1,
    'heads' (one sequence's KV heads split over the ranks) or 'seqs' (each
    rank its own sequences of the batch)."""
    from solidattention_repro_b200 import sharding

    if world == 1:
        if getattr(args, "rank_share", 1) > 1:
            return "share", sharding.shard_kv_heads(w.kv_heads, args.rank_share, 0), 0
        return "single", None, 0
    shard = args.shard
    if shard == "auto":
        shard = "seqs" if w.batch > 1 else "heads"
    if shard == "heads":
        return "heads", sharding.shard_kv_heads(w.kv_heads, world, rank), 0
    return "seqs", None, rank * w.seqs


def job_config(args, w, world: int, shard: str, initial_tail: int) -> dict:
    """The workload both arms run (identical keys and values in both lines)."""
    seqs_total = w.seqs * (world if shard == "seqs" else 1)
    if shard == "heads":
        par = (f"kv-head-split x{world}, outputs gathered every step by "
               + ("the attention kernel's peer-memory stores (NVLink P2P)" if args.gather == "p2p"
                  else "an NCCL all-gather"))
    elif shard == "seqs":
        par = f"sequence-split x{world}, no data-path collective"
    elif shard == "share":
        par = (f"one rank's share of a kv-head split x{args.rank_share} "
               f"(rank 0's KV heads, no gather), on one GPU")
    else:
        par = "single"
    return {
        "workload": w.name, "layers": w.layers, "query_heads": w.query_heads,
        "kv_heads": w.kv_heads, "head_dim": 128, "context_tokens": w.context_blocks * 32,
        "context_min_tokens": (w.context_min_blocks or w.context_blocks) * 32,
        "budget_blocks": w.budget_blocks, "init_blocks": w.init_blocks,
        "local_blocks": w.local_blocks, "hot_blocks": w.hot_blocks, "seqs": seqs_total,
        "tail_tokens_at_start": initial_tail, "parallelism": par,
        "l2": "inputs larger than L2: each step reads its selected KV and all representatives "
              f"({(w.selected_kv_bytes() + w.rep_bytes()) / 1e9:.2f} GB per step at full context)",
        "kv_dtype": "fp16", "accumulate": "fp32", "seed": SEED,
    }


# ------------------------------------------------------------ CPU path (reference's own C++)

def cpu_lib():
    import oracle

    ref = oracle.reference()
    return (ref, "reference") if ref is not None else (oracle.port(), "port")


class HostSeqLayer:
    """One (sequence, layer) of the decode state on the host, in the
    reference's token-major layout: sealed blocks in logical order followed
    by the open tail block, representatives [QH][nb][D], the tail's queries."""

    def __init__(self, blocks, nb, reps, tail_len, ring, extra_blocks: int):
        kh_row = blocks.shape[1:]
        self.blocks = np.zeros((nb + 1 + extra_blocks,) + tuple(kh_row), np.uint16)
        self.blocks[:nb + 1] = blocks[:nb + 1]
        self.nb = nb
        self.reps = np.ascontiguousarray(reps, np.float32)
        self.tail_len = tail_len
        self.ring = np.ascontiguousarray(ring, np.float32)  # [QH][32][D]

    def append(self, q, kv_row):
        """The step's token: its K/V row into the tail block, its queries into
        the ring (a host copy; the reference's store write is host I/O)."""
        self.blocks[self.nb, self.tail_len] = kv_row
        self.ring[:, self.tail_len] = q
        self.tail_len += 1

    def seal(self, lib, qh, kh):
        """The tail holds 32 tokens: rebuild its representative with the
        reference's build over the tail's own queries (T = 32), as the online
        seal does; returns the rebuild's host seconds."""
        t0 = time.perf_counter()
        values, _ = lib.build_representatives(self.ring, self.blocks[self.nb], 32, qh, kh, 128, 32,
                                              32, 4)
        dt = time.perf_counter() - t0
        self.reps = np.ascontiguousarray(np.concatenate([self.reps, values], axis=1))
        self.nb += 1
        self.tail_len = 0
        return dt


class UnitSet:
    """ctypes Unit array over (state, KV head) pairs in (state, head) order,
    with the id and output arrays it points to (kept alive here); the states'
    blocks and `queries` [n_states][QH][D] stay owned by the caller."""

    def __init__(self, oracle_mod, states, queries, kh, grp, budget, n=None):
        pairs = [(i, h) for i in range(len(states)) for h in range(kh)]
        self.pairs = pairs[:n] if n else pairs
        self.states = states
        self.units = (oracle_mod.Unit * len(self.pairs))()
        self.ids = np.zeros((len(self.pairs), budget), np.int64)
        self.out = np.zeros((len(self.pairs), grp, 128), np.float32)
        for k, (i, h) in enumerate(self.pairs):
            u = self.units[k]
            u.blocks = states[i].blocks.ctypes.data
            u.query = queries[i].ctypes.data
            u.kv_head = h
            u.ids_out = self.ids[k].ctypes.data
            u.out = self.out[k].ctypes.data

    def refresh(self):
        """Point every unit at its state's current block count, tail length
        and representatives."""
        for k, (i, _) in enumerate(self.pairs):
            st = self.states[i]
            self.units[k].reps = st.reps.ctypes.data
            self.units[k].nb = st.nb
            self.units[k].tail_len = st.tail_len

    def run(self, lib, w, qh, kh, threads) -> float:
        """Host seconds of the reference path over these units."""
        t0 = time.perf_counter()
        lib.sparse_units(self.units, qh, kh, 128, w.budget_blocks, w.init_blocks, w.local_blocks,
                         np.float32(1.0) / np.sqrt(np.float32(128)), threads)
        return time.perf_counter() - t0


def host_states_from_ctx(ctx, sls):
    """HostSeqLayer copies of the context's current state for sequence-layers
    `sls`: sealed blocks through the table, the open tail, representatives,
    the query ring."""
    nb_all = ctx.num_sealed.cpu().numpy()
    tables = ctx.table.cpu().numpy()
    tails = ctx.tail_block.cpu().numpy()
    tl_all = ctx.tail_len.cpu().numpy()
    states = []
    for sl in sls:
        nb = int(nb_all[sl])
        phys = np.concatenate([tables[sl, :nb], tails[sl:sl + 1]]).astype(np.int64)
        blocks = ctx.read_blocks(phys).cpu().numpy().view(np.uint16)
        reps = ctx.reps[sl, :, :, :nb].permute(0, 2, 1).contiguous().cpu().numpy()
        ring = ctx.query_ring[sl].cpu().numpy()
        states.append(HostSeqLayer(blocks, nb, reps, int(tl_all[sl]), ring, 0))
    return states


def run_cpu_baseline(ctx, w, q_step, seconds, cores):
    """The reference's CPU path (its selector per KV head, packed gather and
    attention, compiled from its sources) on the GPU context's current state
    and query: all cores over 4 sequence-layers, one thread over 4 units;
    each extrapolated to the whole step. Also checks that the CPU's selected
    ids equal the GPU's on the sampled units."""
    import oracle

    lib, kind = cpu_lib()
    sls = list(range(min(4, ctx.num_sl)))
    ctx.select(q_step)
    sel = ctx.selected.cpu().numpy()
    counts = ctx.selected_count.cpu().numpy()
    states = host_states_from_ctx(ctx, sls)
    q = q_step.reshape(ctx.num_sl, ctx.qh, 128)[sls].cpu().numpy()
    qs = [np.ascontiguousarray(q[i]) for i in range(len(sls))]
    grp = ctx.qh // ctx.kh
    units_total = ctx.num_sl * ctx.kh
    result = {"unit": "steps/s", "kind": kind, "cores": cores}
    match = True
    for label, threads, n in (("all", cores, None), ("1thread", 1, 4)):
        us = UnitSet(oracle, states, qs, ctx.kh, grp, w.budget_blocks, n)
        us.refresh()
        times = []
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end or len(times) < 2:
            times.append(us.run(lib, w, ctx.qh, ctx.kh, threads))
        per_step = statistics.median(times) * units_total / len(us.pairs)
        # sequence-steps/s, as the GPU arm counts them
        result[f"steps_per_s_{label}"] = ctx.seqs / per_step
        result[f"runs_{label}"] = len(times)
        ids = us.ids
        for k, (i, h) in enumerate(us.pairs):
            sl = sls[i]
            g = h * ctx.n_groups // ctx.kh
            c = int(counts[sl, g])
            match &= bool(np.array_equal(ids[k, :c], sel[sl, g, :c].astype(np.int64)))
    result["value"] = result["steps_per_s_all"]
    result["ids_match_gpu"] = match
    result["sample"] = (f"the live decode state of {len(sls)} of {ctx.num_sl} sequence-layers "
                        f"({states[0].nb} sealed blocks, tail {states[0].tail_len}): all {cores} "
                        f"threads over their {len(sls) * ctx.kh} (sequence-layer, KV head) units, "
                        f"1 thread over 4 units; medians, extrapolated to the {units_total} units "
                        f"of a step")
    return result


def reference_arm(args, w, rank, world):
    """The reference's own CPU implementation on identical seeded inputs.

    The workload's values come from the same generator calls as the GPU arm
    (torch's CUDA generator on GPU 0, then copied to the host: the data
    generation is not timed and runs none of this repository's kernels).
    Representatives are built on the host by the reference's own function.
    Every step then runs, on host cores, the reference path of a sample of
    the step's (sequence, layer, KV head) units: append the token, select
    per KV head, packed gather, attention, and on the seal step the
    representative rebuild; all cores over the sampled sequence-layers and
    one thread over a subset sized to the time budget, each extrapolated to
    the whole step."""
    if rank != 0:
        return
    import torch

    import oracle
    from solidattention_repro_b200 import workloads

    shard, _, _ = job_layout(args, w, world, 0)
    K, W = args.steps, args.warmup
    total = K + W
    t0 = workloads.tail_for_seal_at_end(K, W)
    lib, kind = cpu_lib()
    cores = os.cpu_count() or 1
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    qh, kh, grp = w.query_heads, w.kv_heads, w.group
    # sampled sequence-layers: spread over the layers (and over the first
    # rank's sequences for a batch), fewer for long contexts (host memory)
    n_sl = max(1, min(4, (4 * 1024) // max(1, w.context_blocks)))
    layers = sorted({round(x) for x in np.linspace(0, w.layers - 1, n_sl)})
    pairs = [(s % w.seqs, l) for s, l in zip(range(len(layers)), layers)]
    setup0 = time.perf_counter()
    info = {"layer_ids": list(range(w.layers))}
    q_base = torch.stack([workloads.base_queries(w, SEED, s, dev) for s in range(w.seqs)])
    info["q_base"] = q_base
    queries, kv_new = workloads.decode_inputs(w, info, total, dev, seed=SEED)
    states, step_q, step_kv = [], [], []
    extra = total // 32 + 2
    for s, layer in pairs:
        nb = w.sequence_blocks(s)
        hot = workloads.hot_blocks(w, SEED, s)
        kv = workloads.prompt_kv(w, SEED, s, layer, q_base[s, layer], hot[layer], dev)
        kv_h = kv.view(torch.int16).cpu().numpy().view(np.uint16).reshape(nb, 32, 2, kh, 128)
        del kv
        pq = workloads.prompt_queries(w, SEED, s, layer, dev).cpu().numpy()
        reps = lib.build_reps_per_block(pq, kv_h, nb, qh, kh, 128, 32, 4, cores)
        del pq
        blocks = np.zeros((nb + 1, 32, 2, kh, 128), np.uint16)
        blocks[:nb] = kv_h
        ring = np.zeros((qh, 32, 128), np.float32)
        st = HostSeqLayer(blocks, nb, reps, 0, ring, extra)
        if t0:
            tq, tkv = workloads.tail_tokens(w, SEED, s, q_base[s], t0, dev)
            tq = tq[:, layer].cpu().numpy()
            tkv = tkv[:, layer].view(torch.int16).cpu().numpy().view(np.uint16)
            for t in range(t0):
                st.append(tq[t], tkv[t])
        states.append(st)
        step_q.append(queries[:, s, layer].cpu().numpy())
        step_kv.append(kv_new[:, s, layer].view(torch.int16).cpu().numpy().view(np.uint16))
    del queries, kv_new
    torch.cuda.synchronize(dev)
    setup_s = time.perf_counter() - setup0
    qbuf = [np.zeros((qh, 128), np.float32) for _ in states]
    set_all = UnitSet(oracle, states, qbuf, kh, grp, w.budget_blocks)
    units_step = w.seqs * w.layers * kh            # units of one sequence-step, per sequence
    sl_step = w.layers                             # sequence-layers per sequence-step
    # one thread over a subset sized to the time budget: calibrate one unit
    for i, st in enumerate(states):
        qbuf[i][:] = step_q[i][0]
    set_cal = UnitSet(oracle, states, qbuf, kh, grp, w.budget_blocks, 1)
    set_cal.refresh()
    unit_s = min(set_cal.run(lib, w, qh, kh, 1) for _ in range(2))
    n1 = int(max(1, min(len(set_all.pairs), args.ref_seconds / max(1e-6, total * unit_s))))
    set_one = UnitSet(oracle, states, qbuf, kh, grp, w.budget_blocks, n1)
    t_all, t_one, t_seal = [], [], []
    for i in range(total):
        for k, st in enumerate(states):
            st.append(step_q[k][i], step_kv[k][i])
            qbuf[k][:] = step_q[k][i]
        set_all.refresh()
        set_one.refresh()
        a = set_all.run(lib, w, qh, kh, cores)
        b = set_one.run(lib, w, qh, kh, 1)
        seal = 0.0
        if states[0].tail_len == 32:
            seal = statistics.mean(st.seal(lib, qh, kh) for st in states)
        if i >= W:
            t_all.append(a)
            t_one.append(b)
            t_seal.append(seal)
    # per sequence-step: unit work scaled from the sample, seal rebuilds of
    # every sequence-layer (spread over the cores in the all-core figure)
    per_units_all = statistics.mean(t_all) * (w.layers * kh) / len(set_all.pairs)
    per_units_one = statistics.mean(t_one) * (w.layers * kh) / len(set_one.pairs)
    seal_mean = statistics.mean(t_seal) if t_seal else 0.0
    step_all = per_units_all + seal_mean * sl_step / min(cores, sl_step)
    step_one = per_units_one + seal_mean * sl_step
    value = 1.0 / step_all
    seals = workloads.seal_steps(t0, W, K)
    sample = (f"per step, {len(states)} sequence-layers of the workload (layers {layers}, "
              f"{states[0].nb} sealed blocks at the end): append, select per KV head, packed "
              f"gather and attention of their {len(set_all.pairs)} units on all {cores} threads and of "
              f"{n1} of them on 1 thread, and the reference's representative rebuild on the "
              f"{seals} seal step(s); extrapolated to the {units_step} units and {sl_step} "
              f"sequence-layers of a sequence-step; inputs generated on GPU 0 by the GPU arm's "
              f"generator calls ({setup_s:.1f} s of setup, not timed)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": 1000.0 / value,
        "higher_is_better": True, "scaling": "weak" if shard == "seqs" else "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded FP16 N(0,1) KV with planted hot blocks, seeded queries "
                "(identical to the GPU arm's)",
        "config": job_config(args, w, world, shard, t0),
        "seals_in_timed_region": seals,
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": kind,
                         "sample": sample, "steps_per_s_all": value,
                         "steps_per_s_1thread": 1.0 / step_one, "threads_all": cores},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)



# ---------------------------------------------------------------- reference shapes

def reference_shapes(pkg, dev) -> dict:
    """The path's kernels at the shapes the reference published numbers for
    (Qwen3-0.6B attention shape, 16 query / 8 KV heads, RTX 4080 Laptop):
    C1.1 attention over 128 selected tokens (39.97 us kernel), C1.2 complete
    backend call with host buffers (90.4 us wall), C2.1 selection over 16
    blocks with budget 4 (14.6 us on the CPU). Device times are CUDA-event
    means over 100 graph-replayed calls; the backend call is the median host
    wall time of a call from Python with pinned host buffers."""
    import torch
    rng = np.random.default_rng(7)
    tokens, qh, kh = 128, 16, 8
    kv = torch.from_numpy(rng.standard_normal(tokens * 2 * kh * 128).astype(np.float16)
                          .view(np.int16)).to(dev)
    q = torch.from_numpy(rng.standard_normal(qh * 128).astype(np.float32)).to(dev)
    reps = torch.from_numpy(rng.standard_normal((qh, 16, 128)).astype(np.float32)).to(dev)

    def graph_us(fn, calls=100):
        side = torch.cuda.Stream(dev)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(calls):
                fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            g.replay()
            e0.record(side)
            g.replay()
            e1.record(side)
        e1.synchronize()
        return 1000.0 * e0.elapsed_time(e1) / calls

    out = {"c1_1_attention_kernel_us": graph_us(lambda: pkg.attention(kv, q, tokens, qh, kh, 128)),
           "c2_1_select_16_blocks_us": graph_us(
               lambda: pkg.select_shared_blocks(q.view(qh, 128), reps, qh, 16, 128, 4, 1, 1))}
    backend = pkg.Backend(dev.index)
    # pinned host buffers, as the reference's allocate_host gives its drivers
    kv_pin = torch.empty(kv.shape, dtype=torch.int16, pin_memory=True)
    q_pin = torch.empty(q.shape, dtype=torch.float32, pin_memory=True)
    kv_pin.copy_(kv.cpu())
    q_pin.copy_(q.cpu())
    kv_h, q_h = kv_pin.numpy().view(np.uint16), q_pin.numpy()
    for _ in range(3):
        backend.attention(kv_h, q_h, tokens, qh, kh, 128, 0.08838834764831845)
    walls = []
    for _ in range(200):
        t0 = time.perf_counter()
        backend.attention(kv_h, q_h, tokens, qh, kh, 128, 0.08838834764831845)
        walls.append(1e6 * (time.perf_counter() - t0))
    backend.close()
    out["c1_2_backend_call_wall_us"] = statistics.median(walls)
    out["reference_published_us"] = {"c1_1_attention_kernel": 39.97, "c1_2_backend_call_wall": 90.433,
                                     "c2_1_select_cpu": 14.579, "hardware": "RTX 4080 Laptop / i9-14900HX"}
    return out


# ---------------------------------------------------------------- our arm

def timed_steps(ctx, step, first, count, use_graph, stream, barrier):
    """Records steps [first, first + count) (when use_graph) and times them
    on the device: (ms, launches of this repository's kernels, clocks)."""
    import torch

    if use_graph:
        # record the timed steps (nothing runs); the timed region replays them
        with torch.cuda.stream(stream), ctx.record():
            for s in range(first, first + count):
                step(s)
    # The sampler is running before the region starts; every rank starts its
    # region after the barrier (a rank that started early would wait for the
    # others' gathered outputs inside its own timed region).
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.wait_first()
    barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        if use_graph:
            ctx.graph_launch()
        else:
            for s in range(first, first + count):
                step(s)
        end.record(stream)
    end.synchronize()
    clock_info = clocks.stop()
    return start.elapsed_time(end), ctx.launches - launches0, clock_info


def replica_run(args, w, dev, rank, world, barrier, max_over_ranks):
    """Every rank decodes its own whole sequence (global index = rank), no
    collective: the weak-scaling counterpart of a KV-head split."""
    import torch

    from solidattention_repro_b200 import workloads

    K, W = args.steps, args.warmup
    t0 = workloads.tail_for_seal_at_end(K, W)
    with torch.cuda.stream(torch.cuda.Stream(dev)):
        ctx, info = workloads.make_context(w, K + W + 64, dev, seed=SEED, seq_offset=rank,
                                           initial_tail=t0)
    queries, kv_new = workloads.decode_inputs(w, info, K + W, dev, seed=SEED + rank)
    out = ctx.new_output()

    def step(s):
        ctx.step(queries[s], kv_new[s], out)

    with torch.cuda.stream(ctx.stream):
        for s in range(W):
            step(s)
    ctx.sync()
    ms, launches, _ = timed_steps(ctx, step, W, K, args.launch == "graph", ctx.stream, barrier)
    bits = ctx.status_bits()
    ctx.close()
    ms = max_over_ranks(ms)
    return {"value": world * K / (ms / 1000.0), "unit": "sequence-steps/s",
            "ms_per_step": ms / K, "scaling": "weak", "gpu_launches": launches,
            "device_status_bits": bits,
            "layout": f"each of the {world} ranks decodes its own whole sequence (global "
                      f"index = rank), all KV heads, no collective"}


def our_arm(args, w, rank, world, local_rank, pkg):
    import torch
    import torch.distributed as dist

    from solidattention_repro_b200 import quality as quality_mod
    from solidattention_repro_b200 import workloads

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    K, W = args.steps, args.warmup
    total = K + W
    e2e_steps = min(K, 500)
    dist_steps = min(K, 100)  # per-step distribution pass (after the timed region)
    shard, kv_slice, seq_offset = job_layout(args, w, world, rank)
    heads_mode = shard == "heads"
    t0 = workloads.tail_for_seal_at_end(K, W)
    seals = workloads.seal_steps(t0, W, K)
    # table room for every append of the run: warmup + timed + e2e steps. The
    # context's stream is its own (a graph cannot record the default stream).
    with torch.cuda.stream(torch.cuda.Stream(dev)):
        ctx, info = workloads.make_context(w, total + e2e_steps + dist_steps + 64, dev, seed=SEED,
                                           kv_heads_slice=kv_slice, seq_offset=seq_offset,
                                           initial_tail=t0)
    phase_bits = {}
    queries, kv_new = workloads.decode_inputs(w, info, total, dev, seed=SEED + seq_offset,
                                              kv_heads_slice=kv_slice)
    out = ctx.new_output()
    stream = ctx.stream
    gathered = None
    p2p = heads_mode and args.gather == "p2p"
    if heads_mode:
        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev)
        if p2p:
            ctx.enable_gather(world, rank)
        barrier()

    def step(s):
        ctx.step(queries[s], kv_new[s], out)
        if p2p:
            # the attention kernel stored every output into all ranks' buffers
            ctx.gather_wait(view=False)
        elif heads_mode:
            # [world][S][L][QH/world][D]: rank order = head order
            dist.all_gather_into_tensor(gathered, out)

    with torch.cuda.stream(stream):
        for s in range(W):
            step(s)
    ctx.sync()
    # NCCL's all-gather stays outside graphs; the peer-memory gather records
    use_graph = args.launch == "graph" and (not heads_mode or p2p)
    ms_local, gpu_launches, clock_info = timed_steps(ctx, step, W, K, use_graph, stream, barrier)
    phase_bits["timed"] = ctx.status_bits()
    ctx.sync()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ms_local)
    seqs_total = w.seqs * (world if shard == "seqs" else 1)
    steps_per_s = seqs_total * K / (ms / 1000.0)

    # ---- per-step distribution: one call per step, CUDA events between steps
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(dist_steps + 1)]
    with torch.cuda.stream(stream):
        evs[0].record(stream)
        for i in range(dist_steps):
            step(W + i)
            evs[i + 1].record(stream)
    evs[-1].synchronize()
    per_step = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(dist_steps))
    phase_bits["dist"] = ctx.status_bits()
    ctx.sync()
    barrier()

    def pct(xs, q):
        return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))] if xs else None
    step_dist = {"p10": pct(per_step, 0.1), "p50": pct(per_step, 0.5), "p90": pct(per_step, 0.9),
                 "max": per_step[-1] if per_step else None, "steps": dist_steps, "unit": "ms",
                 "timing": "CUDA events between consecutive single-step calls, rank 0"}

    # ---- the peer-memory gather against NCCL: one more step's gathered slot
    # equals an NCCL all-gather of every rank's own output (bit for bit)
    gather_check = None
    if p2p:
        with torch.cuda.stream(stream):
            ctx.step(queries[W], kv_new[W], out)
            got = ctx.gather_wait().clone()
            ref = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev)
            dist.all_gather_into_tensor(ref, out)
            ref = ref.permute(1, 2, 0, 3, 4).reshape(got.shape)
            same = torch.equal(got, ref)
        stream.synchronize()
        gather_check = max_over_ranks(0.0 if same else 1.0) == 0.0
        phase_bits["gather_check"] = ctx.status_bits()
        ctx.sync()
        barrier()

    # ---- per-kernel roofline: each kernel alone, on its launch stream
    q_last = queries[total - 1]
    nb_now = ctx.num_sealed.cpu().numpy()
    tail_now = ctx.tail_len.cpu().numpy()
    ctx.select(q_last)
    counts = ctx.selected_count.cpu().numpy()
    kv_bytes = int(sum((int(counts[sl].max()) * 32 + int(tail_now[sl])) * 2 * ctx.kh * 128 * 2
                       for sl in range(ctx.num_sl)))
    rep_bytes = int(sum(int(n) for n in nb_now) * ctx.qh * 128 * 4)

    def time_kernel(fn):
        """Mean device time of one launch: kernel_iters launches recorded into
        a CUDA graph and replayed (no host launch gaps between them)."""
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream), ctx.record():
            for _ in range(args.kernel_iters):
                fn()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ctx.graph_launch()  # warm replay
            e0.record(stream)
            ctx.graph_launch()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / args.kernel_iters

    t_attn = max_over_ranks(time_kernel(lambda: ctx.attend(q_last, out)))
    if p2p:
        # the attention alone kept storing into every rank's gathered slot
        # and counting arrivals: start the gather afresh on every rank
        ctx.sync()
        barrier()
        ctx.gather_restart()
        barrier()
    t_sel = max_over_ranks(time_kernel(lambda: ctx.select(q_last)))
    phase_bits["kernels"] = ctx.status_bits()
    ctx.sync()
    hbm, peak_kind = peaks()
    attn_gbs = kv_bytes / (t_attn * 1e-3) / 1e9
    sel_gbs = rep_bytes / (t_sel * 1e-3) / 1e9
    dominant = ("attention", t_attn, attn_gbs, kv_bytes) if t_attn >= t_sel else \
        ("select", t_sel, sel_gbs, rep_bytes)
    traffic = profile_traffic(dominant[0], args.config, dominant[3])

    # ---- end to end through the public host-buffer call
    qn = w.seqs * w.layers * ctx.qh * 128
    kvn = w.seqs * w.layers * 2 * ctx.kh * 128
    q_host = torch.empty(qn, dtype=torch.float32, pin_memory=True)
    kv_host = torch.empty(kvn, dtype=torch.float16, pin_memory=True)
    out_host = torch.empty(qn, dtype=torch.float16 if w.out_fp16 else torch.float32,
                           pin_memory=True)
    q_host.copy_(queries[0].reshape(-1).cpu())
    kv_host.copy_(kv_new[0].reshape(-1).cpu())
    if heads_mode:
        # H2D of this rank's query/K/V shard, the device step, the gather of
        # the per-head outputs, D2H of the assembled output
        q_dev = torch.empty_like(queries[0])
        kv_dev = torch.empty_like(kv_new[0])
        out_host = torch.empty(tuple(gathered.shape), dtype=gathered.dtype, pin_memory=True)

        def e2e_step():
            with torch.cuda.stream(stream):
                q_dev.copy_(q_host.view_as(q_dev), non_blocking=True)
                kv_dev.copy_(kv_host.view_as(kv_dev), non_blocking=True)
                ctx.step(q_dev, kv_dev, out)
                if p2p:
                    out_host.view(-1).copy_(ctx.gather_wait().reshape(-1), non_blocking=True)
                else:
                    dist.all_gather_into_tensor(gathered, out)
                    out_host.copy_(gathered, non_blocking=True)
            stream.synchronize()
    else:
        def e2e_step():
            ctx.step_host(q_host, kv_host, out_host)
    try:
        for _ in range(3):
            e2e_step()
    finally:
        phase_bits["e2e_warmup"] = ctx.status_bits()
    barrier()
    torch.cuda.synchronize()
    t_e2e = time.perf_counter()
    e2e_times = []
    try:
        for _ in range(e2e_steps):
            t_step = time.perf_counter()
            e2e_step()
            e2e_times.append(1000.0 * (time.perf_counter() - t_step))
    finally:
        phase_bits["e2e"] = ctx.status_bits()
        if any(phase_bits.values()):
            print(json.dumps({"rank": rank, "device_status_bits": phase_bits}), file=sys.stderr)
    e2e_s = max_over_ranks(time.perf_counter() - t_e2e)
    e2e = {"value": seqs_total * e2e_steps / e2e_s, "unit": "steps/s",
           "h2d_bytes_per_step": q_host.numel() * 4 + kv_host.numel() * 2,
           "d2h_bytes_per_step": out_host.numel() * out_host.element_size() + 4,
           "steps": e2e_steps, "timing": "host wall clock around synchronous calls, max over ranks"}
    e2e_times.sort()
    e2e["step_ms"] = {"p10": pct(e2e_times, 0.1), "p50": pct(e2e_times, 0.5),
                      "p90": pct(e2e_times, 0.9), "rank": 0}

    # ---- selection quality of the last step (dense audit, not timed)
    ctx.select(q_last)
    mass = ctx.audit(q_last)
    ctx.sync()
    hot = info["hot"]
    if kv_slice is not None:
        hot = hot[:, :, kv_slice[0]:kv_slice[0] + kv_slice[1]]
    qual = quality_mod.selection_quality(
        mass.cpu().numpy(), ctx.selected.cpu().numpy(), ctx.selected_count.cpu().numpy(),
        ctx.num_sealed.cpu().numpy(), w.budget_blocks, w.init_blocks, w.local_blocks,
        hot.reshape(ctx.num_sl, ctx.kh, -1) if w.hot_blocks else None)
    del mass
    # history prediction (the reference's tiered pipeline): a slot window that
    # follows the selection of the last eight steps' queries
    slots = ctx.new_slots()
    hits = selected = 0
    for k in range(8):
        ctx.select(queries[total - 8 + k])
        _, _, stats = ctx.slot_correct(slots)
        if k:
            st = stats.cpu().numpy()
            hits += int(st[..., 0].sum())
            selected += int(st.sum())
    ctx.sync()
    qual["history_hit_rate"] = hits / selected if selected else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline(ctx, w, q_last, args.cpu_seconds, os.cpu_count() or 1)
    ref_shapes = reference_shapes(pkg, dev) if rank == 0 and world == 1 else None
    ctx.close()
    replicas = None
    if heads_mode and not args.no_replicas:
        barrier()
        replicas = replica_run(args, w, dev, rank, world, barrier, max_over_ranks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": steps_per_s, "unit": "steps/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "weak" if shard == "seqs" else "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded FP16 N(0,1) KV with planted hot blocks, seeded queries",
            "config": job_config(args, w, world, shard, t0),
            "launch": ("one CUDA graph of the timed steps (sa_ctx_graph_launch)" if use_graph
                       else "one sa_ctx_step call per step"),
            "seals_in_timed_region": seals,
            "step_ms_distribution": step_dist,
            "selected_kv_gbs": attn_gbs, "selected_kv_frac": attn_gbs / hbm,
            # one GPU's selected KV of a step (16-token average tail) / the step time
            "step_selected_kv_gbs": w.selected_kv_bytes(16) * (1 if shard == "seqs" else 1.0 / world)
            / (ms / K * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": dominant[0], "achieved": dominant[2],
                         "peak": hbm, "unit": "GB/s", "frac": dominant[2] / hbm,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "bytes_per_launch": dominant[3], "ms_per_launch": dominant[1]},
            "kernels": {
                "attention": {"ms": t_attn, "bytes": kv_bytes, "gbs": attn_gbs,
                              "frac": attn_gbs / hbm},
                "select": {"ms": t_sel, "bytes": rep_bytes, "gbs": sel_gbs,
                           "frac": sel_gbs / hbm},
                "rest_of_step_ms": ms / K - t_attn - t_sel,
                "timing": "each kernel alone: CUDA events around a replayed CUDA graph of "
                          "back-to-back launches, max over ranks; rest_of_step_ms = the step "
                          "minus both (seal, gather, launch gaps, and the overlap that chaining "
                          "them gains)"},
            "quality": qual,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": gpu_launches,
            "replicas": replicas,
            "gather_equals_nccl_all_gather": gather_check,
            "reference_shapes": ref_shapes,
            "device_status_bits": phase_bits,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def probe_streaming(args, pkg):
    """The attention's two ways of staging entries, alone: one launch reads
    `entries` distinct random 16 KB entries of a 1 GiB pool (more than L2),
    CUDA events around `steps` back-to-back launches after `warmup`."""
    import ctypes as C

    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = pkg.load()
    pool_entries, entries = 1 << 16, 288 * 128  # cfg3's selected entries of a step
    pool = torch.zeros(pool_entries * 16384, dtype=torch.uint8, device=dev)
    g = torch.Generator().manual_seed(1)
    ids = torch.randperm(pool_entries, generator=g)[:entries].to(torch.int32).to(dev)
    sink = torch.zeros(1024, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    steps, warmup = max(1, min(args.steps, 50)), max(3, min(args.warmup, 10))
    out = {"probe": "streaming", "entry_bytes": 16384, "entries": entries,
           "pool_bytes": pool_entries * 16384, "ctas_per_sm": 2, "threads": 256,
           "stages": "3 x 32 KB", "steps": steps, "warmup": warmup}
    for mode, name in ((0, "cp_async"), (1, "bulk")):
        def launch():
            rc = lib.sa_probe_stream(C.c_void_p(pool.data_ptr()), pool_entries,
                                     C.c_void_p(ids.data_ptr()), entries, mode,
                                     C.c_void_p(sink.data_ptr()), C.c_void_p(status.data_ptr()),
                                     C.c_void_p(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError(f"sa_probe_stream: {lib.sa_last_error().decode()}")
        for _ in range(warmup):
            launch()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            launch()
        e1.record(stream)
        e1.synchronize()
        us = 1000.0 * e0.elapsed_time(e1) / steps
        out[name] = {"us_per_launch": us, "gbs": entries * 16384 / (us * 1e-6) / 1e9}
    out["status"] = int(status.item())
    hbm, kind = peaks()
    out["peak_gbs"] = hbm
    out["peak_kind"] = kind
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    if args.probe_streaming:
        probe_streaming(args, pkg)
        return
    from solidattention_repro_b200 import workloads

    w = workloads.CONFIGS[args.config]
    if args.layers:
        import dataclasses
        w = dataclasses.replace(w, layers=args.layers, name=f"{w.name}-{args.layers}layers")
    if args.impl == "reference":
        reference_arm(args, w, rank, world)
        return
    our_arm(args, w, rank, world, local_rank, pkg)


if __name__ == "__main__":
    main()
