#!/usr/bin/env python
"""Benchmark of the B200 sparse-KV decode path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3] [--impl ours|reference]

A step is one decode step of the workload: for every (sequence, layer)
append the token's K/V, score + select blocks per KV head, attend over the
selected blocks plus the open tail, and seal the tail when it holds 32
tokens. The default workload is the path's target configuration: Qwen3-8B
shape (32 query / 8 KV heads, head_dim 128, 36 layers), 32K context (1024
blocks), 4096-token budget (1 init + 4 local + 123 dynamic blocks). At N > 1
each rank decodes its own sequences (sequence sharding by global batch index,
no data-path collective): weak scaling; value = all ranks' sequence-steps /
max time. `--config cfg5` (one 128K-context sequence) shards the KV heads
instead: rank r holds KH/N heads of every layer, and each step ends with an
NCCL all-gather of the per-head outputs: strong scaling.

`value` is device-timed with inputs resident in HBM, the timed steps replayed
from one recorded CUDA graph (`--launch eager` issues one call per step); `e2e` runs the same
steps through the public host-buffer call (sa_ctx_step_host: H2D of the
step's query + new K/V, step, D2H of the output, synchronize).
`--impl reference` times the reference's own CPU implementation (the C++
selector + attention compiled from its sources, oracle/_ref) on the host's
cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
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


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", default="cfg3", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kernel-iters", type=int, default=50)
    ap.add_argument("--launch", default="graph", choices=["graph", "eager"],
                    help="timed steps replayed from one recorded CUDA graph (sa_ctx_graph_*) "
                         "or launched one call at a time; KV-head sharding with the NCCL gather runs eager")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="KV-head sharding (cfg5, N > 1): gather the per-head outputs with "
                         "peer-memory stores from the attention kernel (p2p) or an NCCL "
                         "all-gather after it (nccl)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the workload's layer count (small profiling cases)")
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


# ------------------------------------------------------------ CPU baseline

def cpu_lib():
    import oracle

    ref = oracle.reference()
    return (ref, "reference") if ref is not None else (oracle.port(), "port")


def cpu_step_sample(lib, pool_host, table_host, reps_host, q_host, tail_host, tail_len, w,
                    nb, threads):
    ids, out = lib.sparse_step(pool_host, table_host, reps_host, q_host, tail_host, tail_len,
                               w.query_heads, w.kv_heads, 128, 32, nb,
                               min(w.budget_blocks, nb), w.init_blocks, w.local_blocks,
                               np.float32(1.0) / np.sqrt(np.float32(128)), threads)
    return ids, out


def host_sample_from_ctx(ctx, layers):
    """Copy the sampled layers' sealed blocks, tails, tables and reps to host."""
    import torch

    nb_all = ctx.num_sealed.cpu().numpy()
    tables = ctx.table.cpu().numpy()
    tails = ctx.tail_block.cpu().numpy()
    tail_len = int(ctx.tail_len.cpu().numpy()[layers[0]])
    nb = int(nb_all[layers[0]])
    pools, table_rows, tail_rows, reps = [], [], [], []
    for i, l in enumerate(layers):
        phys = np.concatenate([tables[l, :nb], tails[l:l + 1]]).astype(np.int64)
        pools.append(ctx.read_blocks(phys).cpu().numpy().view(np.uint16))
        table_rows.append(np.arange(nb, dtype=np.int32) + i * (nb + 1))
        tail_rows.append(i * (nb + 1) + nb)
        reps.append(ctx.reps[l, :, :, :nb].permute(0, 2, 1).contiguous().cpu().numpy())
    return (np.concatenate(pools), np.stack(table_rows), np.stack(reps),
            np.asarray(tail_rows, np.int32), tail_len, nb)


def run_cpu_baseline(ctx, w, q_step, n_layers_total, seconds, threads):
    """Time the reference CPU path (selection per KV head + gather + attention)
    over a bounded sample of layers of the current decode step; extrapolate."""
    lib, kind = cpu_lib()
    layers = list(range(min(4, n_layers_total)))
    ctx.select(q_step)
    sel = ctx.selected.cpu().numpy()
    pool_h, table_h, reps_h, tail_h, tail_len, nb = host_sample_from_ctx(ctx, layers)
    q_h = q_step.reshape(-1, w.query_heads, 128)[layers].cpu().numpy()
    times, ids = [], None
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        ids, _ = cpu_step_sample(lib, pool_h, table_h, reps_h, q_h, tail_h, tail_len, w, nb, threads)
        times.append(time.perf_counter() - t0)
    per_sample = statistics.median(times)
    steps_per_s = 1.0 / (per_sample * n_layers_total / len(layers))
    eff = min(w.budget_blocks, nb)
    match = bool(np.array_equal(ids, sel[layers][:, :, :eff].astype(np.int64)))
    return {"value": steps_per_s, "unit": "steps/s", "cores": threads, "kind": kind,
            "sample": f"{len(layers)} of {n_layers_total} layers of one decode step "
                      f"(select per KV head + packed gather + attention, {nb} sealed blocks, "
                      f"tail {tail_len}), median of {len(times)} runs, extrapolated to all layers",
            "ids_match_gpu": match}


# ---------------------------------------------------------------- reference arm

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


def reference_arm(args, w, rank):
    """The reference's CPU implementation of the path on host cores (no GPU work)."""
    if rank != 0:
        return
    lib, kind = cpu_lib()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1234)
    total = args.steps + args.warmup
    n_sample = 2 if total > 40 else 4
    n_sample = min(n_sample, w.layers)
    nb = w.context_blocks
    if w.context_min_blocks:
        nb = int(round(np.mean([w.sequence_blocks(b) for b in range(w.batch)])))
    tail_len = 16
    tv = 2 * w.kv_heads * 128
    pool = (rng.standard_normal((n_sample * (nb + 1) * 32 * tv,), dtype=np.float32)
            .astype(np.float16).view(np.uint16))
    table = np.stack([np.arange(nb, dtype=np.int32) + i * (nb + 1) for i in range(n_sample)])
    tails = np.asarray([i * (nb + 1) + nb for i in range(n_sample)], np.int32)
    reps = (rng.standard_normal((n_sample, w.query_heads, nb, 128), dtype=np.float32) * 0.5
            ).astype(np.float16).astype(np.float32)
    q = rng.standard_normal((n_sample, w.query_heads, 128), dtype=np.float32
                            ).astype(np.float16).astype(np.float32)
    for _ in range(args.warmup):
        cpu_step_sample(lib, pool, table, reps, q, tails, tail_len, w, nb, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_step_sample(lib, pool, table, reps, q, tails, tail_len, w, nb, threads)
        times.append(time.perf_counter() - t0)
    per_layer = sum(times) / len(times) / n_sample
    value = 1.0 / (per_layer * w.layers)
    sample = (f"{n_sample} of {w.layers} layers per step (select per KV head + packed gather + "
              f"attention over {min(w.budget_blocks, nb)} blocks + {tail_len}-token tail), "
              f"extrapolated to all layers")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "layers": w.layers, "query_heads": w.query_heads,
                   "kv_heads": w.kv_heads, "head_dim": 128, "context_tokens": nb * 32,
                   "budget_blocks": w.budget_blocks},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from solidattention_repro_b200 import workloads

    w = workloads.CONFIGS[args.config]
    if args.layers:
        import dataclasses
        w = dataclasses.replace(w, layers=args.layers, name=f"{w.name}-{args.layers}layers")
    if args.impl == "reference":
        reference_arm(args, w, rank)
        return

    import torch
    import torch.distributed as dist

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

    total = args.steps + args.warmup
    e2e_steps = min(args.steps, 500)
    dist_steps = min(args.steps, 100)  # per-step distribution pass (after the timed region)
    heads_mode = args.config == "cfg5" and world > 1
    if heads_mode:
        # KV-head sharding of one long sequence
        from solidattention_repro_b200 import sharding
        kv_slice = sharding.shard_kv_heads(w.kv_heads, world, rank)
        seq_offset = 0
    else:
        kv_slice = None
        seq_offset = rank * w.seqs  # sequence sharding by global batch index
    # table room for every append of the run: warmup + timed + e2e steps. The
    # context's stream is its own (a graph cannot record the default stream).
    with torch.cuda.stream(torch.cuda.Stream(dev)):
        ctx, info = workloads.make_context(w, total + e2e_steps + dist_steps + 64, dev, seed=1,
                                           kv_heads_slice=kv_slice, seq_offset=seq_offset)
    phase_bits = {}
    queries, kv_new = workloads.decode_inputs(w, info, total, dev, seed=1 + seq_offset,
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
        for s in range(args.warmup):
            step(s)
    ctx.sync()
    # NCCL's all-gather stays outside graphs; the peer-memory gather records
    use_graph = args.launch == "graph" and (not heads_mode or p2p)
    if use_graph:
        # record the K timed steps (nothing runs); the timed region replays them
        with torch.cuda.stream(stream), ctx.record():
            for s in range(args.warmup, total):
                step(s)
    barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    clocks = ClockSampler(local_rank)
    clocks.wait_first()  # the sampler is running before the region starts
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        if use_graph:
            ctx.graph_launch()
        else:
            for s in range(args.warmup, total):
                step(s)
        end.record(stream)
    end.synchronize()
    clock_info = clocks.stop()
    ms_local = start.elapsed_time(end)
    gpu_launches = ctx.launches - launches0
    phase_bits["timed"] = ctx.status_bits()
    ctx.sync()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ms_local)
    seqs_total = w.seqs if heads_mode else world * w.seqs
    steps_per_s = seqs_total * args.steps / (ms / 1000.0)

    # ---- per-step distribution: one call per step, CUDA events between steps
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(dist_steps + 1)]
    with torch.cuda.stream(stream):
        evs[0].record(stream)
        for i in range(dist_steps):
            step(args.warmup + i)
            evs[i + 1].record(stream)
    evs[-1].synchronize()
    per_step = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(dist_steps))
    phase_bits["dist"] = ctx.status_bits()
    ctx.sync()
    barrier()

    def pct(xs, q):
        return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))] if xs else None
    step_dist = {"p10": pct(per_step, 0.1), "p50": pct(per_step, 0.5), "p90": pct(per_step, 0.9),
                 "steps": dist_steps, "unit": "ms",
                 "timing": "CUDA events between consecutive single-step calls, rank 0"}

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
        for _ in range(3):
            fn()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.kernel_iters):
                fn()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / args.kernel_iters

    t_attn = max_over_ranks(time_kernel(lambda: ctx.attend(q_last, out)))
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
        # H2D of this rank's query/K/V shard, the device step, the all-gather
        # of the per-head outputs, D2H of the assembled output
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
    t0 = time.perf_counter()
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
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": seqs_total * e2e_steps / e2e_s, "unit": "steps/s",
           "h2d_bytes_per_step": q_host.numel() * 4 + kv_host.numel() * 2,
           "d2h_bytes_per_step": out_host.numel() * out_host.element_size() + 4,
           "steps": e2e_steps, "timing": "host wall clock around synchronous calls, max over ranks"}
    e2e_times.sort()
    e2e["step_ms"] = {"p10": pct(e2e_times, 0.1), "p50": pct(e2e_times, 0.5),
                      "p90": pct(e2e_times, 0.9), "rank": 0}

    # ---- selection quality of the last step (dense audit, not timed)
    from solidattention_repro_b200 import quality as quality_mod
    ctx.select(q_last)
    mass = ctx.audit(q_last)
    ctx.sync()
    hot = info["hot"]
    if heads_mode:
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
        cpu = run_cpu_baseline(ctx, w, q_last, w.layers, args.cpu_seconds, os.cpu_count() or 1)
    ref_shapes = reference_shapes(pkg, dev) if rank == 0 and world == 1 else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": steps_per_s, "unit": "steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if heads_mode else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded FP16 N(0,1) KV with planted hot blocks, seeded queries",
            "config": {
                "workload": w.name, "layers": w.layers, "query_heads": w.query_heads,
                "kv_heads": w.kv_heads, "head_dim": 128, "context_tokens": w.context_blocks * 32,
                "budget_blocks": w.budget_blocks, "init_blocks": w.init_blocks,
                "local_blocks": w.local_blocks, "seqs_per_gpu": w.seqs,
                "context_min_tokens": (w.context_min_blocks or w.context_blocks) * 32,
                "parallelism": (f"kv-head-sharded x{world}, outputs gathered by "
                                + ("the attention kernel's peer-memory stores (NVLink P2P)"
                                   if p2p else "an NCCL all-gather") + " every step"
                                if heads_mode else
                                f"sequence-sharded x{world}" if world > 1 else "single"),
                "l2": "inputs larger than L2: each step reads its selected KV and all "
                      "representatives (>1 GB at cfg3)",
                "kv_dtype": "fp16", "accumulate": "fp32",
                "launch": ("one CUDA graph of the timed steps (sa_ctx_graph_launch)" if use_graph
                           else "one sa_ctx_step call per step")},
            "step_ms_distribution": step_dist,
            "selected_kv_gbs": attn_gbs, "selected_kv_frac": attn_gbs / hbm,
            # selected KV (16-token average tail) per GPU-step x per-GPU steps/s
            "step_selected_kv_gbs": w.selected_kv_bytes(16) * steps_per_s / world / 1e9,
            "roofline": {"bound": "hbm", "kernel": dominant[0], "achieved": dominant[2],
                         "peak": hbm, "unit": "GB/s", "frac": dominant[2] / hbm,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "bytes_per_launch": dominant[3], "ms_per_launch": dominant[1]},
            "kernels": {
                "attention": {"ms": t_attn, "bytes": kv_bytes, "gbs": attn_gbs,
                              "frac": attn_gbs / hbm},
                "select": {"ms": t_sel, "bytes": rep_bytes, "gbs": sel_gbs,
                           "frac": sel_gbs / hbm}},
            "quality": qual,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": gpu_launches,
            "reference_shapes": ref_shapes,
            "device_status_bits": phase_bits,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
