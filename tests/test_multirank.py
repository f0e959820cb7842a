"""Multi-rank host logic on CPU (gloo, world_size 2), with the oracle as compute.

* sequence sharding: each rank decodes its own sequences; gathering the
  per-rank outputs reproduces the single-process step, and the step time is
  the max over ranks;
* KV-head sharding: each rank attends for its KV heads of one sequence; an
  all-gather over heads reproduces the full [QH][128] output;
* a rank that fails before a collective makes the other rank's collective
  end with an error after the process-group timeout (no hang).
"""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
SCALE = np.float32(1.0) / np.sqrt(np.float32(128))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _state(seq: int, layers=2, qh=8, kh=4, nb=12):
    """A small seeded decode state of one sequence (host arrays)."""
    rng = np.random.default_rng(seq)
    tv = 2 * kh * 128
    pool = (rng.standard_normal(layers * (nb + 1) * 32 * tv, dtype=np.float32)
            .astype(np.float16).view(np.uint16))
    table = np.stack([np.arange(nb, dtype=np.int32) + i * (nb + 1) for i in range(layers)])
    tails = np.array([i * (nb + 1) + nb for i in range(layers)], np.int32)
    reps = rng.standard_normal((layers, qh, nb, 128), dtype=np.float32)
    q = rng.standard_normal((layers, qh, 128), dtype=np.float32)
    return pool, table, reps, q, tails


def _step(port, seq, heads=None):
    pool, table, reps, q, tails = _state(seq)
    layers, qh, kh, nb = 2, 8, 4, 12
    ids, out = port.sparse_step(pool, table, reps, q, tails, 5, qh, kh, 128, 32, nb, 6, 1, 2,
                                SCALE, 1)
    return ids, out


def _init(rank, world, port_no, timeout_s=30):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    return dist


def _worker_sequences(rank, world, port_no, result_dir):
    sys.path.insert(0, str(ROOT))
    import torch

    import __graft_entry__
    import oracle

    __graft_entry__.load_package()
    from solidattention_repro_b200 import sharding

    dist = _init(rank, world, port_no)
    port = oracle.port()
    first, count = sharding.shard_sequences(4, world, rank)
    outs = [torch.from_numpy(_step(port, s)[1]) for s in range(first, first + count)]
    mine = torch.stack(outs)
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    elapsed = torch.tensor([1.0 + rank], dtype=torch.float64)
    dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    if rank == 0:
        np.save(Path(result_dir) / "seq.npy", torch.cat(gathered).numpy())
        np.save(Path(result_dir) / "time.npy", elapsed.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _worker_heads(rank, world, port_no, result_dir):
    sys.path.insert(0, str(ROOT))
    import torch

    import __graft_entry__
    import oracle

    __graft_entry__.load_package()
    from solidattention_repro_b200 import sharding

    dist = _init(rank, world, port_no)
    port = oracle.port()
    pool, table, reps, q, tails = _state(0)
    kh, qh, g = 4, 8, 2
    h0, hn = sharding.shard_kv_heads(kh, world, rank)
    # this rank's KV heads: per-head selection + attention from the oracle
    ids, out = port.sparse_step(pool, table, reps, q, tails, 5, qh, kh, 128, 32, 12, 6, 1, 2,
                                SCALE, 1)
    mine = torch.from_numpy(np.ascontiguousarray(out[:, h0 * g:(h0 + hn) * g]))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    if rank == 0:
        full = sharding.assemble_heads([x.numpy() for x in gathered], g)
        np.save(Path(result_dir) / "heads.npy", full)
    dist.barrier()
    dist.destroy_process_group()


def _worker_fail(rank, world, port_no, result_dir):
    import torch

    dist = _init(rank, world, port_no, timeout_s=5)
    if rank == 1:
        raise SystemExit(3)  # leaves before the collective
    t = torch.ones(1)
    try:
        dist.all_reduce(t)
        status = "completed"
    except Exception as e:  # gloo reports the missing peer
        status = f"error: {type(e).__name__}"
    (Path(result_dir) / "fail.txt").write_text(status)


def test_sequence_sharding_matches_single_process(port, tmp_path):
    mp.spawn(_worker_sequences, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got = np.load(tmp_path / "seq.npy")
    want = np.stack([_step(port, s)[1] for s in range(4)])
    assert np.array_equal(got, want)
    assert float(np.load(tmp_path / "time.npy")[0]) == 2.0  # max over ranks


def test_kv_head_sharding_all_gather_matches_full(port, tmp_path):
    mp.spawn(_worker_heads, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got = np.load(tmp_path / "heads.npy")
    assert np.array_equal(got, _step(port, 0)[1])


def test_missing_rank_ends_collective_with_error(tmp_path):
    ctx = mp.start_processes(_worker_fail, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    try:
        ctx.join(timeout=120)
    except Exception:
        pass  # rank 1's exit is reported as a process failure
    for p in ctx.processes:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    status = (tmp_path / "fail.txt").read_text()
    assert status.startswith("error"), status


def test_shard_ranges_cover_everything():
    import __graft_entry__

    __graft_entry__.load_package()
    from solidattention_repro_b200 import sharding

    for total in (1, 7, 8, 64):
        for world in (1, 2, 3, 8):
            parts = [sharding.shard_range(total, world, r) for r in range(world)]
            covered = [i for f, c in parts for i in range(f, f + c)]
            assert covered == list(range(total))
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    assert sharding.shard_kv_heads(8, 8, 3) == (3, 1)
    with pytest.raises(ValueError):
        sharding.shard_kv_heads(8, 3, 0)
