"""Parity at the benchmark configurations themselves.

Each test builds the decode context of one benchmark config with the
workload generator the bench uses (seeded FP16 N(0,1) KV, planted hot
blocks, representatives built by the rebuild kernel from seeded prompt
queries, seeded decode queries), keeping the config's blocks per unit,
budget, init/local counts and head layout at full size and only fewer of
its layers. Every decode step is then checked against the CPU oracle run on
the context's own state (representatives, block table, pool rows):

* selected block ids per KV head: identical to the reference selector
  (cpp/src/selection.cpp:96-147, per KV-head group) -- scores are computed in
  the reference's order, so no near-tie exemption is needed;
* attention outputs: the reference attention (cpp/src/attention_reference.cpp:
  55-96) over the selected blocks gathered in ascending order plus the open
  tail, as cpp/src/selection_main.cpp:196-218 packs them; FP16 output within
  max-abs 2e-3 and cosine 0.99999, FP32 output within 2e-5 and 0.999999 (the
  reference's own C1 gate, cpp/src/attention_main.cpp:265-270);
* the seal step: the sealed block's representative equals the reference's
  rebuild over the tail's 32 queries (values within 1e-6, except at a
  received-mass near-tie on the top-4 boundary).

cfg1 is the C1-style recipe: one layer, 64 blocks, selection = {0} plus 13
seeded dynamic ids from 1..61 plus {62, 63}, FP16 output.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from conftest import cosine, fp16_normal
from test_gpu_context import _reps_oracle

pytestmark = pytest.mark.gpu

D = 128
SCALE = np.float32(1.0) / np.sqrt(np.float32(D))


def _check_step(port, ctx, q, nb_before, tail_before, tl_before, out, step, tol):
    """One decode step of every (seq, layer) against the oracle on the
    context's own state; the token of this step is the tail's last row."""
    qh, kh = ctx.qh, ctx.kh
    grp = qh // kh
    table = ctx.table.cpu().numpy()
    sel = ctx.selected.cpu().numpy()
    counts = ctx.selected_count.cpu().numpy()
    got_all = out.float().cpu().numpy().reshape(ctx.num_sl, qh, D)
    q = q.cpu().numpy().reshape(ctx.num_sl, qh, D)
    for sl in range(ctx.num_sl):
        nb = int(nb_before[sl])
        reps = ctx.reps[sl, :, :, :nb].permute(0, 2, 1).contiguous().cpu().numpy()
        eff = min(ctx.budget, nb)
        init = min(ctx.config.init_blocks, eff)
        local = min(ctx.config.local_blocks, max(0, eff - init))
        ids, _ = port.select_grouped(q[sl], reps, qh, grp, nb, D, eff, init, local)
        assert (counts[sl] == eff).all(), (step, sl, counts[sl])
        assert np.array_equal(sel[sl][:, :eff], ids), (step, sl)
        phys = np.unique(np.concatenate([table[sl][ids.ravel()], [tail_before[sl]]]))
        rows = ctx.read_blocks(phys).cpu().numpy().view(np.uint16)  # [n][32][2][KH][D]
        at = {int(p): i for i, p in enumerate(phys)}
        tail_rows = int(tl_before[sl]) + 1
        want = np.zeros((qh, D), np.float32)
        for h in range(kh):
            parts = [rows[at[int(table[sl][b])]][:, :, h] for b in ids[h]]
            parts.append(rows[at[int(tail_before[sl])]][:tail_rows, :, h])
            packed = np.ascontiguousarray(np.concatenate(parts)).reshape(-1)
            want[h * grp:(h + 1) * grp] = port.attention(
                packed, q[sl, h * grp:(h + 1) * grp], len(ids[h]) * 32 + tail_rows, grp, 1, D,
                SCALE)
        err = float(np.abs(got_all[sl] - want).max())
        assert err <= tol[0] and cosine(got_all[sl], want) >= tol[1], (step, sl, err)


def _check_seal(port, ctx, nb_before, tail_before):
    """The block sealed by the last step: moved into the table unchanged, its
    representative rebuilt from the tail's 32 queries as the reference does
    (cpp/src/online_seal_main.cpp:41 -> cpp/src/selection.cpp:12-94)."""
    nb_after = ctx.num_sealed.cpu().numpy()
    assert (nb_after == nb_before + 1).all()
    assert (ctx.tail_len.cpu().numpy() == 0).all()
    table = ctx.table.cpu().numpy()
    ring = ctx.query_ring.cpu().numpy()
    for sl in range(ctx.num_sl):
        nb = int(nb_before[sl])
        assert table[sl, nb] == tail_before[sl]
        blk = ctx.read_blocks([int(tail_before[sl])]).cpu().numpy().view(np.uint16).reshape(-1)
        v, _, received = _reps_oracle(port, ring[sl], blk, ctx.qh, ctx.kh)
        got_v = ctx.reps[sl, :, :, nb].cpu().numpy()
        for h in range(ctx.qh):
            if np.abs(got_v[h] - v[h]).max() > 1e-6:
                srt = np.sort(received[h])[::-1]
                assert abs(srt[3] - srt[4]) <= 1e-6 * max(1.0, abs(srt[3])), (sl, h)


def _run_config(pkg, port, cuda, w, layer_ids, steps, initial_tail, seed,
                kv_heads_slice=None):
    from solidattention_repro_b200 import workloads

    ctx, info = workloads.make_context(w, steps, cuda, seed=seed, initial_tail=initial_tail,
                                       layer_ids=layer_ids, kv_heads_slice=kv_heads_slice)
    queries, kv_new = workloads.decode_inputs(w, info, steps, cuda, seed=seed,
                                              kv_heads_slice=kv_heads_slice)
    assert (ctx.tail_len.cpu().numpy() == initial_tail).all()
    nb0 = ctx.num_sealed.cpu().numpy().copy()
    seq_blocks = np.repeat(np.asarray(info["seq_blocks"]), len(layer_ids))
    assert np.array_equal(nb0, seq_blocks)
    tol = (2e-3, 0.99999) if w.out_fp16 else (2e-5, 0.999999)
    seals = 0
    for step in range(steps):
        nb_before = ctx.num_sealed.cpu().numpy().copy()
        tail_before = ctx.tail_block.cpu().numpy().copy()
        tl_before = ctx.tail_len.cpu().numpy().copy()
        out = ctx.step(queries[step], kv_new[step])
        ctx.sync()
        _check_step(port, ctx, queries[step], nb_before, tail_before, tl_before, out, step, tol)
        if (tl_before == 31).all():
            _check_seal(port, ctx, nb_before, tail_before)
            seals += 1
    assert seals == workloads.seal_steps(initial_tail, 0, steps) >= 1
    assert ctx.status_bits() == 0
    ctx.close()


def test_cfg1_c1_recipe_fixed_selection(pkg, port, cuda):
    """BASELINE cfg1: one Qwen3-0.6B-shaped layer (16 query / 8 KV heads),
    64 blocks, selection {0} + 13 seeded dynamic ids + {62, 63}, FP16 output;
    through the paged context (caller-set selection) and the stateless packed
    call, both against the reference attention over the packed gather."""
    rng = np.random.default_rng(20250101)
    qh, kh, nb = 16, 8, 64
    dyn = np.sort(rng.choice(np.arange(1, 62), size=13, replace=False))
    ids = np.concatenate([[0], dyn, [62, 63]]).astype(np.int64)
    kv = fp16_normal(rng, (nb, 32, 2, kh, D))
    q = fp16_normal(rng, (qh, D)).view(np.float16).astype(np.float32)
    packed = np.ascontiguousarray(kv[ids]).reshape(-1)
    want = port.attention(packed, q, 16 * 32, qh, kh, D, SCALE)
    for out_fp16 in (True, False):
        tol = (2e-3, 0.99999) if out_fp16 else (2e-5, 0.999999)
        ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=1, seqs=1, pool_blocks=nb + 2,
                                table_blocks=nb + 1, budget_blocks=16, init_blocks=1,
                                local_blocks=2, out_fp16=out_fp16, device=cuda)
        phys = ctx.prefill(0, 0, nb)
        ctx.write_blocks(phys[:nb], torch.from_numpy(kv.view(np.float16)))
        ctx.selected[0, :, :16] = torch.from_numpy(ids.astype(np.int32)).to(cuda)
        ctx.selected_count[0, :] = 16
        got = ctx.attend(torch.from_numpy(q).to(cuda).view(1, 1, qh, D))
        ctx.sync()
        got = got.float().cpu().numpy().reshape(qh, D)
        assert np.abs(got - want).max() <= tol[0] and cosine(got, want) >= tol[1]
        ctx.close()
        got = pkg.attention(torch.from_numpy(packed.view(np.int16)).to(cuda),
                            torch.from_numpy(q).to(cuda), 16 * 32, qh, kh, D, float(SCALE),
                            out_fp16=out_fp16).float().cpu().numpy()
        assert np.abs(got - want).max() <= tol[0] and cosine(got, want) >= tol[1]


def test_cfg2_steps_across_a_seal(pkg, port, cuda):
    """BASELINE cfg2 (Qwen3-0.6B shape, 512 blocks, budget 1 + 4 + 59, 8 hot
    blocks per layer and KV head): tails pre-filled with 30 tokens, so the
    second step seals and the last two select over the new block too."""
    from solidattention_repro_b200 import workloads

    _run_config(pkg, port, cuda, workloads.CONFIGS["cfg2"], [0, 27], steps=4, initial_tail=30,
                seed=2)


def test_cfg3_thirty_three_steps_with_the_seal(pkg, port, cuda):
    """BASELINE cfg3 (Qwen3-8B shape, 1024 blocks, budget 1 + 4 + 123, 16 hot
    blocks): 33 decode steps from empty tails, the 32nd sealing every tail
    and rebuilding its representative, the 33rd selecting over 1025 blocks."""
    from solidattention_repro_b200 import workloads

    _run_config(pkg, port, cuda, workloads.CONFIGS["cfg3"], [0, 35], steps=33, initial_tail=0,
                seed=1)


def test_cfg4_variable_length_sequences(pkg, port, cuda):
    """BASELINE cfg4: three of its seeded sequences (contexts uniform in
    [8K, 32K] tokens, budget 64 blocks) in one paged pool, tails pre-filled
    so that the second step seals."""
    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg4"], seqs=3)
    assert len({w.sequence_blocks(s) for s in range(3)}) == 3
    _run_config(pkg, port, cuda, w, [0, 35], steps=3, initial_tail=30, seed=4)


@pytest.mark.parametrize("kv_heads_slice", [None, (3, 1)])
def test_cfg5_long_context(pkg, port, cuda, kv_heads_slice):
    """BASELINE cfg5 (128K context = 4096 blocks, budget 1 + 8 + 247, 32 hot
    blocks): top-k keys recomputed from L2 (units above 2048 blocks) and
    units split over several attention CTAs; also one KV head alone, the
    share of one GPU when the 8 KV heads are sharded over 8 GPUs."""
    from solidattention_repro_b200 import workloads

    _run_config(pkg, port, cuda, workloads.CONFIGS["cfg5"], [0, 35], steps=4, initial_tail=30,
                seed=5, kv_heads_slice=kv_heads_slice)
