"""GPU parity of the paged decode context: append -> select -> attend -> seal.

Each decode step is checked against the CPU oracle run on the context's own
state (pool bytes, block tables and representatives copied back), so the
comparison isolates the device path:
* selected ids: identical to the reference selector per KV head;
* attention: FP32 max-abs <= 2e-5 / cosine >= 0.999999 (FP16 output: 2e-3 /
  0.99999) against the reference attention over the gathered blocks + tail;
* seal: the tail block moves into the table unchanged, the new block's
  representative equals the reference's build over the tail's 32 queries
  (offsets exact up to received-mass near-ties), generation and free list
  advance.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import cosine

pytestmark = pytest.mark.gpu

D = 128


def _oracle_step(port, pool, table, nb, reps, q, tail_phys, tail_len, qh, kh, budget, init,
                 local, scale):
    """Reference selection per KV head + attention over gathered blocks and tail."""
    grp = qh // kh
    reps_ref = np.ascontiguousarray(np.transpose(reps[:, :, :nb], (0, 2, 1)))  # [qh][nb][d]
    eff_budget = min(budget, nb)
    ids = np.zeros((kh, eff_budget), np.int64)
    if nb > 0:
        ids, _ = port.select_grouped(q, reps_ref, qh, grp, nb, D, eff_budget,
                                     min(init, eff_budget), min(local, max(0, eff_budget - min(init, eff_budget))))
    out = np.zeros((qh, D), np.float32)
    for h in range(kh):
        rows = [pool[table[b]][:, :, h] for b in ids[h]] if nb > 0 else []
        rows.append(pool[tail_phys][:tail_len, :, h])
        packed = np.ascontiguousarray(np.concatenate(rows)).reshape(-1)
        tokens = len(rows[:-1]) * 32 + tail_len
        out[h * grp:(h + 1) * grp] = port.attention(packed, q[h * grp:(h + 1) * grp], tokens, grp,
                                                    1, D, scale)
    return ids, out


def _reps_oracle(port, q_ring, kv_block, qh, kh, window=32, topk=4):
    vals = np.zeros(qh * D, np.float32)
    offs = np.zeros(qh * topk, np.int64)
    received = np.zeros(qh * 32, np.float32)
    port.lib.sao_build_representatives.argtypes = [C.c_void_p] * 2 + [C.c_size_t] * 7 + [C.c_void_p] * 3
    assert port.lib.sao_build_representatives(
        np.ascontiguousarray(q_ring).ctypes.data, np.ascontiguousarray(kv_block).ctypes.data, 32, qh,
        kh, D, 32, window, topk, vals.ctypes.data, offs.ctypes.data, received.ctypes.data) == 0
    return vals.reshape(qh, D), offs.reshape(qh, topk), received.reshape(qh, 32)


@pytest.mark.parametrize("qh,kh,out_fp16", [(8, 2, False), (16, 8, True), (4, 4, False)])
def test_decode_steps_with_seal_match_oracle(pkg, port, cuda, qh, kh, out_fp16):
    layers, seqs, nb0, budget, init, local = 2, 2, 40, 10, 1, 2
    steps = 36  # the 32nd step fills the tail and seals it
    rng = np.random.default_rng(qh * 100 + kh)
    g = torch.Generator().manual_seed(qh + kh)
    ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=layers, seqs=seqs,
                            pool_blocks=seqs * layers * (nb0 + 4), table_blocks=nb0 + 4,
                            budget_blocks=budget, init_blocks=init, local_blocks=local,
                            out_fp16=out_fp16, device=cuda)
    for s in range(seqs):
        for l in range(layers):
            phys = ctx.prefill(s, l, nb0)
            ctx.write_blocks(phys[:nb0], torch.randn(nb0, 32, 2, kh, D, generator=g).half())
            pq = torch.randn(qh, nb0 * 32, D, generator=g).half().float().to(cuda)
            ctx.build_reps(s, l, 0, nb0, pq)
    ctx.sync()
    scale = np.float32(1) / np.sqrt(np.float32(D))
    tol = (2e-3, 0.99999) if out_fp16 else (2e-5, 0.999999)
    for step in range(steps):
        q = (rng.standard_normal((seqs, layers, qh, D), dtype=np.float32)).astype(np.float16).astype(np.float32)
        kvn = rng.standard_normal((seqs, layers, 2, kh, D), dtype=np.float32).astype(np.float16)
        nb_before = ctx.num_sealed.cpu().numpy().copy()
        tail_before = ctx.tail_block.cpu().numpy().copy()
        out = ctx.step(torch.from_numpy(q).to(cuda), torch.from_numpy(kvn).to(cuda))
        ctx.sync()
        pool = ctx.read_blocks(np.arange(ctx.pool.shape[0])).cpu().numpy().view(np.uint16)
        table = ctx.table.cpu().numpy()
        reps = ctx.reps.cpu().numpy()
        sel = ctx.selected.cpu().numpy()
        got = out.float().cpu().numpy()
        for s in range(seqs):
            for l in range(layers):
                sl = s * layers + l
                tail_len = step % 32 + 1
                ids, want = _oracle_step(port, pool, table[sl], nb_before[sl], reps[sl],
                                         q[s, l], tail_before[sl], tail_len, qh, kh, budget,
                                         init, local, scale)
                assert np.array_equal(sel[sl][:, :ids.shape[1]], ids), (step, s, l)
                err = np.abs(got[s, l] - want).max()
                assert err <= tol[0] and cosine(got[s, l], want) >= tol[1], (step, s, l, err)
        if step == 31:  # sealed this step
            nb_after = ctx.num_sealed.cpu().numpy()
            assert (nb_after == nb_before + 1).all()
            assert (ctx.tail_len.cpu().numpy() == 0).all()
            assert (ctx.generation.cpu().numpy() == 1).all()
            new_tails = ctx.tail_block.cpu().numpy()
            assert len(set(new_tails.tolist()) | set(table[:, :nb0].ravel().tolist())) == \
                len(new_tails) + table[:, :nb0].size
            ring = ctx.query_ring.cpu().numpy()
            for sl in range(seqs * layers):
                assert table[sl, nb_before[sl]] == tail_before[sl]
                blk = pool[tail_before[sl]].reshape(-1)
                v, o, received = _reps_oracle(port, ring[sl], blk, qh, kh)
                got_v = reps[sl][:, :, nb_before[sl]]
                for h in range(qh):
                    mass = received[h]
                    if np.abs(got_v[h] - v[h]).max() > 1e-6:
                        # allowed only for a received-mass near-tie at the top-4 boundary
                        srt = np.sort(mass)[::-1]
                        assert abs(srt[3] - srt[4]) <= 1e-6 * max(1.0, abs(srt[3])), (sl, h)
    ctx.close()


def test_lifecycle_bytes_follow_reference_formula(pkg, port, cuda):
    """Token rows appended with the reference's synthetic byte formula
    (cpp/src/kv_lifecycle_main.cpp:34-35) are sealed into blocks whose bytes
    equal the reference's sealed store blocks; 31 tail tokens do not seal,
    the 32nd does; generation counts seals."""
    layers, qh, kh = 4, 16, 8
    tv = 2 * kh * D
    decode = 160
    ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=layers, seqs=1,
                            pool_blocks=layers * 8, table_blocks=8, budget_blocks=4,
                            init_blocks=1, local_blocks=1, device=cuda)
    for l in range(layers):
        ctx.prefill(0, l, 0)
    q = torch.zeros(1, layers, qh, D, device=cuda)
    for token in range(decode):
        vals = np.array([[(l * 1009 + token * 37 + v * 13) & 0xFFFF for v in range(tv)]
                         for l in range(layers)], np.uint16)
        ctx.step(q, torch.from_numpy(vals.view(np.int16)).to(cuda).view(1, layers, 2, kh, D))
        if token == 30:
            assert (ctx.num_sealed.cpu().numpy() == 0).all()
            assert (ctx.tail_len.cpu().numpy() == 31).all()
        if token == 31:
            assert (ctx.num_sealed.cpu().numpy() == 1).all()
            assert (ctx.tail_len.cpu().numpy() == 0).all()
    # the formula's bit patterns include FP16 NaNs, so only that bit may be set
    assert ctx.status_bits() & ~pkg.SA_DEV_NONFINITE == 0
    res = port.lifecycle_run(layers, qh, kh, D, 32, 32, decode, 0, with_store=True)
    store = res["store"].reshape(layers, res["capacity_blocks"], 32, tv)
    pool = ctx.read_blocks(np.arange(ctx.pool.shape[0])).cpu().numpy().view(np.uint16).reshape(-1, 32, tv)
    table = ctx.table.cpu().numpy()
    nb = ctx.num_sealed.cpu().numpy()
    gen = ctx.generation.cpu().numpy()
    assert (nb == decode // 32).all() and (gen == decode // 32).all()
    # the reference keeps 32 local tokens unsealed: its sealed blocks are our first ones
    for l in range(layers):
        for b in range(res["sealed_total"] // layers):
            assert np.array_equal(pool[table[l, b]], store[l, b]), (l, b)
    ctx.close()


def test_pool_exhaustion_sets_status_not_fault(pkg, cuda):
    ctx = pkg.DecodeContext(query_heads=4, kv_heads=4, layers=1, seqs=1, pool_blocks=2,
                            table_blocks=8, budget_blocks=2, init_blocks=0, local_blocks=1,
                            device=cuda)
    ctx.prefill(0, 0, 0)  # takes 1 block as the tail, 1 left free
    q = torch.zeros(1, 1, 4, D, device=cuda)
    kv = torch.zeros(1, 1, 2, 4, D, dtype=torch.float16, device=cuda)
    for _ in range(65):  # two seals wanted, one possible; the 65th append finds a full tail
        ctx.step(q, kv)
    bits = ctx.status_bits()
    assert bits & pkg.SA_DEV_POOL_EMPTY
    assert bits & pkg.SA_DEV_TAIL_FULL
    with pytest.raises(pkg.SparseKVError):
        ctx.sync()
    ctx.close()


def test_variable_context_batch_matches_oracle(pkg, port, cuda):
    """A batch whose sequences hold different numbers of sealed blocks (the
    batched paged-decode configuration): every (sequence, layer) selects over
    its own block count and attends over its own table."""
    qh, kh, layers, budget, init, local = 16, 8, 2, 12, 1, 3
    seq_nb = [14, 40, 27]
    seqs = len(seq_nb)
    rng = np.random.default_rng(5)
    g = torch.Generator().manual_seed(5)
    ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=layers, seqs=seqs,
                            pool_blocks=layers * sum(n + 3 for n in seq_nb),
                            table_blocks=max(seq_nb) + 2, budget_blocks=budget,
                            init_blocks=init, local_blocks=local, out_fp16=True, device=cuda)
    for s, nb in enumerate(seq_nb):
        for l in range(layers):
            phys = ctx.prefill(s, l, nb)
            ctx.write_blocks(phys[:nb], torch.randn(nb, 32, 2, kh, D, generator=g).half())
            ctx.build_reps(s, l, 0, nb, torch.randn(qh, nb * 32, D, generator=g).half().float().to(cuda))
    ctx.sync()
    scale = np.float32(1) / np.sqrt(np.float32(D))
    for step in range(3):
        q = rng.standard_normal((seqs, layers, qh, D), dtype=np.float32).astype(np.float16).astype(np.float32)
        kvn = rng.standard_normal((seqs, layers, 2, kh, D), dtype=np.float32).astype(np.float16)
        nb_before = ctx.num_sealed.cpu().numpy().copy()
        tail_before = ctx.tail_block.cpu().numpy().copy()
        out = ctx.step(torch.from_numpy(q).to(cuda), torch.from_numpy(kvn).to(cuda))
        ctx.sync()
        assert ctx.status_bits() == 0
        pool = ctx.read_blocks(np.arange(ctx.pool.shape[0])).cpu().numpy().view(np.uint16)
        table, reps, sel = ctx.table.cpu().numpy(), ctx.reps.cpu().numpy(), ctx.selected.cpu().numpy()
        counts = ctx.selected_count.cpu().numpy()
        got = out.float().cpu().numpy()
        for s in range(seqs):
            for l in range(layers):
                sl = s * layers + l
                assert nb_before[sl] == seq_nb[s]
                ids, want = _oracle_step(port, pool, table[sl], nb_before[sl], reps[sl], q[s, l],
                                         tail_before[sl], step + 1, qh, kh, budget, init, local, scale)
                assert (counts[sl] == min(budget, seq_nb[s])).all()
                assert np.array_equal(sel[sl][:, :ids.shape[1]], ids), (step, s, l)
                err = np.abs(got[s, l] - want).max()
                assert err <= 2e-3 and cosine(got[s, l], want) >= 0.99999, (step, s, l, err)
    ctx.close()


def test_kv_head_shards_reassemble_the_unsharded_step(pkg, cuda):
    """KV-head sharding (the long-context multi-GPU layout) on one device: two
    contexts holding KV heads [0, 4) and [4, 8) of the same sequence select
    the same blocks per KV head as the unsharded context, and their outputs,
    concatenated over heads (the all-gather's layout), equal its output."""
    import dataclasses

    from solidattention_repro_b200 import sharding, workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="shard-test", layers=2,
                            context_blocks=96, budget_blocks=20, hot_blocks=4)
    full, info = workloads.make_context(w, 8, cuda, seed=3)
    q, kv = workloads.decode_inputs(w, info, 4, cuda, seed=3)
    shards = []
    for r in range(2):
        sl = sharding.shard_kv_heads(w.kv_heads, 2, r)
        ctx, inf = workloads.make_context(w, 8, cuda, seed=3, kv_heads_slice=sl)
        qs, kvs = workloads.decode_inputs(w, inf, 4, cuda, seed=3, kv_heads_slice=sl)
        shards.append((sl, ctx, qs, kvs))
    for step in range(4):
        want = full.step(q[step], kv[step]).float().cpu().numpy()
        want_ids = full.selected.cpu().numpy()
        outs = []
        for (kh0, khn), ctx, qs, kvs in shards:
            outs.append(ctx.step(qs[step], kvs[step]).float().cpu().numpy())
            # selection group = one KV head: the shard's groups are the full context's
            assert np.array_equal(ctx.selected.cpu().numpy(), want_ids[:, kh0:kh0 + khn]), step
        got = sharding.assemble_heads(outs, w.group)
        assert got.shape == want.shape
        assert np.abs(got - want).max() <= 2e-3 and cosine(got.ravel(), want.ravel()) >= 0.999999
    for _, ctx, _, _ in shards:
        assert ctx.status_bits() == 0
        ctx.close()
    full.close()


def test_gather_over_peer_buffers_assembles_all_heads(pkg, cuda):
    """The attention epilogue's gather: two KV-head shards of one sequence
    (emulated ranks on one GPU, one stream) store their outputs into both
    ranks' gathered buffers; each buffer's slot then holds the full head set,
    equal to the unsharded context's output, for consecutive steps
    (alternating slots). The emulated ranks run the step's stages one call at
    a time -- both attentions before either wait -- so every wait is already
    satisfied when it runs (a decode step would wait inside its own seal
    kernel for a rank queued behind it)."""
    import dataclasses

    from solidattention_repro_b200 import sharding, workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg3"], name="gather-test", layers=3,
                            context_blocks=80, budget_blocks=16, hot_blocks=4)
    full, info = workloads.make_context(w, 8, cuda, seed=4)
    q, kv = workloads.decode_inputs(w, info, 3, cuda, seed=4)
    ranks = []
    for r in range(2):
        sl = sharding.shard_kv_heads(w.kv_heads, 2, r)
        ctx, inf = workloads.make_context(w, 8, cuda, seed=4, kv_heads_slice=sl)
        qs, kvs = workloads.decode_inputs(w, inf, 3, cuda, seed=4, kv_heads_slice=sl)
        ranks.append((ctx, qs, kvs))
    bufs = [ctx.gather_buffer(2)[0] for ctx, _, _ in ranks]
    for r, (ctx, _, _) in enumerate(ranks):
        ctx.gather_attach(r, bufs)
    with pytest.raises(pkg.SparseKVError):
        ranks[0][0].gather_wait()  # nothing gathered yet
    slots = set()
    for step in range(3):
        want = full.step(q[step], kv[step]).float().cpu().numpy()
        locals_ = []
        for ctx, qs, kvs in ranks:
            ctx.append(qs[step], kvs[step])
            ctx.select(qs[step])
            locals_.append(ctx.attend(qs[step]).float().cpu().numpy())
        for r, (ctx, _, _) in enumerate(ranks):
            got_t = ctx.gather_wait()
            ctx.seal()
            ctx.sync()
            slots.add(got_t.data_ptr() - bufs[r])
            got = got_t.float().cpu().numpy()
            assert np.array_equal(got, sharding.assemble_heads(locals_, w.group)), (step, r)
            assert np.abs(got - want).max() <= 2e-3 and \
                cosine(got.ravel(), want.ravel()) >= 0.999999, (step, r)
    assert len(slots) == 2  # consecutive attends alternate between the two slots
    for ctx, _, _ in ranks:
        assert ctx.status_bits() == 0
        ctx.close()
    full.close()


def test_recorded_gather_steps_replay_like_eager_steps(pkg, cuda):
    """The gather's slot parity and expected arrival count live on the device,
    so attention + gather-wait pairs recorded into a graph replay correctly:
    a one-rank gather (its own buffer, so no wait depends on another kernel)
    replays five recorded steps, then an eager sixth step's wait finds that
    step's output in the slot the host names."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg3"], name="gather-graph-test", layers=2,
                            context_blocks=48, budget_blocks=12, hot_blocks=2)
    steps = 6
    plain, info = workloads.make_context(w, steps, cuda, seed=12)
    with torch.cuda.stream(torch.cuda.Stream(cuda)):
        rec, _ = workloads.make_context(w, steps, cuda, seed=12)
    q, kv = workloads.decode_inputs(w, info, steps, cuda, seed=12)
    own, _ = rec.gather_buffer(1)
    rec.gather_attach(0, [own])
    outs = [rec.new_output() for _ in range(steps)]
    torch.cuda.synchronize(cuda)
    with rec.record():
        for s in range(steps - 1):
            rec.step(q[s], kv[s], outs[s])
            rec.gather_wait(view=False)
    rec.graph_launch()
    rec.step(q[steps - 1], kv[steps - 1], outs[steps - 1])
    gathered = rec.gather_wait()
    rec.sync()
    for s in range(steps):
        want = plain.step(q[s], kv[s])
        assert torch.equal(outs[s], want), s
    assert torch.equal(gathered.reshape(outs[-1].shape), outs[-1])
    for c in (rec, plain):
        assert c.status_bits() == 0
        c.close()


def test_recorded_gather_view_needs_an_even_attend_count(pkg, cuda):
    """A gathered-slot view handed out while recording is a fixed address in
    the graph, while every replay flips the device-side slot parity once per
    gathered attention: a recording with such a view and an odd number of
    gathered attentions is refused at graph_end; with an even number, a
    recorded consumer of the view reads the right step's outputs on every
    replay (checked over two replays against an unrecorded context)."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg3"], name="gather-parity-test", layers=2,
                            context_blocks=40, budget_blocks=10, hot_blocks=2)
    plain, info = workloads.make_context(w, 16, cuda, seed=21)
    side = torch.cuda.Stream(cuda)
    with torch.cuda.stream(side):
        rec, _ = workloads.make_context(w, 16, cuda, seed=21)
    q, kv = workloads.decode_inputs(w, info, 5, cuda, seed=21)
    own, _ = rec.gather_buffer(1)
    rec.gather_attach(0, [own])
    outs = rec.new_output()
    torch.cuda.synchronize(cuda)
    with pytest.raises(pkg.SparseKVError) as e:
        with rec.record():
            for s in range(5):
                rec.step(q[s], kv[s], outs)
                rec.gather_wait(view=(s == 4))
    assert e.value.status == pkg.SA_ERR_UNSUPPORTED
    # nothing of the refused recording ran; start the gather afresh
    rec.gather_attach(0, [own])
    dst = torch.empty((w.seqs, w.layers, w.query_heads, 128), dtype=torch.float16, device=cuda)
    with torch.cuda.stream(side), rec.record():
        for s in range(4):
            rec.step(q[s], kv[s], outs)
            view = rec.gather_wait(view=(s == 3))
        dst.copy_(view)  # a recorded consumer of the last step's slot
    for replay in range(2):
        with torch.cuda.stream(side):
            rec.graph_launch()
        side.synchronize()
        for s in range(4):
            want = plain.step(q[s], kv[s])
        plain.sync()
        assert torch.equal(dst, want.view(dst.shape)), replay
    for c in (rec, plain):
        assert c.status_bits() == 0
        c.close()


def test_gather_wait_gives_up_and_reports_timeout(pkg, cuda):
    """A gather wait whose arrivals never come (a rank that never attends)
    gives up at its bounded limit (about a second) and reports
    SA_DEV_TIMEOUT in the status word instead of hanging; the next
    synchronisation returns SA_ERR_TIMEOUT. Before that, a step's own wait
    (in its seal kernel) and an explicit wait after a standalone attention
    both pass."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg3"], name="gather-timeout-test", layers=1,
                            context_blocks=16, budget_blocks=8, hot_blocks=1)
    ctx, info = workloads.make_context(w, 4, cuda, seed=13)
    q, kv = workloads.decode_inputs(w, info, 2, cuda, seed=13)
    own, _ = ctx.gather_buffer(1)
    ctx.gather_attach(0, [own])
    ctx.step(q[0], kv[0])         # the step's seal kernel waits: the arrivals are there
    ctx.gather_wait(view=False)   # nothing left to wait for after a step
    assert ctx.sync() == 0
    ctx.attend(q[0])              # an attention of its own ...
    ctx.gather_wait(view=False)   # ... and its wait kernel
    assert ctx.sync() == 0
    ctx.close()
    # a two-rank gather whose second rank never attends (its buffer is a
    # plain allocation here): this rank's step waits for arrivals that never come
    ctx, info = workloads.make_context(w, 4, cuda, seed=13)
    own, nbytes = ctx.gather_buffer(2)
    absent = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    ctx.gather_attach(0, [own, absent.data_ptr()])
    ctx.step(q[1], kv[1])
    with pytest.raises(pkg.SparseKVError) as e:
        ctx.sync()
    assert e.value.status == pkg.SA_ERR_TIMEOUT
    assert ctx.status_bits() & pkg.SA_DEV_TIMEOUT
    ctx.close()


def test_dense_audit_matches_oracle_restatement(pkg, port, cuda):
    """sa_ctx_audit against the oracle's restatement of audit_dense_selection
    (pipeline_main.cpp:502-569: FP32 logits, expf, double denominator, the
    mass-ranked oracle set), per (seq-layer, KV head) over the context's own
    sealed blocks and open tail. Tolerance: the kernel computes the logits
    with fused multiply-adds and exp2 of log2e-scaled logits; with N(0, 1)
    keys and queries that moves a logit by about 5e-7 and a probability by
    the same relative amount, so rtol 2e-5 leaves a factor of 40. The host
    quality figures from the kernel's masses then equal the oracle's figures
    from its own masses, for the context's selection."""
    from solidattention_repro_b200 import quality

    qh, kh, layers, seqs, nb = 8, 2, 2, 2, 20
    budget, init, local = 8, 1, 2
    g = torch.Generator().manual_seed(11)
    ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=layers, seqs=seqs,
                            pool_blocks=seqs * layers * (nb + 3), table_blocks=nb + 2,
                            budget_blocks=budget, init_blocks=init, local_blocks=local,
                            out_fp16=False, device=cuda)
    for s in range(seqs):
        for l in range(layers):
            phys = ctx.prefill(s, l, nb)
            ctx.write_blocks(phys[:nb], torch.randn(nb, 32, 2, kh, D, generator=g).half())
    ctx.sync()
    rng = np.random.default_rng(3)
    for _ in range(5):  # a few tail tokens
        q = rng.standard_normal((seqs, layers, qh, D), dtype=np.float32)
        kvn = rng.standard_normal((seqs, layers, 2, kh, D), dtype=np.float32).astype(np.float16)
        ctx.append(torch.from_numpy(q).to(cuda), torch.from_numpy(kvn).to(cuda))
    q = rng.standard_normal((seqs, layers, qh, D), dtype=np.float32)
    ctx.select(torch.from_numpy(q).to(cuda))
    mass = ctx.audit(torch.from_numpy(q).to(cuda)).cpu().numpy()
    ctx.sync()
    pool = ctx.read_blocks(np.arange(ctx.pool.shape[0])).cpu().numpy()
    table, tails = ctx.table.cpu().numpy(), ctx.tail_block.cpu().numpy()
    tl = ctx.tail_len.cpu().numpy()
    selected, counts = ctx.selected.cpu().numpy(), ctx.selected_count.cpu().numpy()
    groups = selected.shape[1]
    grp = qh // kh
    want_mass, want_recall = [], []
    for sl in range(seqs * layers):
        for h in range(kh):
            keys = np.concatenate([pool[table[sl, :nb]][:, :, 0, h].reshape(-1, D),
                                   pool[tails[sl]][:tl[sl], 0, h]])
            qq = q.reshape(-1, qh, D)[sl, h * grp:(h + 1) * grp]
            want = port.dense_block_mass(keys, qq, 32, 1.0 / np.sqrt(D))
            assert want.shape == (nb + 1,)
            np.testing.assert_allclose(mass[sl, h, :nb], want[:nb], rtol=2e-5, atol=1e-9)
            assert mass[sl, h, -1] == pytest.approx(want[nb], rel=2e-5)
            assert (mass[sl, h, nb:-1] == 0).all()
            assert abs(mass[sl, h].sum() - 1.0) <= 1e-5
            gi = h * groups // kh
            a, r = port.audit_selection(want[:nb], selected[sl, gi, :counts[sl, gi]], budget,
                                        init, local, want[nb])
            want_mass.append(a)
            want_recall.append(r)
    res = quality.selection_quality(mass, selected, counts, ctx.num_sealed.cpu().numpy(),
                                    budget, init, local)
    assert res["units"] == seqs * layers * kh
    assert res["selected_mass"] == pytest.approx(np.mean(want_mass), rel=2e-5)
    assert res["oracle_recall"] == pytest.approx(np.mean(want_recall), abs=1e-12)
    ctx.close()


def test_selection_beats_random_on_planted_blocks(pkg, cuda):
    """The audit's quality figures on a cfg2-shaped context (two layers). The
    configured plant (+0.5 * unit q_hat on keys of norm ~11) lifts a hot
    block's representative score by about 3 against score noise of about 6,
    and N(0,1) keys give a near-uniform dense attention, so the figures are
    checked against random selection: hot blocks are recalled at least twice
    as often as a random pick of the dynamic blocks would, the oracle set
    clearly more often, and the selected mass is above the uniform share."""
    import dataclasses

    from solidattention_repro_b200 import quality, workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="quality-test", layers=2)
    ctx, info = workloads.make_context(w, 8, cuda, seed=2)
    q, kv = workloads.decode_inputs(w, info, 4, cuda, seed=2)
    for s in range(4):
        ctx.step(q[s], kv[s])
    ctx.select(q[3])
    mass = ctx.audit(q[3])
    ctx.sync()
    hot = info["hot"].reshape(w.seqs * w.layers, w.kv_heads, -1)
    res = quality.selection_quality(mass.cpu().numpy(), ctx.selected.cpu().numpy(),
                                    ctx.selected_count.cpu().numpy(),
                                    ctx.num_sealed.cpu().numpy(), w.budget_blocks,
                                    w.init_blocks, w.local_blocks, hot)
    print(res)
    nb = int(ctx.num_sealed.cpu().numpy()[0])
    forced = w.init_blocks + w.local_blocks
    dyn_rate = (w.budget_blocks - forced) / (nb - forced)  # random pick of a dynamic block
    oracle_random = (forced + (w.budget_blocks - forced) * dyn_rate) / w.budget_blocks
    assert res["units"] == w.layers * w.kv_heads
    assert res["hot_recall"] >= 2 * dyn_rate
    assert res["oracle_recall"] >= 1.3 * oracle_random
    assert w.budget_blocks / (nb + 1) < res["selected_mass"] <= 1.0 + 1e-5
    ctx.close()


def test_step_host_matches_device_step_pinned_and_pageable(pkg, cuda):
    """sa_ctx_step_host, the end-to-end call of a host decode loop, with
    pinned mapped buffers (used in place: K/V read and output written over
    the bus, status mirrored by the seal) and with pageable buffers (staged
    copies): both equal the device-pointer step bit for bit, across a seal."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="host-step-test", layers=2,
                            context_blocks=40, budget_blocks=12, hot_blocks=2)
    steps = 34
    ctxs = [workloads.make_context(w, steps, cuda, seed=6) for _ in range(3)]
    q, kv = workloads.decode_inputs(w, ctxs[0][1], steps, cuda, seed=6)
    q_pin = torch.empty(q[0].shape, dtype=torch.float32, pin_memory=True)
    kv_pin = torch.empty(kv[0].shape, dtype=torch.float16, pin_memory=True)
    out_pin = torch.empty(ctxs[0][0].new_output().shape, dtype=torch.float16, pin_memory=True)
    for s in range(steps):
        want = ctxs[0][0].step(q[s], kv[s]).cpu().numpy()
        q_pin.copy_(q[s].cpu())
        kv_pin.copy_(kv[s].cpu())
        ctxs[1][0].step_host(q_pin, kv_pin, out_pin)
        q_np, kv_np = q[s].cpu().numpy().copy(), kv[s].cpu().numpy().copy()
        out_np = np.empty(want.shape, np.float16)
        ctxs[2][0].step_host(q_np, kv_np, out_np)
        assert np.array_equal(out_pin.numpy(), want), s
        assert np.array_equal(out_np, want), s
    for c, _ in ctxs:
        assert c.status_bits() == 0
    ref = ctxs[0][0]
    for c, _ in ctxs[1:]:
        for name in ("num_sealed", "tail_len", "tail_block", "generation", "selected"):
            assert torch.equal(getattr(c, name), getattr(ref, name)), name
    assert (ref.generation.cpu().numpy() == 1).all()  # the 32nd append sealed
    for c, _ in ctxs:
        c.close()


def test_recorded_steps_replay_like_eager_steps(pkg, cuda):
    """sa_ctx_graph_begin / _end / _launch: decode steps recorded into a CUDA
    graph and replayed give the eager steps' outputs and state bit for bit,
    across a seal; synchronising calls are refused while recording."""
    import dataclasses

    from solidattention_repro_b200 import SparseKVError, workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="graph-step-test", layers=2,
                            context_blocks=40, budget_blocks=12, hot_blocks=2)
    steps = 34
    eager, info = workloads.make_context(w, steps, cuda, seed=9)
    side = torch.cuda.Stream(cuda)
    with torch.cuda.stream(side):
        rec, _ = workloads.make_context(w, steps, cuda, seed=9)
    q, kv = workloads.decode_inputs(w, info, steps, cuda, seed=9)
    outs = [rec.new_output() for _ in range(steps)]
    torch.cuda.synchronize(cuda)
    launches = rec.launches
    with rec.record():
        for s in range(steps):
            rec.step(q[s], kv[s], outs[s])
        with pytest.raises(SparseKVError):
            rec.sync()
    assert rec.launches == launches  # recording launches nothing
    assert int(rec.tail_len.cpu()[0]) == int(eager.tail_len.cpu()[0])
    rec.graph_launch()
    rec.sync()
    want = [eager.step(q[s], kv[s]) for s in range(steps)]
    eager.sync()
    for s in range(steps):
        assert torch.equal(outs[s], want[s]), s
    assert rec.launches - launches == eager.launches - launches
    for name in ("num_sealed", "tail_len", "tail_block", "generation", "selected", "reps"):
        assert torch.equal(getattr(rec, name), getattr(eager, name)), name
    assert (eager.generation.cpu().numpy() == 1).all()  # the 32nd append sealed
    for c in (rec, eager):
        assert c.status_bits() == 0
        c.close()


def test_stage_calls_match_the_fused_step_across_seals(pkg, cuda):
    """The stage calls (sa_ctx_append, _select, _attend, _seal: the token is
    counted at once and the seal runs its full pass) and the fused step (the
    token pending until the seal, which commits alone unless the append
    flagged a filled tail) give the same outputs and state bit for bit, also
    when the two are interleaved on one context, across two seals."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="stage-step-test", layers=2,
                            context_blocks=40, budget_blocks=12, hot_blocks=2)
    steps = 70
    fused, info = workloads.make_context(w, steps, cuda, seed=11)
    mixed, _ = workloads.make_context(w, steps, cuda, seed=11)
    q, kv = workloads.decode_inputs(w, info, steps, cuda, seed=11)
    for s in range(steps):
        want = fused.step(q[s], kv[s])
        if s % 3 == 1:
            got = mixed.step(q[s], kv[s])
        else:
            mixed.append(q[s], kv[s])
            mixed.select(q[s])
            got = mixed.attend(q[s])
            mixed.seal()
        assert torch.equal(got, want), s
    for name in ("num_sealed", "tail_len", "tail_block", "generation", "selected", "reps", "table"):
        assert torch.equal(getattr(mixed, name), getattr(fused, name)), name
    assert (fused.generation.cpu().numpy() == 2).all()
    for c in (fused, mixed):
        assert c.status_bits() == 0
        c.close()


def test_slot_table_follows_the_selection_bit_exact(pkg, port, cuda):
    """sa_ctx_slot_correct over a decode loop: a resident window that starts
    empty and follows each step's selection equals the oracle's
    compare_prediction restatement bit for bit (slots, misses, replacement
    slots, hit/miss counts)."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg2"], name="slots-test", layers=2,
                            context_blocks=96, budget_blocks=24, hot_blocks=4)
    ctx, info = workloads.make_context(w, 40, cuda, seed=8)
    q, kv = workloads.decode_inputs(w, info, 36, cuda, seed=8)
    slots = ctx.new_slots()
    ref = slots.cpu().numpy().reshape(-1, w.budget_blocks)
    total_hits = 0
    for s in range(36):
        ctx.step(q[s], kv[s])
        misses, replace, stats = ctx.slot_correct(slots)
        ctx.sync()
        sel = ctx.selected.cpu().numpy().reshape(-1, w.budget_blocks)
        cnt = ctx.selected_count.cpu().numpy().reshape(-1)
        ref, mi, re, st = port.slot_correct(sel, cnt, ref)
        assert np.array_equal(slots.cpu().numpy().reshape(ref.shape), ref), s
        assert np.array_equal(misses.cpu().numpy().reshape(mi.shape), mi), s
        assert np.array_equal(replace.cpu().numpy().reshape(re.shape), re), s
        assert np.array_equal(stats.cpu().numpy().reshape(st.shape), st), s
        if s > 0:
            total_hits += int(st[:, 0].sum())
    assert total_hits > 0  # consecutive selections overlap (the forced blocks at least)
    assert ctx.status_bits() == 0
    ctx.close()


def test_store_blocks_round_trip_reference_format(pkg, cuda):
    """sa_ctx_import_blocks / sa_ctx_export_blocks: logical blocks move between
    the head-major pool and the reference's store rows [32][2][KH][128], from
    device memory and from pinned host memory, equal to the token-major
    conversion of the pool; pageable host memory is refused, not touched."""
    qh, kh, nb = 8, 4, 12
    ctx = pkg.DecodeContext(query_heads=qh, kv_heads=kh, layers=2, seqs=2,
                            pool_blocks=4 * (nb + 2), table_blocks=nb + 1, budget_blocks=4,
                            init_blocks=1, local_blocks=1, device=cuda)
    g = torch.Generator().manual_seed(9)
    for s in range(2):
        for l in range(2):
            ctx.prefill(s, l, nb)
    store = torch.randn(nb, 32, 2, kh, D, generator=g).half()
    ctx.import_blocks(1, 0, 0, store.to(cuda))                  # from device memory
    pinned = torch.randn(5, 32, 2, kh, D, generator=g).half().pin_memory()
    ctx.import_blocks(1, 1, 3, pinned)                          # from pinned host memory
    ctx.sync()
    table = ctx.table.cpu().numpy()
    assert torch.equal(ctx.read_blocks(table[2, :nb]).cpu(), store)
    assert torch.equal(ctx.read_blocks(table[3, 3:8]).cpu(), pinned)
    assert torch.equal(ctx.export_blocks(1, 0, 0, nb).cpu(), store)
    host = torch.empty(5, 32, 2, kh, D, dtype=torch.float16).pin_memory()
    ctx.export_blocks(1, 1, 3, 5, host)
    ctx.sync()
    assert torch.equal(host, pinned)
    with pytest.raises(pkg.SparseKVError):
        ctx.import_blocks(0, 0, 0, torch.zeros(1, 32, 2, kh, D, dtype=torch.float16))  # pageable
    with pytest.raises(pkg.SparseKVError):
        ctx.export_blocks(0, 0, nb, 2)  # beyond the table
    assert ctx.status_bits() == 0
    ctx.close()


def test_step_raw_fuses_qk_norm_rope_into_the_append(pkg, port, cuda):
    """sa_ctx_step_raw (q/k norm + RoPE + FP16 pack fused with the append) equals
    sa_ctx_step fed with the oracle's transformed queries and keys: the query
    ring, the packed K (plus one FP16 ulp) and the attention output within
    the float tolerance of CUDA's vs the C library's powf/cosf/sinf/rsqrt,
    V exactly, and the selections identical."""
    import dataclasses

    from solidattention_repro_b200 import workloads

    w = dataclasses.replace(workloads.CONFIGS["cfg3"], name="raw-test", layers=2, seqs=2,
                            context_blocks=48, budget_blocks=12, hot_blocks=2)
    raw, _ = workloads.make_context(w, 8, cuda, seed=5)
    ref, _ = workloads.make_context(w, 8, cuda, seed=5)
    rng = np.random.default_rng(12)
    qw = (1 + 0.1 * rng.standard_normal((w.layers, 128))).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal((w.layers, 128))).astype(np.float32)
    positions = np.array([48 * 32, 48 * 32 + 7000], np.int32)
    theta, eps = 1.0e6, 1e-6
    for step in range(3):
        q = rng.standard_normal((w.seqs, w.layers, w.query_heads, 128), dtype=np.float32)
        k = rng.standard_normal((w.seqs, w.layers, w.kv_heads, 128), dtype=np.float32)
        v = rng.standard_normal((w.seqs, w.layers, w.kv_heads, 128), dtype=np.float32)
        tl = raw.tail_len.cpu().numpy().copy()
        tb = raw.tail_block.cpu().numpy().copy()
        got = raw.step_raw(*(torch.from_numpy(a).to(cuda) for a in (q, k, v, qw, kw)),
                           torch.from_numpy(positions + step).to(cuda), theta, eps)
        qt, kt = q.copy(), k.copy()
        for s in range(w.seqs):
            for l in range(w.layers):
                qt[s, l] = port.head_norm_rope(q[s, l], qw[l], positions[s] + step, theta, eps)
                kt[s, l] = port.head_norm_rope(k[s, l], kw[l], positions[s] + step, theta, eps)
        kv = np.stack([kt, v], 2).astype(np.float16)  # [S, L, 2, KH, 128]
        want = ref.step(torch.from_numpy(qt).to(cuda), torch.from_numpy(kv).to(cuda))
        ref.sync()
        raw.sync()
        g, wn = got.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.abs(g - wn).max() <= 2e-3 and cosine(g.ravel(), wn.ravel()) >= 0.99999, step
        assert np.array_equal(raw.selected.cpu().numpy(), ref.selected.cpu().numpy()), step
        ring = raw.query_ring.cpu().numpy()
        pool = raw.pool.cpu().numpy()
        for s in range(w.seqs):
            for l in range(w.layers):
                sl = s * w.layers + l
                # an ulp of CUDA's vs the C library's powf moves the FP32 angle
                # by ~1e-7 * position radians
                tol = (1e-5 + 2e-7 * float(positions[s] + step)) * np.abs(qt[s, l]).max()
                np.testing.assert_allclose(ring[sl, :, tl[sl]], qt[s, l], rtol=1e-5, atol=tol)
                # the packed K: the same angle tolerance, plus one FP16 ulp
                k16 = pool[tb[sl], :, 0, tl[sl]].astype(np.float32)
                ktol = (1e-5 + 2e-7 * float(positions[s] + step)) * np.abs(kt[s, l]).max(1,
                                                                                   keepdims=True)
                ulp = np.abs(kt[s, l]) * 2.0 ** -10 + 2.0 ** -24
                assert (np.abs(k16 - kt[s, l]) <= ktol + ulp).all()
                assert np.array_equal(pool[tb[sl], :, 1, tl[sl]], v[s, l].astype(np.float16))
    assert raw.status_bits() == 0
    raw.close()
    ref.close()
