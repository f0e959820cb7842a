"""GPU parity of the stateless sm_100a kernels against the CPU oracle.

Tolerances (from the reference's gates and the path's contract):
* attention, FP32 output: max-abs <= 2e-5 and cosine >= 0.999999
  (cpp/src/attention_main.cpp:265-270);
* attention, FP16 output: max-abs <= 2e-3 and cosine >= 0.99999;
* selection: scores bit-identical, block ids identical;
* representatives: offsets identical except near-ties of received mass
  (gap < 1e-6 relative), values within 1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, fp16_normal

pytestmark = pytest.mark.gpu

SCALE = np.float32(1.0) / np.sqrt(np.float32(128))


def _t(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(dev)


# ------------------------------------------------------------- attention

def test_c1_fixture_attention_matches_reference_gate(pkg, port, cuda):
    kv, q = port.c1_fixture()
    want = port.attention(kv, q, 128, 16, 8, 128, np.float32(0.08838834764831845))
    got = pkg.attention(_t(kv, cuda, torch.int16), _t(q, cuda), 128, 16, 8, 128,
                        0.08838834764831845).cpu().numpy()
    assert np.abs(got - want).max() <= 2e-5
    assert cosine(got, want) >= 0.999999


@pytest.mark.parametrize("tokens", [1, 7, 31, 32, 33, 100, 512, 4100])
@pytest.mark.parametrize("qh,kh", [(16, 8), (32, 8), (4, 1), (8, 8), (64, 8)])
def test_packed_attention_fp32(pkg, port, cuda, tokens, qh, kh):
    rng = np.random.default_rng(tokens * 131 + qh * 7 + kh)
    kv = fp16_normal(rng, tokens * 2 * kh * 128)
    q = rng.standard_normal(qh * 128, dtype=np.float32)
    want = port.attention(kv, q, tokens, qh, kh, 128, SCALE)
    got = pkg.attention(_t(kv, cuda, torch.int16), _t(q, cuda), tokens, qh, kh, 128,
                        float(SCALE)).cpu().numpy()
    assert np.abs(got - want).max() <= 2e-5, np.abs(got - want).max()
    assert cosine(got, want) >= 0.999999


@pytest.mark.parametrize("tokens", [512, 2048 + 17])
def test_packed_attention_fp16_output(pkg, port, cuda, tokens):
    rng = np.random.default_rng(tokens)
    kv = fp16_normal(rng, tokens * 2 * 8 * 128)
    q = fp16_normal(rng, 32 * 128).view(np.float16).astype(np.float32)
    want = port.attention(kv, q, tokens, 32, 8, 128, SCALE)
    got = pkg.attention(_t(kv, cuda, torch.int16), _t(q, cuda), tokens, 32, 8, 128, float(SCALE),
                        out_fp16=True).float().cpu().numpy()
    assert np.abs(got - want).max() <= 2e-3
    assert cosine(got, want) >= 0.99999


def test_attention_rejects_what_the_reference_rejects(pkg, cuda):
    kv = torch.zeros(64 * 2 * 8 * 128, dtype=torch.int16, device=cuda)
    q = torch.zeros(16 * 128, device=cuda)
    with pytest.raises(pkg.SparseKVError) as e:
        pkg.attention(kv, q, 0, 16, 8, 128)
    assert e.value.status == pkg.SA_ERR_INVALID_ARG
    with pytest.raises(pkg.SparseKVError) as e:
        pkg.attention(kv, q, 64, 12, 8, 128)
    assert e.value.status == pkg.SA_ERR_INVALID_ARG
    with pytest.raises(pkg.SparseKVError) as e:
        pkg.attention(kv, q, 64, 16, 8, 64)
    assert e.value.status == pkg.SA_ERR_UNSUPPORTED


# ------------------------------------------------------------- selection

def _reps_dim_major(reps_ref):
    """[qh][blocks][d] -> [qh][d][blocks]"""
    return np.ascontiguousarray(np.transpose(reps_ref, (0, 2, 1)))


@pytest.mark.parametrize("qh,group,blocks,budget,init,local", [
    (16, 16, 16, 4, 1, 1),       # the C2.1 shared mode
    (16, 2, 512, 64, 1, 4),      # per KV head, Qwen3-0.6B shape
    (32, 4, 1024, 128, 1, 4),    # per KV head, Qwen3-8B shape
    (32, 4, 4096, 256, 1, 8),    # long context (a grid small enough for the deep variant)
    (32, 4, 16384, 256, 1, 8),   # the maximum: 1024 CTAs, the occupancy-bound variant
    (4, 4, 1, 1, 0, 1),          # single block
    (8, 2, 50, 50, 1, 1),        # budget == blocks
    (8, 2, 50, 5, 2, 3),         # everything forced
    (8, 8, 37, 9, 0, 0),         # no forced blocks, ragged count
    (32, 32, 1000, 17, 3, 2),    # shared mode, several CTAs
])
@pytest.mark.parametrize("layout", ["reference", "dim_major"])
def test_select_bit_exact(pkg, port, cuda, qh, group, blocks, budget, init, local, layout):
    rng = np.random.default_rng(blocks * 10 + qh + budget)
    q = rng.standard_normal((qh, 128), dtype=np.float32)
    reps = rng.standard_normal((qh, blocks, 128), dtype=np.float32) * np.float32(0.5)
    want_ids, want_scores = port.select_grouped(q, reps, qh, group, blocks, 128, budget, init, local)
    dev_reps = reps if layout == "reference" else _reps_dim_major(reps)
    ids, scores = pkg.select_shared_blocks(_t(q, cuda), _t(dev_reps, cuda), qh, blocks, 128,
                                           budget, init, local, group=group, layout=layout)
    assert np.array_equal(scores.cpu().numpy().view(np.uint32), want_scores.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), want_ids)


def test_select_ties_go_to_lower_block(pkg, port, cuda):
    rng = np.random.default_rng(5)
    qh, blocks = 8, 300
    base = rng.standard_normal((qh, 10, 128), dtype=np.float32)
    reps = np.ascontiguousarray(base[:, rng.integers(0, 10, blocks)])  # many exact duplicates
    q = rng.standard_normal((qh, 128), dtype=np.float32)
    for budget in (3, 40, 97):
        want, _ = port.select_grouped(q, reps, qh, 2, blocks, 128, budget, 1, 1)
        ids, _ = pkg.select_shared_blocks(_t(q, cuda), _t(reps, cuda), qh, blocks, 128, budget,
                                          1, 1, group=2)
        assert np.array_equal(ids.cpu().numpy(), want)


def test_select_signed_zero_and_equal_scores(pkg, port, cuda):
    qh, blocks = 2, 64
    q = np.zeros((qh, 128), np.float32)   # every score is +-0: all tie
    reps = np.random.default_rng(0).standard_normal((qh, blocks, 128), dtype=np.float32)
    reps[:, ::2] *= -1
    want, _ = port.select_grouped(q, reps, qh, qh, blocks, 128, 10, 1, 1)
    ids, _ = pkg.select_shared_blocks(_t(q, cuda), _t(reps, cuda), qh, blocks, 128, 10, 1, 1)
    assert np.array_equal(ids.cpu().numpy(), want)


@pytest.mark.parametrize("blocks", [1200, 5000])  # order keys in shared memory / from L2
@pytest.mark.parametrize("case", ["crowded_bucket", "infinite_score", "two_values",
                                  "nested_scales"])
def test_select_top_k_adversarial_scores(pkg, port, cuda, case, blocks):
    """Adversarial score sets for the top-k: two far outliers above
    near-equal scores (a second bucket level), an infinite score (an
    overflowing range), scores of only two values (more equal keys at the
    threshold than can be ranked directly), and outliers nested at four
    scales above near-equal scores (more bucket levels than the linear
    select takes, so the radix select finishes)."""
    rng = np.random.default_rng({"crowded_bucket": 1, "infinite_score": 2, "two_values": 3,
                                 "nested_scales": 4}[case])
    qh, budget = 4, 100
    q = rng.standard_normal((qh, 128), dtype=np.float32)
    base = rng.standard_normal((qh, 1, 128), dtype=np.float32)
    if case == "two_values":
        reps = np.repeat(base, blocks, axis=1)
        reps[:, ::3] = -reps[:, ::3]
    else:
        reps = base + rng.standard_normal((qh, blocks, 128), dtype=np.float32) * np.float32(1e-4)
        reps[:, 7] *= 1e4
        reps[:, 900] *= -1e4
        if case == "infinite_score":
            reps[:, 33] = np.float32(1e30) * np.sign(q)
        if case == "nested_scales":
            for b, f in ((11, 1e6), (12, 3e3), (13, 3.0), (14, 1e6), (15, 3e3)):
                reps[:, b] *= np.float32(f)
    reps = np.ascontiguousarray(reps.astype(np.float32))
    want, _ = port.select_grouped(q, reps, qh, qh, blocks, 128, budget, 1, 2)
    ids, _ = pkg.select_shared_blocks(_t(q, cuda), _t(reps, cuda), qh, blocks, 128, budget, 1, 2)
    assert np.array_equal(ids.cpu().numpy(), want)


def test_select_rejects_what_the_reference_rejects(pkg, cuda):
    q = torch.zeros(4, 128, device=cuda)
    reps = torch.zeros(4, 8, 128, device=cuda)
    for args in [(4, 8, 128, 9, 1, 1), (4, 8, 128, 0, 0, 0), (4, 8, 128, 2, 2, 1), (4, 0, 128, 1, 0, 0)]:
        with pytest.raises(pkg.SparseKVError) as e:
            pkg.select_shared_blocks(q, reps, *args)
        assert e.value.status == pkg.SA_ERR_INVALID_ARG


# ------------------------------------------------------- representatives

def _offsets_gap_aware(got_off, want_off, received, tokens_per_head, topk, rel=1e-6):
    """Offsets equal except where the swapped tokens' received masses nearly tie."""
    qh, blocks, _ = want_off.shape
    flips = 0
    for h in range(qh):
        for b in range(blocks):
            g, w = list(got_off[h, b]), list(want_off[h, b])
            if g == w:
                continue
            mass = received[h, b * 32:(b + 1) * 32]
            gs, ws = [float(mass[i]) for i in g], [float(mass[i]) for i in w]
            assert np.allclose(sorted(gs), sorted(ws), rtol=rel, atol=1e-7), (h, b, g, w)
            flips += 1
    return flips


def test_c21_kat_on_gpu(pkg, port, cuda):
    """The reference's C2.1 known answer: hash 7873450381430813043, blocks [0, 8, 13, 15]."""
    kv, pq, q = port.c21_fixture()
    vals, offs = pkg.build_local_causal_representatives(_t(pq, cuda), _t(kv, cuda, torch.int16),
                                                        512, 16, 8, 128, 32, 32, 4)
    offs = offs.cpu().numpy().astype(np.int64)
    want_vals, want_offs = port.build_representatives(pq, kv, 512, 16, 8, 128, 32, 32, 4)
    if port.fnv_offsets(offs) != 7873450381430813043:
        # only an expf last-bit near-tie may differ; prove it is one
        import ctypes as C
        received = np.zeros(16 * 512, np.float32)
        vv = np.zeros(16 * 16 * 128, np.float32)
        oo = np.zeros(16 * 16 * 4, np.int64)
        port.lib.sao_build_representatives.argtypes = [C.c_void_p] * 2 + [C.c_size_t] * 7 + [C.c_void_p] * 3
        port.lib.sao_build_representatives(pq.ctypes.data, kv.ctypes.data, 512, 16, 8, 128, 32, 32, 4,
                                           vv.ctypes.data, oo.ctypes.data, received.ctypes.data)
        _offsets_gap_aware(offs, want_offs, received.reshape(16, 512), 512, 4)
    ids, _ = pkg.select_shared_blocks(_t(q, cuda), vals.contiguous(), 16, 16, 128, 4, 1, 1)
    assert ids.cpu().numpy().tolist() == [[0, 8, 13, 15]]
    assert np.abs(vals.cpu().numpy() - want_vals).max() <= 1e-6


@pytest.mark.parametrize("tokens,qh,kh,window,topk", [
    (32, 32, 8, 32, 4),      # the online-seal call (cpp/src/online_seal_main.cpp:41)
    (64, 16, 8, 32, 4),
    (96, 4, 1, 5, 3),
    (64, 8, 2, 1, 1),        # window 1: every key receives exactly its own query's mass
    (160, 8, 8, 64, 32),
    (32, 2, 1, 17, 7),
])
def test_representatives_match_oracle(pkg, port, cuda, tokens, qh, kh, window, topk):
    import ctypes as C
    rng = np.random.default_rng(tokens + qh + window)
    kv = fp16_normal(rng, tokens * 2 * kh * 128)
    pq = fp16_normal(rng, qh * tokens * 128).view(np.float16).astype(np.float32)
    vals, offs = pkg.build_local_causal_representatives(_t(pq, cuda), _t(kv, cuda, torch.int16),
                                                        tokens, qh, kh, 128, 32, window, topk)
    blocks = tokens // 32
    received = np.zeros(qh * tokens, np.float32)
    want_vals = np.zeros(qh * blocks * 128, np.float32)
    want_offs = np.zeros(qh * blocks * topk, np.int64)
    port.lib.sao_build_representatives.argtypes = [C.c_void_p] * 2 + [C.c_size_t] * 7 + [C.c_void_p] * 3
    assert port.lib.sao_build_representatives(
        pq.ctypes.data, kv.ctypes.data, tokens, qh, kh, 128, 32, window, topk,
        want_vals.ctypes.data, want_offs.ctypes.data, received.ctypes.data) == 0
    got_offs = offs.cpu().numpy().astype(np.int64)
    _offsets_gap_aware(got_offs, want_offs.reshape(qh, blocks, topk),
                       received.reshape(qh, tokens), tokens, topk)
    same = (got_offs == want_offs.reshape(qh, blocks, topk)).all(axis=2)
    got_vals = vals.cpu().numpy()
    want_vals = want_vals.reshape(qh, blocks, 128)
    assert np.abs(got_vals[same] - want_vals[same]).max(initial=0) <= 1e-6
    if window == 1:
        assert np.allclose(received, 1.0)


# ------------------------------------------------------------ pack / backend

def test_pack_kv_fp16_is_rne(pkg, port, cuda):
    rng = np.random.default_rng(3)
    k = rng.standard_normal(1024, dtype=np.float32) * 3
    v = rng.standard_normal(1024, dtype=np.float32)
    k[:8] = [1.9999, 0.49999, 65519, 65520, 1e-8, 6e-8, -0.0, 2 ** -25]
    packed = torch.zeros(4 * 2048, dtype=torch.int16, device=cuda)
    pkg.pack_kv_fp16(packed, _t(k, cuda), _t(v, cuda), 2)
    row = packed.view(4, 2048)[2].cpu().numpy().view(np.uint16)
    with np.errstate(over="ignore"):  # 65520 rounds to +inf on purpose
        k_half = k.astype(np.float16)
    assert np.array_equal(row[:1024], k_half.view(np.uint16))
    assert np.array_equal(row[1024:], v.astype(np.float16).view(np.uint16))
    assert np.array_equal(row[:1024], port.float_to_half_rne(k))


def test_backend_variants(pkg, port):
    kv, q = port.c1_fixture()
    want = port.attention(kv, q, 128, 16, 8, 128, np.float32(0.08838834764831845)).ravel()
    be = pkg.Backend(0)
    assert be.name() == "b200-sm100a"
    out, t = be.attention(kv, q, 128, 16, 8, 128, 0.08838834764831845)
    assert np.abs(out - want).max() <= 2e-5 and t["kernel_ms"] > 0
    chk, _ = be.attention(kv, q, 128, 16, 8, 128, 0.08838834764831845, consume=True)
    ref_chk = float(np.sum(want.astype(np.float64) * (1 + (np.arange(want.size) % 17) * 1e-3)))
    assert abs(float(chk[0]) - ref_chk) <= 1e-4
    data = np.arange(4096, dtype=np.uint8)
    checksum, _ = be.execute(data, 0x5a)
    assert checksum == int((data ^ 0x5a).astype(np.uint64).sum())
    be.close()


# ------------------------------------------------------------- streaming probe

def test_streaming_probe_modes_read_the_same_bytes(pkg, cuda):
    """sa_probe_stream: the per-lane cp.async and the bulk-copy readers fold
    the same words of the same entries (the sink of every CTA agrees), and no
    bounded mbarrier wait gives up."""
    import ctypes as C

    lib = pkg.load()
    pool_entries, n = 512, 1000
    g = torch.Generator().manual_seed(3)
    pool = torch.randint(0, 256, (pool_entries * 16384,), dtype=torch.uint8, generator=g).to(cuda)
    ids = torch.randint(0, pool_entries, (n,), dtype=torch.int32, generator=g).to(cuda)
    stream = torch.cuda.current_stream(cuda)
    sinks = []
    for mode in (0, 1):
        sink = torch.zeros(1024, dtype=torch.int64, device=cuda)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        rc = lib.sa_probe_stream(C.c_void_p(pool.data_ptr()), pool_entries,
                                 C.c_void_p(ids.data_ptr()), n, mode, C.c_void_p(sink.data_ptr()),
                                 C.c_void_p(status.data_ptr()), C.c_void_p(stream.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        sinks.append(sink.cpu())
    assert torch.equal(sinks[0], sinks[1])
    assert bool(sinks[0].ne(0).any())
