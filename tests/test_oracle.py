"""The CPU oracle against the reference's own outputs and published answers.

* golden_ref.npz: outputs of the reference's C++ (compiled from its sources)
  on seeded cases -- the C restatement must match them bit for bit;
* the reference's published known answers (C2.1 selection, P1.3b.0 lifecycle);
* python_twins.json: the reference's Python twins on their own test inputs;
* when oracle/_ref is built, the restatement against the reference directly.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import cases  # noqa: E402

from conftest import cosine  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "golden_ref.npz")


@pytest.fixture(scope="module")
def twins():
    return json.loads((GOLDEN / "python_twins.json").read_text())


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# --------------------------------------------- golden vectors of the reference

@pytest.mark.parametrize("i", range(len(cases.ATTENTION)))
def test_attention_matches_reference_outputs(port, golden, i):
    kv, q, tokens, qh, kh = cases.attention_case(i)
    assert cases.digest(kv, q) == str(golden[f"attn{i}_sha"])
    got = port.attention(kv, q, tokens, qh, kh, 128, cases.SCALE).ravel()
    assert np.array_equal(bits(got), bits(golden[f"attn{i}_out"]))


@pytest.mark.parametrize("i", range(len(cases.SELECTION)))
def test_selection_matches_reference_outputs(port, golden, i):
    q, reps, qh, group, blocks, budget, init, local = cases.selection_case(i)
    assert cases.digest(q, reps) == str(golden[f"sel{i}_sha"])
    ids, scores = port.select_grouped(q, reps, qh, group, blocks, 128, budget, init, local)
    assert np.array_equal(ids, golden[f"sel{i}_ids"])
    assert np.array_equal(bits(scores), bits(golden[f"sel{i}_scores"]))


@pytest.mark.parametrize("i", range(len(cases.REPRESENTATIVES)))
def test_representatives_match_reference_outputs(port, golden, i):
    kv, pq, tokens, qh, kh, window, topk = cases.representatives_case(i)
    assert cases.digest(kv, pq) == str(golden[f"rep{i}_sha"])
    vals, offs = port.build_representatives(pq, kv, tokens, qh, kh, 128, 32, window, topk)
    assert np.array_equal(bits(vals), bits(golden[f"rep{i}_values"]))
    assert np.array_equal(offs, golden[f"rep{i}_offsets"])


# ----------------------------------------------- published known answers

def test_c21_known_answer(port):
    """docs/cpp-versions/C2.1-infllm-selection-uring.md:40,67 and
    artifacts/runs/*C2.1*-metrics.json: offset hash 7873450381430813043,
    blocks [0, 8, 13, 15], selected-vs-dense cosine 0.987693."""
    kv, pq, q = port.c21_fixture()
    vals, offs = port.build_representatives(pq, kv, 512, 16, 8, 128, 32, 32, 4)
    assert port.fnv_offsets(offs) == 7873450381430813043
    ids, _ = port.select_shared_blocks(q, vals, 16, 16, 128, 4, 1, 1)
    assert ids.tolist() == [0, 8, 13, 15]
    packed = port.gather_packed(kv, ids, 32, None, 0, 2048)
    sparse = port.attention(packed, q, 128, 16, 8, 128, cases.SCALE)
    dense = port.attention(kv, q, 512, 16, 8, 128, cases.SCALE)
    assert round(cosine(sparse, dense), 6) == 0.987693


def test_p13b0_lifecycle_known_answer(port):
    """docs/native-pipeline/P1.3b0-native-kv-lifecycle.md:22-28: 28 layers x
    512 tokens -> 448 sealed blocks, 7,168 representative audits, tail 32,
    generation 16, store of 121,110,528 bytes."""
    r = port.lifecycle_run(28, 16, 8, 128, 32, 32, 512, 16)
    assert r["sealed_total"] == 448
    assert r["representative_audits"] == 7168
    assert r["tail_tokens_layer0"] == 32
    assert r["generation_layer0"] == 16
    assert 28 * r["capacity_blocks"] * 32 * 2 * 8 * 128 * 2 == 121_110_528


def test_seal_boundary(port):
    """63 resident tokens do not seal; the 64th seals one block, leaving 32
    (tests/test_kv_lifecycle.py:13-37 and the P1.3b.0 boundary test)."""
    r = port.lifecycle_run(1, 4, 2, 2, 32, 32, 31, 0)
    assert r["sealed_total"] == 0 and r["tail_tokens_layer0"] == 63
    r = port.lifecycle_run(1, 4, 2, 2, 32, 32, 32, 0)
    assert r["sealed_total"] == 1 and r["tail_tokens_layer0"] == 32


def test_c1_fixture_attention_port_equals_reference(port, ref):
    """C1 (cpp/src/attention_main.cpp:118-160): the restated fixture through the
    restated attention equals the reference's attention bit for bit."""
    kv, q = port.c1_fixture()
    out = port.attention(kv, q, 128, 16, 8, 128, np.float32(0.08838834764831845))
    want = ref.attention(kv, q, 128, 16, 8, 128, np.float32(0.08838834764831845))
    assert np.array_equal(bits(out), bits(want))


# ---------------------------------------------------------- Python twins

def test_window1_masses_match_python_twin(port, twins):
    """tests/test_selection.py:6-12: with window 1 every key receives mass 1."""
    q = np.array([[10.0, 0.0], [0.0, 10.0]], np.float32)          # [T=2][D=2], one head
    kv = np.zeros((2, 2, 1, 2), np.uint16)
    kv[:, 0, 0] = q.astype(np.float16).view(np.uint16)
    kv[:, 1, 0] = kv[:, 0, 0]
    mass = port.received_mass(q.reshape(1, 2, 2), kv, 2, 1, 1, 2, 1, 1, 1)
    assert mass.tolist() == twins["window1_scores"]


def test_received_masses_match_python_twin(port, twins):
    c = twins["masses_case"]
    qh, kh, tokens, d = 4, 2, 64, 16
    q = np.array(c["query"], np.uint16).view(np.float16).astype(np.float32).reshape(qh, tokens, d)
    key = np.array(c["key"], np.uint16).reshape(kh, tokens, d)
    kv = np.zeros((tokens, 2, kh, d), np.uint16)
    kv[:, 0] = key.transpose(1, 0, 2)
    kv[:, 1] = key.transpose(1, 0, 2)
    mass = port.received_mass(q, kv, tokens, qh, kh, d, 32, c["window"], 4)
    want = np.array(c["scores"], np.float32).reshape(qh, tokens)
    assert np.abs(mass - want).max() <= 2e-5  # torch's batched softmax rounds differently


def test_gqa_selection_matches_python_twin(port, twins):
    """tests/test_selection.py:15-23 (the twin accepts [0] or [1]; the C++
    selector, and so this build, returns [0])."""
    c = twins["gqa_select"]
    q = np.array(c["query"], np.float32)
    reps = np.array(c["reps"], np.float32)
    ids, _ = port.select_shared_blocks(q, reps, 2, 2, 2, 1, 0, 0)
    assert ids.tolist() == c["chosen"] == [0]


def test_lifecycle_twin_planted_indices(port, twins):
    """tests/test_kv_lifecycle.py:22-37: planted scores at 7, 9, 11, 13 give
    those four representative indices; the C++ audit rule agrees."""
    t = twins["tail64"]
    assert t["sealed"] == 1 and t["length"] == 32
    assert port.top4_first_max(np.array(t["planted_scores"], np.float32)).tolist() == t["indices"][0]
    assert twins["tail63"] == {"sealed": 0, "length": 63}


# ---------------------------------------------------------------- numerics

def test_half_to_float_is_exact_for_every_pattern(port):
    h = np.arange(65536, dtype=np.uint16)
    got = port.half_to_float(h)
    want = h.view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert np.isnan(got[nan]).all()


def test_rne_conversion_matches_numpy(port):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200_000, dtype=np.float32) * 3,
                        np.array([0.0, -0.0, 1.9999, 0.49999, 65504, 65519, 65520, 1e9, -1e9,
                                  6e-8, 5.96e-8, 2.98e-8, 2 ** -25, 2 ** -24 * 1.5, np.inf, -np.inf],
                                 np.float32)])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(port.float_to_half_rne(x), want)


def test_reference_float_to_half_drops_the_carry(port, ref):
    """The reference's conversion (attention_reference.cpp:11-28) is not RNE:
    1.9999f becomes 1.0 (the rounded mantissa carry is lost)."""
    for v in (1.9999, 0.49999, 0.1, -3.3):
        assert port.lib.sao_ref_float_to_half(v) == ref.float_to_half(v)
    assert np.uint16(port.lib.sao_ref_float_to_half(1.9999)).view(np.float16) == np.float16(1.0)


# ------------------------------------------------- restatement vs reference

@pytest.mark.parametrize("seed", range(3))
def test_port_equals_reference_on_random_cases(port, ref, seed):
    rng = np.random.default_rng(1000 + seed)
    tokens, qh, kh = int(rng.integers(1, 300)), 8, 2
    kv = cases.fp16(rng, tokens * 2 * kh * 128)
    q = rng.standard_normal(qh * 128, dtype=np.float32)
    a = port.attention(kv, q, tokens, qh, kh, 128, cases.SCALE)
    b = ref.attention(kv, q, tokens, qh, kh, 128, cases.SCALE)
    assert np.array_equal(bits(a), bits(b))
    blocks = int(rng.integers(8, 200))
    reps = rng.standard_normal((qh, blocks, 128), dtype=np.float32)
    qq = rng.standard_normal((qh, 128), dtype=np.float32)
    i1, s1 = port.select_grouped(qq, reps, qh, 4, blocks, 128, 8, 1, 2)
    i2, s2 = ref.select_grouped(qq, reps, qh, 4, blocks, 128, 8, 1, 2)
    assert np.array_equal(i1, i2) and np.array_equal(bits(s1), bits(s2))
    t = 32 * int(rng.integers(1, 4))
    pq = cases.fp16(rng, 4 * t * 128).view(np.float16).astype(np.float32)
    kv2 = cases.fp16(rng, t * 2 * 2 * 128)
    v1, o1 = port.build_representatives(pq, kv2, t, 4, 2, 128, 32, 17, 4)
    v2, o2 = ref.build_representatives(pq, kv2, t, 4, 2, 128, 32, 17, 4)
    assert np.array_equal(bits(v1), bits(v2)) and np.array_equal(o1, o2)


def test_cpu_step_port_equals_reference(port, ref):
    """The CPU decode step used as the baseline: restatement == reference."""
    rng = np.random.default_rng(7)
    layers, qh, kh, nb = 2, 8, 2, 20
    tv = 2 * kh * 128
    pool = cases.fp16(rng, layers * (nb + 1) * 32 * tv)
    table = np.stack([np.arange(nb, dtype=np.int32) + i * (nb + 1) for i in range(layers)])
    tails = np.array([i * (nb + 1) + nb for i in range(layers)], np.int32)
    reps = rng.standard_normal((layers, qh, nb, 128), dtype=np.float32)
    q = rng.standard_normal((layers, qh, 128), dtype=np.float32)
    a = port.sparse_step(pool, table, reps, q, tails, 9, qh, kh, 128, 32, nb, 6, 1, 2, cases.SCALE, 2)
    b = ref.sparse_step(pool, table, reps, q, tails, 9, qh, kh, 128, 32, nb, 6, 1, 2, cases.SCALE, 2)
    assert np.array_equal(a[0], b[0]) and np.array_equal(bits(a[1]), bits(b[1]))


def _units_for(oracle_mod, pool, reps, q, tails_len, nb_list, qh, kh, grp, budget):
    """Unit descriptors over per-(layer) block arrays [nb + 1][32][2][KH][D]."""
    keep, units = [], (oracle_mod.Unit * (len(nb_list) * kh))()
    ids = np.zeros((len(nb_list), kh, budget), np.int64)
    out = np.zeros((len(nb_list), qh, 128), np.float32)
    for i, nb in enumerate(nb_list):
        for h in range(kh):
            u = units[i * kh + h]
            u.blocks, u.reps, u.query = pool[i].ctypes.data, reps[i].ctypes.data, q[i].ctypes.data
            u.nb, u.tail_len, u.kv_head = nb, tails_len, h
            u.ids_out = ids[i, h].ctypes.data
            u.out = out[i, h * grp:(h + 1) * grp].ctypes.data
    keep.append((pool, reps, q))
    return units, ids, out, keep


def test_cpu_unit_step_equals_layer_step(port, ref):
    """The unit-list CPU step (units of sequence-layers with their own block
    counts in one parallel loop) gives the layer step's ids and outputs, and
    the reference's own build of it gives the same bits."""
    import oracle as oracle_mod

    rng = np.random.default_rng(8)
    qh, kh, nb, tail = 8, 2, 20, 9
    grp = qh // kh
    tv = 2 * kh * 128
    pools = [cases.fp16(rng, (nb + 1) * 32 * tv) for _ in range(2)]
    reps = [rng.standard_normal((qh, nb, 128), dtype=np.float32) for _ in range(2)]
    q = [rng.standard_normal((qh, 128), dtype=np.float32) for _ in range(2)]
    want = port.sparse_step(np.concatenate(pools), np.stack([np.arange(nb, dtype=np.int32) + i * (nb + 1)
                                                            for i in range(2)]),
                            np.stack(reps), np.stack(q),
                            np.array([nb, 2 * nb + 1], np.int32), tail, qh, kh, 128, 32, nb, 6, 1,
                            2, cases.SCALE, 2)
    for lib in (port, ref):
        units, ids, out, _ = _units_for(oracle_mod, pools, reps, q, tail, [nb, nb], qh, kh, grp, 6)
        lib.sparse_units(units, qh, kh, 128, 6, 1, 2, cases.SCALE, 3)
        assert np.array_equal(ids, want[0]) and np.array_equal(bits(out), bits(want[1]))


def test_per_block_reps_equal_single_block_builds(port, ref):
    rng = np.random.default_rng(9)
    qh, kh, blocks = 8, 2, 5
    t = 32 * blocks
    pq = cases.fp16(rng, qh * t * 128).view(np.float16).astype(np.float32).reshape(qh, t, 128)
    kv = cases.fp16(rng, t * 2 * kh * 128).reshape(t, -1)
    want = np.stack([port.build_representatives(np.ascontiguousarray(pq[:, b * 32:(b + 1) * 32]),
                                                kv[b * 32:(b + 1) * 32], 32, qh, kh, 128, 32, 32,
                                                4)[0][:, 0] for b in range(blocks)], axis=1)
    for lib in (port, ref):
        got = lib.build_reps_per_block(pq, kv, blocks, qh, kh, 128, 32, 4, 3)
        assert np.array_equal(bits(got), bits(want))


def _compare_prediction(predicted, oracle):
    """cpp/src/pipeline_main.cpp:686-717, transliterated: hits, misses (oracle
    order), replacement slots (slot order), and the corrected resident set."""
    evicted = [s for s, b in enumerate(predicted) if b not in oracle]
    misses = [b for b in oracle if b not in predicted]
    assert len(misses) == len(evicted)  # the reference throws otherwise
    corrected = list(predicted)
    for m, s in zip(misses, evicted):
        corrected[s] = m
    assert sorted(corrected) == list(oracle)
    return len(predicted) - len(evicted), misses, evicted, corrected


def test_slot_correct_matches_compare_prediction(port):
    """The oracle's slot correction equals the reference's compare_prediction
    on full windows (both sets `budget` distinct blocks)."""
    rng = np.random.default_rng(21)
    budget, nb = 16, 60
    sel, cnt, slots, want = [], [], [], []
    for _ in range(200):
        predicted = rng.choice(nb, budget, replace=False).tolist()
        overlap = rng.integers(0, budget + 1)
        keep = rng.choice(predicted, overlap, replace=False).tolist()
        rest = [b for b in rng.permutation(nb).tolist() if b not in predicted][:budget - overlap]
        oracle = sorted(keep + rest)
        want.append(_compare_prediction(predicted, oracle))
        sel.append(oracle)
        cnt.append(budget)
        slots.append(predicted)
    got_slots, mi, re, st = port.slot_correct(np.array(sel), np.array(cnt), np.array(slots))
    for u, (hits, misses, evicted, corrected) in enumerate(want):
        assert st[u].tolist() == [hits, len(misses)]
        assert mi[u, :len(misses)].tolist() == misses and (mi[u, len(misses):] == -1).all()
        assert re[u, :len(evicted)].tolist() == evicted and (re[u, len(evicted):] == -1).all()
        assert got_slots[u].tolist() == corrected


def test_slot_correct_empty_slots_and_short_selections(port):
    """Generalisation beyond the reference's equal counts: empty slots are
    always overwritten and slots freed beyond the misses are emptied, so the
    corrected window holds exactly the selection; hits never move."""
    rng = np.random.default_rng(22)
    budget, nb = 12, 40
    for _ in range(300):
        count = int(rng.integers(0, budget + 1))
        sel = np.full(budget, -1, np.int32)
        sel[:count] = np.sort(rng.choice(nb, count, replace=False))
        slots = rng.choice(nb, budget, replace=False).astype(np.int32)
        slots[rng.random(budget) < 0.3] = -1
        got, mi, re, st = port.slot_correct(sel[None], np.array([count]), slots[None])
        got, mi, re = got[0], mi[0], re[0]
        assert sorted(b for b in got if b >= 0) == sel[:count].tolist()
        hits = [s for s in range(budget) if slots[s] >= 0 and slots[s] in sel[:count]]
        assert all(got[s] == slots[s] for s in hits) and st[0, 0] == len(hits)
        n_miss = count - len(hits)
        assert st[0, 1] == n_miss and (mi[n_miss:] == -1).all() and (re[n_miss:] == -1).all()
        assert all(got[re[k]] == mi[k] for k in range(n_miss))


def test_head_norm_rope_matches_float64(port):
    """The oracle's q/k norm + RoPE (head_rms + rope of qwen_layer_main.cpp)
    against a float64 evaluation of the same formulas, with the angle
    position * frequency formed in FP32 as the reference forms it (at
    position 32767 that rounding alone moves the angle by ~2e-3 rad)."""
    rng = np.random.default_rng(31)
    rows = rng.standard_normal((6, 128), dtype=np.float32) * 3
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    for pos, theta in [(0, 1e6), (17, 1e6), (32767, 1e6), (4000, 1e4)]:
        got = port.head_norm_rope(rows, w, pos, theta, 1e-6)
        x = rows.astype(np.float64)
        x = x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-6) * w
        i = np.arange(64, dtype=np.float32)
        freq = np.power(np.float32(theta), np.float32(-2.0) * i / np.float32(128.0))
        ang = (np.float32(pos) * freq.astype(np.float32)).astype(np.float64)
        c, s = np.cos(ang), np.sin(ang)
        want = np.concatenate([x[:, :64] * c - x[:, 64:] * s, x[:, 64:] * c + x[:, :64] * s], 1)
        # powf / cosf / sinf of the C library may round an ulp off numpy's
        np.testing.assert_allclose(got, want, rtol=1e-5,
                                   atol=(1e-5 + 2e-7 * pos) * np.abs(want).max())


# ------------------------------------------ audit_dense_selection restatement

def test_dense_block_mass_matches_float64(port):
    """sao_dense_block_mass restates pipeline_main.cpp:517-543 (FP32 logits,
    expf, double denominator) at the reference's own audit shape (512 tokens,
    16 heads, 16 blocks of 32): within FP32 logit rounding of a float64
    softmax, and its blocks sum to 1. A partial last block (an open tail)
    takes the remaining tokens."""
    rng = np.random.default_rng(5)
    for tokens in (512, 300):
        keys = rng.standard_normal((tokens, 128)).astype(np.float16)
        q = rng.standard_normal((16, 128)).astype(np.float32)
        m = port.dense_block_mass(keys, q, 32, 1.0 / np.sqrt(128.0))
        lg = q.astype(np.float64) @ keys.astype(np.float64).T / np.sqrt(128.0)
        p = np.exp(lg - lg.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        pad = np.zeros((16, -(-tokens // 32) * 32))
        pad[:, :tokens] = p
        want = pad.reshape(16, -1, 32).sum(2).mean(0)
        assert m.shape == want.shape
        np.testing.assert_allclose(m, want, rtol=2e-6)
        assert abs(m.sum() - 1.0) < 1e-12


def test_audit_selection_reference_case_and_product_quality(port, pkg):
    """sao_audit_selection at the reference's fixed case (16 blocks, forced 0
    and 15, budget 4: pipeline_main.cpp:544-569), including a tie that the
    stable sort gives to the lower block; then the product's host figures
    (quality.selection_quality) equal it unit by unit on random masses."""
    from solidattention_repro_b200 import quality

    m = np.full(16, 0.01)
    m[[3, 6, 9]] = [0.2, 0.3, 0.2]  # 3 and 9 tie: 3 ranks first
    sel_mass, recall = port.audit_selection(m, [0, 6, 9, 15], 4, 1, 1)
    assert recall == 0.75  # oracle set {0, 15, 6, 3}
    assert sel_mass == pytest.approx(0.01 + 0.3 + 0.2 + 0.01)
    assert port.audit_selection(m, [0, 3, 6, 15], 4, 1, 1)[1] == 1.0

    rng = np.random.default_rng(9)
    n_sl, kh, groups, budget, init, local, table = 6, 4, 2, 6, 1, 2, 24
    nb = rng.integers(4, table + 1, n_sl)
    mass = np.zeros((n_sl, kh, table + 1))
    selected = np.full((n_sl, groups, budget), -1, np.int32)
    counts = np.zeros((n_sl, groups), np.int32)
    for sl in range(n_sl):
        for h in range(kh):
            raw = rng.random(nb[sl] + 1)
            raw /= raw.sum()
            mass[sl, h, :nb[sl]] = raw[:-1]
            mass[sl, h, -1] = raw[-1]
        for g in range(groups):
            c = min(budget, nb[sl])
            selected[sl, g, :c] = np.sort(rng.choice(nb[sl], c, replace=False))
            counts[sl, g] = c
    got = quality.selection_quality(mass, selected, counts, nb, budget, init, local)
    want_mass, want_recall = [], []
    for sl in range(n_sl):
        for h in range(kh):
            g = h * groups // kh
            a, r = port.audit_selection(mass[sl, h, :nb[sl]], selected[sl, g, :counts[sl, g]],
                                        budget, init, local, mass[sl, h, -1])
            want_mass.append(a)
            want_recall.append(r)
    assert got["units"] == n_sl * kh
    assert got["selected_mass"] == pytest.approx(np.mean(want_mass), abs=1e-12)
    assert got["oracle_recall"] == pytest.approx(np.mean(want_recall), abs=1e-12)
