"""Host-side logic that needs no GPU: workload byte accounting (the roofline
numerators), the bench's clock-sample parsing and profile lookup."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def workloads(pkg):
    from solidattention_repro_b200 import workloads as w

    return w


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_bytes_match_the_configs(workloads):
    """Per-step algorithmic bytes of the benchmark configs (selected KV and
    representatives scanned), as the roofline numerators use them."""
    c = workloads.CONFIGS
    assert c["cfg1"].selected_kv_bytes() == 2_097_152
    assert c["cfg2"].selected_kv_bytes() == 234_881_024
    assert c["cfg2"].rep_bytes() == 117_440_512
    assert c["cfg3"].selected_kv_bytes() == 603_979_776
    assert c["cfg3"].rep_bytes() == 603_979_776
    assert c["cfg5"].selected_kv_bytes() == 1_207_959_552
    assert c["cfg5"].rep_bytes() == 2_415_919_104
    # budgets: init + local + dynamic
    assert (c["cfg3"].init_blocks, c["cfg3"].local_blocks, c["cfg3"].budget_blocks) == (1, 4, 128)
    assert (c["cfg5"].init_blocks, c["cfg5"].local_blocks, c["cfg5"].budget_blocks) == (1, 8, 256)


def test_batched_config_context_draws(workloads):
    """cfg4: 64 sequences with seeded contexts uniform in [8192, 32768] tokens
    (whole blocks), a 2048-token budget each, 8 per GPU; a sequence's length
    depends only on its global batch index, so sequence shards compose."""
    w = workloads.CONFIGS["cfg4"]
    assert (w.batch, w.seqs, w.budget_blocks, w.query_heads, w.kv_heads, w.layers) == \
        (64, 8, 64, 32, 8, 36)
    nbs = [w.sequence_blocks(b) for b in range(w.batch)]
    assert nbs == [w.sequence_blocks(b) for b in range(w.batch)]
    assert all(256 <= n <= 1024 for n in nbs)
    assert len(set(nbs)) > 32  # genuinely variable
    # the 8 ranks' shards are the whole batch
    from solidattention_repro_b200 import sharding

    owned = [sharding.shard_sequences(w.batch, 8, r) for r in range(8)]
    assert [o[1] for o in owned] == [w.seqs] * 8
    assert sorted(i for f, n in owned for i in range(f, f + n)) == list(range(w.batch))
    # fixed-context configs ignore the draw
    assert workloads.CONFIGS["cfg3"].sequence_blocks(17) == 1024


def test_clock_sampler_parses_nvidia_smi_rows(bench):
    s = bench.ClockSampler.__new__(bench.ClockSampler)

    class FakeProc:
        def terminate(self):
            pass

        def communicate(self, timeout=None):
            rows = ["0, 1965, 1965, 700.5, 0x0, Not Active, Not Active, Not Active, Not Active",
                    "0, 1950, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active",
                    "0, 1965, 1965, 910.0, 0x0, Not Active, Not Active, Not Active, Not Active"]
            return "\n".join(rows) + "\n", ""

    s.proc = FakeProc()
    s.gpu = 0
    out = s.stop()
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 3


def test_profile_traffic_lookup(bench, tmp_path, monkeypatch):
    (tmp_path / "profiles").mkdir()
    (tmp_path / "profiles" / "x.md").write_text(
        "traffic_per_launch[attention@cfg3]: 605000000\n")
    (tmp_path / "profiles" / "y.md").write_text(
        "traffic_per_launch[select@cfg3]: 612000000 per 600000000 algorithmic bytes\n")
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.profile_traffic("attention", "cfg3") == 605000000.0
    # a capture of a 600 MB launch scaled to the timed 650 MB launch
    assert bench.profile_traffic("select", "cfg3", 650_000_000) == 612000000 * 650 / 600
    assert bench.profile_traffic("select", "cfg3") == 612000000.0
    assert bench.profile_traffic("select", "cfg5") is None


@pytest.mark.parametrize("steps,warmup", [(20, 5), (2000, 20), (1, 0), (32, 0), (33, 3), (7, 3)])
def test_tail_prefill_puts_a_seal_at_the_end_of_the_timed_steps(workloads, steps, warmup):
    """The bench pre-fills every open tail so that its last timed step seals
    (a block seals on the step that appends its 32nd token), whatever the
    step counts, and counts the seals of its timed window."""
    t0 = workloads.tail_for_seal_at_end(steps, warmup)
    assert 0 <= t0 < 32
    # replay the lifecycle: tail length before step i is (t0 + i) mod 32
    tail, sealed_at = t0, []
    for i in range(warmup + steps):
        tail += 1
        if tail == 32:
            sealed_at.append(i)
            tail = 0
    assert sealed_at and sealed_at[-1] == warmup + steps - 1
    timed = [i for i in sealed_at if i >= warmup]
    assert workloads.seal_steps(t0, warmup, steps) == len(timed) >= 1
    assert len(timed) == (steps + 31 - 0) // 32 if steps >= 32 else len(timed) == 1
