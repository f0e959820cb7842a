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
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.profile_traffic("attention", "cfg3") == 605000000.0
    assert bench.profile_traffic("select", "cfg3") is None
