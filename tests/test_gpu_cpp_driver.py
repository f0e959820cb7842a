"""The reference's native driver flows through the C++ drop-in adapter.

Compiles tests/cpp/b200_driver_main.cpp against include/sa_b200_backend.hpp,
libsa_b200.so and the reference's own CPU functions (oracle/_ref), then runs
it: C1 over every AcceleratorBackend variant, C2.1 through the b200::
selector, problems beyond the reference's token caps, and the reference's
error conditions as exceptions.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
pytestmark = pytest.mark.gpu


def build_driver() -> Path:
    ref_dir = ROOT / "oracle" / "_ref"
    if not (ref_dir / "libsa_ref.so").exists():
        pytest.skip("oracle/_ref was not built (reference sources absent at build time)")
    pkg_dir = ROOT / "solidattention-repro_b200"
    out = ROOT / "_build" / "b200_driver"
    out.parent.mkdir(exist_ok=True)
    cmd = ["g++", "-std=c++20", "-O2", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "cpp" / "b200_driver_main.cpp"), f"-L{pkg_dir}", "-lsa_b200",
           f"-L{ref_dir}", "-lsa_ref", f"-Wl,-rpath,{pkg_dir}:{ref_dir}", "-o", str(out)]
    subprocess.run(cmd, check=True)
    return out


def test_reference_driver_flows_through_the_b200_adapter():
    exe = build_driver()
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(run.stdout, run.stderr)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "ALL PASSED" in run.stdout
