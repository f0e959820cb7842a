"""Shared pytest setup: the `gpu` marker, package/oracle loaders, helpers.

GPU tests (marked ``gpu``) call the sm_100a kernels through the C ABI of
libsa_b200.so and check them against the CPU oracle (oracle/, test
infrastructure). CPU tests cover the oracle against the reference's golden
vectors, host logic, and that the library loads and exports its symbols.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402
import oracle  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    """Run files named test_zz_* after every other test file."""
    items.sort(key=lambda it: 1 if Path(str(it.fspath)).name.startswith("test_zz_") else 0)


@pytest.fixture(scope="session")
def port():
    return oracle.port()


@pytest.fixture(scope="session")
def ref():
    r = oracle.reference()
    if r is None:
        pytest.skip("oracle/_ref not built (reference sources absent at build time)")
    return r


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def fp16_normal(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    """FP16 N(0, scale^2) bit patterns, rounded to nearest even."""
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(
        np.float16).view(np.uint16)


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def gap_aware_equal(got_ids, ref_ids, scores, gap: float = 1e-5) -> bool:
    """Selected ids equal, except swaps between blocks whose scores differ < gap."""
    got, want = set(map(int, got_ids)), set(map(int, ref_ids))
    if got == want:
        return True
    extra, missing = sorted(got - want), sorted(want - got)
    if len(extra) != len(missing):
        return False
    return all(abs(float(scores[a]) - float(scores[b])) < gap for a, b in zip(extra, missing))
