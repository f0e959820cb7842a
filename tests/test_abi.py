"""The C ABI library loads and exports every entry point include/*.h declares.

No GPU work: the calls below are either pure host functions or argument
rejections that return before any CUDA call.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        for m in re.finditer(r"SA_API\s+[^;(]*?\b(sa_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_expected_surface():
    names = declared_symbols()
    for must in ["sa_attention_packed", "sa_select_blocks", "sa_build_representatives",
                 "sa_pack_kv_fp16", "sa_backend_attention", "sa_ctx_step", "sa_ctx_step_host",
                 "sa_last_error"]:
        assert must in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_declares_every_symbol():
    """The ctypes binding sets a prototype for every entry point the header declares."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_sa_lib", ROOT / "solidattention-repro_b200" / "_lib.py")
    lib = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(lib)
    missing = [n for n in declared_symbols() if n not in lib.PROTOTYPES]
    assert not missing, missing


def test_shared_mode_workspace_includes_the_head_split(pkg):
    """Groups above four heads split over CTAs need dot and counter scratch."""
    lib = pkg.load()
    per_kv_head = lib.sa_select_workspace_size(16, 4, 1024)
    shared = lib.sa_select_workspace_size(16, 16, 1024)
    # the shared group's 16 heads x 1024 blocks of FP32 dots
    assert shared - per_kv_head >= 16 * 1024 * 4 - 4 * 1024 * 4


def test_graph_calls_reject_a_null_context(pkg):
    lib = pkg.load()
    for fn in (lib.sa_ctx_graph_begin, lib.sa_ctx_graph_end, lib.sa_ctx_graph_launch):
        assert fn(None) == pkg.SA_ERR_INVALID_ARG


def test_host_only_calls(pkg):
    lib = pkg.load()
    assert lib.sa_version().decode().startswith("sa_b200")
    assert lib.sa_status_string(pkg.SA_ERR_INVALID_ARG).decode() == "invalid argument"
    assert lib.sa_attention_workspace_size(4100, 32, 8) > 0
    assert lib.sa_select_workspace_size(32, 4, 1024) >= 8 * 1024 * 4


def test_reference_rejections_without_a_gpu(pkg):
    """Dimensions the reference rejects (std::runtime_error) come back as
    SA_ERR_INVALID_ARG before any device work, with a message."""
    lib = pkg.load()
    dummy = C.c_void_p(16)
    # select_shared_blocks: budget > blocks (cpp/src/selection.cpp:99-105)
    rc = lib.sa_select_blocks(dummy, dummy, 128, 1, 1, 4, 4, 8, 128, 9, 1, 1, dummy, None, dummy,
                              1 << 20, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    assert b"selection dimensions" in lib.sa_last_error()
    # init + local > budget
    rc = lib.sa_select_blocks(dummy, dummy, 128, 1, 1, 4, 4, 8, 128, 2, 2, 1, dummy, None, dummy,
                              1 << 20, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    # attention_reference: query heads not a multiple of KV heads, zero tokens
    rc = lib.sa_attention_packed(dummy, dummy, 10, 12, 8, 128, C.c_float(0.1), dummy, 0, dummy,
                                 1 << 20, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    rc = lib.sa_attention_packed(dummy, dummy, 0, 16, 8, 128, C.c_float(0.1), dummy, 0, dummy,
                                 1 << 20, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    # build_local_causal_representatives: tokens not a multiple of the block
    rc = lib.sa_build_representatives(dummy, dummy, 33, 4, 2, 128, 32, 32, 4, dummy, dummy, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    assert b"representative dimensions" in lib.sa_last_error()
    # topk larger than a block
    rc = lib.sa_build_representatives(dummy, dummy, 64, 4, 2, 128, 32, 32, 33, dummy, dummy, None)
    assert rc == pkg.SA_ERR_INVALID_ARG
    # the streaming probe: no pool, an unknown mode, an unaligned pool
    assert lib.sa_probe_stream(None, 4, dummy, 4, 0, dummy, None, None) == pkg.SA_ERR_INVALID_ARG
    assert lib.sa_probe_stream(dummy, 4, dummy, 4, 2, dummy, None, None) == pkg.SA_ERR_INVALID_ARG
    assert lib.sa_probe_stream(C.c_void_p(24), 4, dummy, 4, 0, dummy, None,
                               None) == pkg.SA_ERR_INVALID_ARG


def test_context_config_validation_without_a_gpu(pkg):
    lib = pkg.load()
    base = dict(device=0, query_heads=32, kv_heads=8, head_dim=128, layers=2, seqs=1,
                pool_blocks=64, table_blocks=16, budget_blocks=8, init_blocks=1, local_blocks=2,
                select_group=4, rep_window=32, rep_topk=4, out_fp16=1, scale=0.088)
    for bad, status in [({"head_dim": 64}, pkg.SA_ERR_UNSUPPORTED),
                        ({"query_heads": 30}, pkg.SA_ERR_INVALID_ARG),
                        ({"init_blocks": 5, "local_blocks": 4}, pkg.SA_ERR_INVALID_ARG),
                        ({"select_group": 2}, pkg.SA_ERR_INVALID_ARG),
                        ({"rep_window": 65}, pkg.SA_ERR_UNSUPPORTED)]:
        cfg = pkg.CtxConfig(**{**base, **bad})
        h = C.c_void_p()
        assert lib.sa_ctx_create(C.byref(cfg), C.byref(h)) == status
        assert not h.value


@pytest.mark.parametrize("name", ["oracle/liboracle.so", "solidattention-repro_b200/libsa_b200.so"])
def test_built_libraries_present(name):
    assert (ROOT / name).exists(), f"{name} missing: run python __graft_entry__.py build"
