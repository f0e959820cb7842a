"""ctypes binding of libsa_b200.so (the C ABI in include/sa_b200.h).

Loading fails loudly when the library is missing: there is no CPU or
pure-PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsa_b200.so"

SA_OK = 0
SA_ERR_INVALID_ARG = -1
SA_ERR_UNSUPPORTED = -2
SA_ERR_CAPACITY = -3
SA_ERR_CUDA = -4
SA_ERR_DEVICE = -5
SA_ERR_TIMEOUT = -6
SA_ERR_NO_MEMORY = -7

SA_DEV_BAD_BLOCK = 0x1
SA_DEV_TAIL_FULL = 0x2
SA_DEV_POOL_EMPTY = 0x4
SA_DEV_NONFINITE = 0x8
SA_DEV_TIMEOUT = 0x10
SA_DEV_TABLE_FULL = 0x20

SA_ATTN_COPY_OUTPUT = 0x1
SA_ATTN_CONSUME = 0x2


class SparseKVError(RuntimeError):
    """A libsa_b200 call returned a non-zero sa_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


class CtxConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "device", "query_heads", "kv_heads", "head_dim", "layers", "seqs", "pool_blocks",
        "table_blocks", "budget_blocks", "init_blocks", "local_blocks", "select_group",
        "rep_window", "rep_topk", "out_fp16")] + [("scale", C.c_float)]


class CtxPtrs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "pool", "reps", "table", "num_sealed", "tail_block", "tail_len", "generation",
        "query_ring", "selected", "selected_count", "scores", "free_list", "free_top",
        "status")]


class Timings(C.Structure):
    _fields_ = [("h2d_ms", C.c_double), ("kernel_ms", C.c_double),
                ("consumer_ms", C.c_double), ("d2h_ms", C.c_double)]


_vp = C.c_void_p
_sz = C.c_size_t
_i32 = C.c_int32
_i64 = C.c_int64

# name -> (restype, argtypes); every symbol declared in include/sa_b200.h
PROTOTYPES = {
    "sa_status_string": (C.c_char_p, [C.c_int]),
    "sa_last_error": (C.c_char_p, []),
    "sa_version": (C.c_char_p, []),
    "sa_attention_workspace_size": (_sz, [_sz, _sz, _sz]),
    "sa_attention_packed": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, C.c_float, _vp, C.c_int,
                                      _vp, _sz, _vp]),
    "sa_attention_packed_noalloc": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, C.c_float, _vp,
                                              C.c_int, _vp]),
    "sa_select_workspace_size": (_sz, [_sz, _sz, _sz]),
    "sa_select_blocks": (C.c_int, [_vp, _vp, _i64, _i64, _i64, _sz, _sz, _sz, _sz, _sz, _sz,
                                   _sz, _vp, _vp, _vp, _sz, _vp]),
    "sa_build_representatives": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _vp,
                                           _vp, _vp]),
    "sa_pack_kv_fp16": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "sa_backend_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "sa_backend_destroy": (C.c_int, [_vp]),
    "sa_backend_name": (C.c_char_p, [_vp]),
    "sa_backend_host_alloc": (C.c_int, [_vp, _sz, C.POINTER(_vp)]),
    "sa_backend_host_free": (C.c_int, [_vp, _vp]),
    "sa_backend_attention": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, C.c_float, C.c_int,
                                       _vp, C.POINTER(Timings)]),
    "sa_backend_select": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp, _vp]),
    "sa_backend_build_representatives": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz,
                                                   _sz, _vp, _vp]),
    "sa_backend_execute": (C.c_int, [_vp, _vp, _sz, C.c_uint8, C.POINTER(Timings),
                                     C.POINTER(C.c_uint64)]),
    "sa_ctx_create": (C.c_int, [C.POINTER(CtxConfig), C.POINTER(_vp)]),
    "sa_ctx_destroy": (C.c_int, [_vp]),
    "sa_ctx_get_ptrs": (C.c_int, [_vp, C.POINTER(CtxPtrs)]),
    "sa_ctx_set_stream": (C.c_int, [_vp, _vp]),
    "sa_ctx_stream": (_vp, [_vp]),
    "sa_ctx_reset": (C.c_int, [_vp]),
    "sa_ctx_prefill": (C.c_int, [_vp, _i32, _i32, _i32, _vp]),
    "sa_ctx_build_reps": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _i32]),
    "sa_ctx_step": (C.c_int, [_vp, _vp, _vp, _i32, _vp]),
    "sa_ctx_step_host": (C.c_int, [_vp, _vp, _vp, _i32, _vp]),
    "sa_ctx_append": (C.c_int, [_vp, _vp, _vp, _i32]),
    "sa_ctx_select": (C.c_int, [_vp, _vp]),
    "sa_ctx_attend": (C.c_int, [_vp, _vp, _vp]),
    "sa_ctx_seal": (C.c_int, [_vp]),
    "sa_ctx_sync": (C.c_int, [_vp, C.POINTER(C.c_uint32)]),
    "sa_ctx_launch_count": (C.c_uint64, [_vp]),
    "sa_ctx_graph_begin": (C.c_int, [_vp]),
    "sa_ctx_graph_end": (C.c_int, [_vp]),
    "sa_ctx_graph_launch": (C.c_int, [_vp]),
    "sa_ctx_audit": (C.c_int, [_vp, _vp, _vp]),
    "sa_ctx_slot_correct": (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "sa_ctx_step_raw": (C.c_int, [_vp] * 7 + [C.c_float, C.c_float, _vp]),
    "sa_ctx_import_blocks": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _vp]),
    "sa_ctx_export_blocks": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _vp]),
    "sa_ctx_gather_buffer": (C.c_int, [_vp, _i32, C.POINTER(_vp), C.POINTER(_sz)]),
    "sa_ctx_gather_attach": (C.c_int, [_vp, _i32, C.POINTER(_vp)]),
    "sa_ctx_gather_wait": (C.c_int, [_vp, C.POINTER(_vp)]),
    "sa_ipc_export": (C.c_int, [_i32, _vp, _vp]),
    "sa_ipc_open": (C.c_int, [_i32, _vp, C.POINTER(_vp)]),
    "sa_ipc_close": (C.c_int, [_i32, _vp]),
    "sa_probe_stream": (C.c_int, [_vp, C.c_int64, _vp, C.c_int64, _i32, _vp, _vp, _vp]),
}

_LIB = None


def load() -> C.CDLL:
    """The loaded library with prototypes set; raises if it is not built.

    SA_B200_LIB names another build of the same library (a copy built
    elsewhere, e.g. with different nvcc flags); it must export every symbol
    below, and nothing else is loaded in its place."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.environ.get("SA_B200_LIB", str(LIB_PATH))
    if not Path(path).exists():
        raise ImportError(
            f"libsa_b200.so not found at {path}: build it with "
            "`python __graft_entry__.py build` (nvcc, sm_100a). There is no fallback.")
    lib = C.CDLL(path)
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def check(status: int, what: str = "") -> None:
    """Raise SparseKVError for a non-zero sa_status, with the library's message."""
    if status != SA_OK:
        lib = load()
        msg = lib.sa_last_error().decode() or lib.sa_status_string(status).decode()
        raise SparseKVError(status, f"{what}: {msg}" if what else msg)
