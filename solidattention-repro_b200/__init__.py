"""B200 (sm_100a) decode-time sparse-KV path: Python host mirror of the C ABI.

The compute lives in libsa_b200.so (hand-written sm_100a CUDA); this package
only binds it with ctypes and uses PyTorch for device memory and streams.
Names and argument meanings follow the reference (ZjuXxxc/solidattention-repro):

* :func:`attention`                  -- cpp/src/attention_reference.cpp:55-96
* :func:`select_shared_blocks`       -- cpp/src/selection.cpp:96-147
* :func:`build_local_causal_representatives` -- cpp/src/selection.cpp:12-94
* :func:`pack_kv_fp16`               -- cpp/src/qwen_layer_main.cpp:270-281
* :class:`Backend`                   -- cpp/include/solidattention/backend.hpp:41-58
* :class:`DecodeContext`             -- the P1.3 KV lifecycle,
  cpp/src/kv_lifecycle_main.cpp:25-113 and cpp/src/online_seal_main.cpp:34-47

Invalid dimensions raise :class:`SparseKVError` with status
``SA_ERR_INVALID_ARG`` where the reference throws ``std::runtime_error``.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import math

import numpy as np
import torch

from ._lib import (SA_ATTN_CONSUME, SA_ATTN_COPY_OUTPUT, SA_DEV_BAD_BLOCK, SA_DEV_NONFINITE,
                   SA_DEV_POOL_EMPTY, SA_DEV_TABLE_FULL, SA_DEV_TAIL_FULL, SA_DEV_TIMEOUT,
                   SA_ERR_CAPACITY, SA_ERR_DEVICE, SA_ERR_INVALID_ARG, SA_ERR_TIMEOUT,
                   SA_ERR_UNSUPPORTED, CtxConfig, CtxPtrs, SparseKVError, Timings, check, load)

__all__ = [
    "attention", "select_shared_blocks", "build_local_causal_representatives", "pack_kv_fp16",
    "Backend", "DecodeContext", "SparseKVError", "load", "version",
]

BLOCK_TOKENS = 32
HEAD_DIM = 128


def version() -> str:
    return load().sa_version().decode()


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dev_ptr(t: torch.Tensor, dtype: torch.dtype, name: str) -> int:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _kv_ptr(kv: torch.Tensor) -> int:
    if kv.dtype not in (torch.float16, torch.int16, torch.uint16):
        raise TypeError("interleaved_kv must hold FP16 bit patterns (float16/int16/uint16)")
    return _dev_ptr(kv, kv.dtype, "interleaved_kv")


class _CudaArray:
    """Wraps a raw device pointer for torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {
            "data": (int(ptr), False), "shape": tuple(int(s) for s in shape),
            "typestr": typestr, "version": 3, "strides": None}


def _view(ptr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.int32: "<i4"}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)


# ------------------------------------------------------------ stateless ops

def attention(interleaved_kv: torch.Tensor, query: torch.Tensor, tokens: int, query_heads: int,
              kv_heads: int, head_dim: int = HEAD_DIM, scale: float | None = None,
              out_fp16: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """GQA decode attention over a packed [tokens][2][kv_heads][head_dim] FP16 buffer.

    Same semantics as the reference's ``attention_reference(AttentionProblem)``;
    returns [query_heads][head_dim] FP32 (or FP16 when ``out_fp16``).
    """
    lib = load()
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    dev = query.device
    if out is None:
        out = torch.empty(query_heads, head_dim, device=dev,
                          dtype=torch.float16 if out_fp16 else torch.float32)
    ws_bytes = lib.sa_attention_workspace_size(tokens, query_heads, kv_heads) if kv_heads else 0
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    check(lib.sa_attention_packed(_kv_ptr(interleaved_kv), _dev_ptr(query, torch.float32, "query"),
                                  tokens, query_heads, kv_heads, head_dim, C.c_float(scale),
                                  out.data_ptr(), int(out_fp16), ws.data_ptr(), ws.numel(),
                                  _stream(dev)), "attention")
    return out


def select_shared_blocks(query: torch.Tensor, representatives: torch.Tensor, query_heads: int,
                         blocks: int, head_dim: int, budget_blocks: int, init_blocks: int,
                         local_blocks: int, group: int | None = None,
                         layout: str = "reference") -> tuple[torch.Tensor, torch.Tensor]:
    """Block selection; returns (block_ids int32 [groups][budget], mean_head_scores [groups][blocks]).

    ``group`` query heads share one selection (default: all heads -- the
    reference's shared mode; ``query_heads // kv_heads`` selects per KV head).
    ``layout`` "reference" is [query_heads][blocks][head_dim]; "dim_major" is
    [query_heads][head_dim][blocks].
    """
    lib = load()
    group = query_heads if group is None else group
    if layout == "reference":
        strides = (blocks * head_dim, head_dim, 1)
    elif layout == "dim_major":
        strides = (head_dim * blocks, 1, blocks)
    else:
        raise ValueError("layout must be 'reference' or 'dim_major'")
    dev = query.device
    n_groups = query_heads // group if group and query_heads % group == 0 else 1
    ids = torch.empty(n_groups, max(budget_blocks, 1), dtype=torch.int32, device=dev)
    scores = torch.empty(n_groups, max(blocks, 1), dtype=torch.float32, device=dev)
    ws_bytes = lib.sa_select_workspace_size(query_heads, group, blocks) if group else 0
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)  # the call zeroes its counters
    check(lib.sa_select_blocks(_dev_ptr(query, torch.float32, "query"),
                               _dev_ptr(representatives, torch.float32, "representatives"),
                               *strides, query_heads, group, blocks, head_dim, budget_blocks,
                               init_blocks, local_blocks, ids.data_ptr(), scores.data_ptr(),
                               ws.data_ptr(), ws.numel(), _stream(dev)), "select_shared_blocks")
    return ids, scores


def build_local_causal_representatives(prompt_queries: torch.Tensor, interleaved_kv: torch.Tensor,
                                       tokens: int, query_heads: int, kv_heads: int,
                                       head_dim: int, block_tokens: int, local_window: int,
                                       representative_topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (values FP32 [qh][blocks][head_dim], chosen offsets int32 [qh][blocks][topk])."""
    lib = load()
    dev = prompt_queries.device
    blocks = tokens // block_tokens if block_tokens else 0
    values = torch.empty(max(query_heads * blocks * head_dim, 1), dtype=torch.float32, device=dev)
    offsets = torch.empty(max(query_heads * blocks * representative_topk, 1), dtype=torch.int32,
                          device=dev)
    check(lib.sa_build_representatives(
        _dev_ptr(prompt_queries, torch.float32, "prompt_queries"), _kv_ptr(interleaved_kv),
        tokens, query_heads, kv_heads, head_dim, block_tokens, local_window,
        representative_topk, values.data_ptr(), offsets.data_ptr(), _stream(dev)),
        "build_local_causal_representatives")
    return (values[: query_heads * blocks * head_dim].view(query_heads, blocks, head_dim),
            offsets[: query_heads * blocks * representative_topk].view(
                query_heads, blocks, representative_topk))


def pack_kv_fp16(packed: torch.Tensor, key: torch.Tensor, value: torch.Tensor, token: int) -> None:
    """Write FP32 key/value (RNE to FP16) into row ``token`` of packed [rows][K|V]."""
    check(load().sa_pack_kv_fp16(_kv_ptr(packed), _dev_ptr(key, torch.float32, "key"),
                                 _dev_ptr(value, torch.float32, "value"), token, key.numel(),
                                 _stream(key.device)), "pack_kv_fp16")


# ---------------------------------------------------------------- backend

class Backend:
    """Host-buffer attention with the reference AcceleratorBackend's timing split."""

    def __init__(self, device: int = 0):
        self._lib = load()
        h = C.c_void_p()
        check(self._lib.sa_backend_create(device, C.byref(h)), "sa_backend_create")
        self._h = h

    def name(self) -> str:
        return self._lib.sa_backend_name(self._h).decode()

    def attention(self, kv: np.ndarray, query: np.ndarray, tokens: int, query_heads: int,
                  kv_heads: int, head_dim: int, scale: float, copy_output: bool = True,
                  consume: bool = False):
        kv = np.ascontiguousarray(kv, np.uint16)
        query = np.ascontiguousarray(query, np.float32)
        out = np.zeros(1 if consume else query_heads * head_dim, np.float32)
        flags = (SA_ATTN_COPY_OUTPUT if copy_output or consume else 0) | \
            (SA_ATTN_CONSUME if consume else 0)
        t = Timings()
        check(self._lib.sa_backend_attention(self._h, kv.ctypes.data, query.ctypes.data, tokens,
                                             query_heads, kv_heads, head_dim, C.c_float(scale),
                                             flags, out.ctypes.data, C.byref(t)), "attention")
        return out, {"h2d_ms": t.h2d_ms, "kernel_ms": t.kernel_ms,
                     "consumer_ms": t.consumer_ms, "d2h_ms": t.d2h_ms}

    def execute(self, data: np.ndarray, mask: int):
        data = np.ascontiguousarray(data, np.uint8)
        t = Timings()
        checksum = C.c_uint64(0)
        check(self._lib.sa_backend_execute(self._h, data.ctypes.data, data.nbytes, mask,
                                           C.byref(t), C.byref(checksum)), "execute")
        return int(checksum.value), {"h2d_ms": t.h2d_ms, "kernel_ms": t.kernel_ms,
                                     "d2h_ms": t.d2h_ms}

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.sa_backend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------- decode context

class DecodeContext:
    """Paged sparse-KV decode state on one GPU (wraps ``sa_ctx``).

    All kernels run on the torch stream that was current when the context was
    created (so torch ops and CUDA events order with them). Tensor attributes
    are zero-copy views of the context's device buffers:

    ``pool`` [pool_blocks, KH, 2, 32, 128] FP16 (head-major blocks: K rows then
    V rows of one KV head are one contiguous 16 KB run; ``write_blocks`` /
    ``read_blocks`` convert from / to the reference's token-major rows
    [blocks, 32, 2, KH, 128]); ``reps`` [S*L, QH, 128, cap];
    ``table`` [S*L, table_blocks]; ``num_sealed``/``tail_block``/``tail_len``/
    ``generation`` [S*L]; ``query_ring`` [S*L, QH, 32, 128];
    ``selected`` [S*L, groups, budget]; ``selected_count`` [S*L, groups];
    ``scores`` [S*L, groups, cap]; (S*L index = seq * layers + layer).
    """

    def __init__(self, *, query_heads: int, kv_heads: int, layers: int, seqs: int,
                 pool_blocks: int, table_blocks: int, budget_blocks: int, init_blocks: int,
                 local_blocks: int, select_group: int | None = None, rep_window: int = 32,
                 rep_topk: int = 4, out_fp16: bool = True, scale: float | None = None,
                 head_dim: int = HEAD_DIM, device: int | torch.device | None = None):
        self._lib = load()
        if device is None:
            index = torch.cuda.current_device()
        elif isinstance(device, torch.device):
            index = device.index if device.index is not None else torch.cuda.current_device()
        else:
            index = int(device)
        self.device = torch.device("cuda", index)
        group = query_heads // kv_heads
        cfg = CtxConfig(device=self.device.index, query_heads=query_heads, kv_heads=kv_heads,
                        head_dim=head_dim, layers=layers, seqs=seqs, pool_blocks=pool_blocks,
                        table_blocks=table_blocks, budget_blocks=budget_blocks,
                        init_blocks=init_blocks, local_blocks=local_blocks,
                        select_group=select_group or group, rep_window=rep_window,
                        rep_topk=rep_topk, out_fp16=int(out_fp16),
                        scale=scale if scale is not None else 1.0 / math.sqrt(head_dim))
        self.config = cfg
        h = C.c_void_p()
        check(self._lib.sa_ctx_create(C.byref(cfg), C.byref(h)), "sa_ctx_create")
        self._h = h
        self.stream = torch.cuda.current_stream(self.device)
        check(self._lib.sa_ctx_set_stream(h, self.stream.cuda_stream), "sa_ctx_set_stream")
        p = CtxPtrs()
        check(self._lib.sa_ctx_get_ptrs(h, C.byref(p)), "sa_ctx_get_ptrs")
        self.qh, self.kh, self.layers, self.seqs = query_heads, kv_heads, layers, seqs
        self.num_sl = seqs * layers
        self.n_groups = query_heads // cfg.select_group
        self.budget = budget_blocks
        self.table_blocks = table_blocks
        self.cap = (table_blocks + 3) & ~3
        self.out_fp16 = bool(out_fp16)
        d, n = self.device, self.num_sl
        self.pool = _view(p.pool, (pool_blocks, kv_heads, 2, BLOCK_TOKENS, head_dim), torch.float16, d)
        self.reps = _view(p.reps, (n, query_heads, head_dim, self.cap), torch.float32, d)
        self.table = _view(p.table, (n, table_blocks), torch.int32, d)
        self.num_sealed = _view(p.num_sealed, (n,), torch.int32, d)
        self.tail_block = _view(p.tail_block, (n,), torch.int32, d)
        self.tail_len = _view(p.tail_len, (n,), torch.int32, d)
        self.generation = _view(p.generation, (n,), torch.int32, d)
        self.query_ring = _view(p.query_ring, (n, query_heads, BLOCK_TOKENS, head_dim),
                                torch.float32, d)
        self.selected = _view(p.selected, (n, self.n_groups, budget_blocks), torch.int32, d)
        self.selected_count = _view(p.selected_count, (n, self.n_groups), torch.int32, d)
        self.scores = _view(p.scores, (n, self.n_groups, self.cap), torch.float32, d)
        self.free_list = _view(p.free_list, (pool_blocks,), torch.int32, d)
        self.free_top = _view(p.free_top, (1,), torch.int32, d)
        self.status = _view(p.status, (1,), torch.int32, d)

    # ---- setup
    def write_blocks(self, phys, kv_token_major: torch.Tensor) -> None:
        """Store token-major blocks [n, 32, 2, KH, 128] (the reference's row
        layout) into pool blocks `phys` (head-major)."""
        idx = torch.as_tensor(np.asarray(phys, np.int64), device=self.device)
        self.pool[idx] = kv_token_major.to(self.device).permute(0, 3, 2, 1, 4).to(torch.float16)

    def read_blocks(self, phys) -> torch.Tensor:
        """Pool blocks `phys` as token-major rows [n, 32, 2, KH, 128]."""
        idx = torch.as_tensor(np.asarray(phys, np.int64), device=self.device)
        return self.pool[idx].permute(0, 3, 2, 1, 4).contiguous()

    def reset(self) -> None:
        check(self._lib.sa_ctx_reset(self._h), "sa_ctx_reset")

    def prefill(self, seq: int, layer: int, blocks: int) -> np.ndarray:
        """Give (seq, layer) `blocks` sealed blocks + an open tail; returns physical ids."""
        phys = np.zeros(blocks + 1, np.int32)
        check(self._lib.sa_ctx_prefill(self._h, seq, layer, blocks, phys.ctypes.data),
              "sa_ctx_prefill")
        return phys

    def build_reps(self, seq: int, layer: int, first: int, count: int,
                   prompt_queries: torch.Tensor, window: int = 32, topk: int = 4,
                   per_block: bool = True) -> None:
        check(self._lib.sa_ctx_build_reps(
            self._h, seq, layer, first, count,
            _dev_ptr(prompt_queries, torch.float32, "prompt_queries"), window, topk,
            int(per_block)), "sa_ctx_build_reps")

    # ---- decode
    def _io(self, query, kv_new):
        kv_fp32 = kv_new.dtype == torch.float32
        if not kv_fp32 and kv_new.dtype not in (torch.float16, torch.int16):
            raise TypeError("kv_new must be float16 or float32")
        return (_dev_ptr(query, torch.float32, "query"), _dev_ptr(kv_new, kv_new.dtype, "kv_new"),
                int(kv_fp32))

    def new_output(self) -> torch.Tensor:
        return torch.empty(self.seqs, self.layers, self.qh, HEAD_DIM, device=self.device,
                           dtype=torch.float16 if self.out_fp16 else torch.float32)

    def step(self, query: torch.Tensor, kv_new: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
        """Append, select, attend, seal for every (seq, layer); asynchronous."""
        out = self.new_output() if out is None else out
        q, kv, f32 = self._io(query, kv_new)
        check(self._lib.sa_ctx_step(self._h, q, kv, f32, out.data_ptr()), "sa_ctx_step")
        return out

    def step_raw(self, q_raw: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor,
                 q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, positions: torch.Tensor,
                 rope_theta: float = 1.0e6, norm_eps: float = 1e-6,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """Decode step from raw projections (q/k norm + RoPE + FP16 pack fused
        with the append; sa_ctx_step_raw). q_raw [S, L, QH, 128], k_raw and v
        [S, L, KH, 128] FP32; q_norm_w, k_norm_w [L, 128]; positions [S] int32."""
        out = self.new_output() if out is None else out
        check(self._lib.sa_ctx_step_raw(
            self._h, _dev_ptr(q_raw, torch.float32, "q_raw"), _dev_ptr(k_raw, torch.float32, "k_raw"),
            _dev_ptr(v, torch.float32, "v"), _dev_ptr(q_norm_w, torch.float32, "q_norm_w"),
            _dev_ptr(k_norm_w, torch.float32, "k_norm_w"), _dev_ptr(positions, torch.int32, "positions"),
            float(rope_theta), float(norm_eps), out.data_ptr()), "sa_ctx_step_raw")
        return out

    def step_host(self, query: np.ndarray | torch.Tensor, kv_new: np.ndarray | torch.Tensor,
                  out: np.ndarray | torch.Tensor, kv_fp32: bool = False) -> None:
        """End-to-end step from host buffers (H2D, step, D2H, synchronize)."""
        def ptr(x):
            return x.data_ptr() if isinstance(x, torch.Tensor) else x.ctypes.data
        check(self._lib.sa_ctx_step_host(self._h, ptr(query), ptr(kv_new), int(kv_fp32), ptr(out)),
              "sa_ctx_step_host")

    def append(self, query, kv_new) -> None:
        q, kv, f32 = self._io(query, kv_new)
        check(self._lib.sa_ctx_append(self._h, q, kv, f32), "sa_ctx_append")

    def select(self, query) -> None:
        check(self._lib.sa_ctx_select(self._h, _dev_ptr(query, torch.float32, "query")),
              "sa_ctx_select")

    def attend(self, query, out: torch.Tensor | None = None) -> torch.Tensor:
        out = self.new_output() if out is None else out
        check(self._lib.sa_ctx_attend(self._h, _dev_ptr(query, torch.float32, "query"),
                                      out.data_ptr()), "sa_ctx_attend")
        return out

    def seal(self) -> None:
        check(self._lib.sa_ctx_seal(self._h), "sa_ctx_seal")

    def sync(self) -> int:
        """Synchronize; raise on device status bits; return them (0)."""
        bits = C.c_uint32(0)
        check(self._lib.sa_ctx_sync(self._h, C.byref(bits)), "sa_ctx_sync")
        return int(bits.value)

    def status_bits(self) -> int:
        bits = C.c_uint32(0)
        self._lib.sa_ctx_sync(self._h, C.byref(bits))
        return int(bits.value)

    def audit(self, query: torch.Tensor) -> torch.Tensor:
        """Dense attention mass per block [S*L, KH, table_blocks + 1] (the last
        entry = the open tail) for this query; see sa_ctx_audit."""
        mass = torch.empty(self.num_sl, self.kh, self.table_blocks + 1, device=self.device,
                           dtype=torch.float32)
        check(self._lib.sa_ctx_audit(self._h, _dev_ptr(query, torch.float32, "query"),
                                     mass.data_ptr()), "sa_ctx_audit")
        return mass

    def import_blocks(self, seq: int, layer: int, first: int, store: torch.Tensor) -> None:
        """Fill logical blocks [first, first + n) of (seq, layer) from store rows
        [n, 32, 2, KH, 128] FP16 (device or pinned host; sa_ctx_import_blocks)."""
        if store.dtype != torch.float16 or store.dim() != 5 or store.shape[1:] != (
                BLOCK_TOKENS, 2, self.kh, HEAD_DIM) or not store.is_contiguous():
            raise ValueError("store must be contiguous float16 [n, 32, 2, KH, 128]")
        check(self._lib.sa_ctx_import_blocks(self._h, seq, layer, first, store.shape[0],
                                             store.data_ptr()), "sa_ctx_import_blocks")

    def export_blocks(self, seq: int, layer: int, first: int, count: int,
                      out: torch.Tensor | None = None) -> torch.Tensor:
        """Logical blocks [first, first + count) of (seq, layer) as store rows
        [count, 32, 2, KH, 128] FP16 (sa_ctx_export_blocks); `out` may be a
        pinned host tensor."""
        if out is None:
            out = torch.empty(count, BLOCK_TOKENS, 2, self.kh, HEAD_DIM, dtype=torch.float16,
                              device=self.device)
        check(self._lib.sa_ctx_export_blocks(self._h, seq, layer, first, count, out.data_ptr()),
              "sa_ctx_export_blocks")
        return out

    def new_slots(self) -> torch.Tensor:
        """An empty slot table [S*L, groups, budget] (-1) for slot_correct."""
        return torch.full((self.num_sl, self.n_groups, self.budget), -1, dtype=torch.int32,
                          device=self.device)

    def slot_correct(self, slots: torch.Tensor):
        """Correct `slots` in place against the current selection; returns
        (misses, replace, stats) [S*L, groups, budget] / [..., 2] (see
        sa_ctx_slot_correct)."""
        if slots.shape != (self.num_sl, self.n_groups, self.budget) or slots.dtype != torch.int32:
            raise ValueError("slots must be int32 [S*L, groups, budget]")
        misses = torch.empty_like(slots)
        replace = torch.empty_like(slots)
        stats = torch.empty(self.num_sl, self.n_groups, 2, dtype=torch.int32, device=self.device)
        check(self._lib.sa_ctx_slot_correct(self._h, slots.data_ptr(), misses.data_ptr(),
                                            replace.data_ptr(), stats.data_ptr()),
              "sa_ctx_slot_correct")
        return misses, replace, stats

    @property
    def launches(self) -> int:
        return int(self._lib.sa_ctx_launch_count(self._h))

    # ---- decode-step graphs
    def graph_begin(self) -> None:
        """Start recording this context's stream-ordered calls into a CUDA
        graph instead of running them (sa_ctx_graph_begin). The context must
        have been created on a non-default stream."""
        check(self._lib.sa_ctx_graph_begin(self._h), "sa_ctx_graph_begin")

    def graph_end(self) -> None:
        """Close the recording, instantiate and upload it (sa_ctx_graph_end)."""
        check(self._lib.sa_ctx_graph_end(self._h), "sa_ctx_graph_end")

    def graph_launch(self) -> None:
        """Replay the recorded calls on the context's stream (sa_ctx_graph_launch)."""
        check(self._lib.sa_ctx_graph_launch(self._h), "sa_ctx_graph_launch")

    @contextlib.contextmanager
    def record(self):
        """`with ctx.record(): ctx.step(...)` records the calls of the block;
        `ctx.graph_launch()` replays them."""
        self.graph_begin()
        try:
            yield self
        except BaseException:
            # close the capture so the stream stays usable; the body's error wins
            self._lib.sa_ctx_graph_end(self._h)
            raise
        self.graph_end()

    # ---- KV-head sharding: outputs gathered over peer memory
    def gather_buffer(self, world: int) -> tuple[int, int]:
        """(device pointer, bytes) of this rank's gathered buffer for `world` ranks."""
        ptr, nbytes = C.c_void_p(), C.c_size_t()
        check(self._lib.sa_ctx_gather_buffer(self._h, world, C.byref(ptr), C.byref(nbytes)),
              "sa_ctx_gather_buffer")
        self._gather_world = world
        return int(ptr.value), int(nbytes.value)

    def gather_attach(self, rank: int, peer_ptrs) -> None:
        """Attach every rank's gathered buffer (device pointers, own at `rank`)."""
        arr = (C.c_void_p * len(peer_ptrs))(*[int(x) for x in peer_ptrs])
        check(self._lib.sa_ctx_gather_attach(self._h, rank, arr), "sa_ctx_gather_attach")

    def enable_gather(self, world: int, rank: int, group=None) -> None:
        """Exchange gathered-buffer IPC handles with the other ranks of a
        torch.distributed group and attach them (one process per GPU)."""
        import torch.distributed as dist

        own, _ = self.gather_buffer(world)
        handle = (C.c_uint8 * 64)()
        check(self._lib.sa_ipc_export(self.device.index, C.c_void_p(own), handle), "sa_ipc_export")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(own)
                continue
            buf = (C.c_uint8 * 64).from_buffer_copy(h)
            ptr = C.c_void_p()
            check(self._lib.sa_ipc_open(self.device.index, buf, C.byref(ptr)), "sa_ipc_open")
            self._opened.append(int(ptr.value))
            ptrs.append(int(ptr.value))
        self.gather_attach(rank, ptrs)
        self._gather_ptrs = (rank, ptrs)

    def gather_restart(self) -> None:
        """Re-attach the buffers of enable_gather: zero this rank's arrival
        counter and epoch (every rank calls it, with no gathered attention in
        flight anywhere, e.g. after attention launches without their waits or
        after a timed-out wait)."""
        rank, ptrs = self._gather_ptrs
        self.gather_attach(rank, ptrs)

    def gather_wait(self, view: bool = True) -> torch.Tensor | None:
        """Enqueue the wait for every rank's outputs of the latest attention;
        returns the gathered slot [S, L, world*QH, 128] (valid until the
        attention after next), or None when view is False."""
        if not view:
            check(self._lib.sa_ctx_gather_wait(self._h, None), "sa_ctx_gather_wait")
            return None
        ptr = C.c_void_p()
        check(self._lib.sa_ctx_gather_wait(self._h, C.byref(ptr)), "sa_ctx_gather_wait")
        return _view(int(ptr.value), (self.seqs, self.layers, self._gather_world * self.qh, HEAD_DIM),
                     torch.float16 if self.out_fp16 else torch.float32, self.device)

    def close(self) -> None:
        for ptr in getattr(self, "_opened", []):
            self._lib.sa_ipc_close(self.device.index, C.c_void_p(ptr))
        self._opened = []
        if getattr(self, "_h", None):
            self._lib.sa_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
