"""ctypes access to the CPU parity checker.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg, never by the product package. Two libraries:

* ``liboracle.so`` -- the plain-C restatement of the reference's path
  (``oracle/sa_oracle.c``, each function citing the reference file:line);
* ``_ref/libsa_ref.so`` -- the reference's own ``attention_reference.cpp`` and
  ``selection.cpp`` compiled unmodified (``oracle/Makefile``), present when the
  reference tree was available at build time.

All wrappers take and return numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libsa_ref.so"

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def reference_root_dir(reference_root: str | None = None) -> str | None:
    """The reference project's checkout: the caller's path, else the
    SA_REFERENCE_ROOT environment variable, else a checkout named `reference`
    beside this repository's directory; None when none of them holds the
    reference's sources (a machine that only runs the prebuilt libraries)."""
    candidates = [reference_root, os.environ.get("SA_REFERENCE_ROOT"),
                  str(HERE.parent.parent / "reference")]
    for c in candidates:
        if c and Path(c, "cpp", "src", "selection.cpp").exists():
            return c
    return None


def build(reference_root: str | None = None) -> None:
    """Compile liboracle.so, and _ref/libsa_ref.so when the reference tree exists."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    ref = reference_root_dir(reference_root)
    if ref is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)


class Unit(C.Structure):
    """One (sequence, layer, KV head) of a CPU decode step (sao_unit /
    saref_unit): blocks [nb + 1][32][2][KH][D] FP16 (sealed blocks, then the
    open tail), reps [QH][nb][D] FP32, query [QH][D] FP32, ids_out [budget]
    int64, out [QH/KH][D] FP32."""
    _fields_ = [("blocks", C.c_void_p), ("reps", C.c_void_p), ("query", C.c_void_p),
                ("nb", _sz), ("tail_len", _sz), ("kv_head", _sz), ("ids_out", C.c_void_p),
                ("out", C.c_void_p)]


class _Lib:
    def __init__(self, path: Path, prefix: str):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (run oracle.build())")
        self.lib = C.CDLL(str(path))
        self.prefix = prefix
        p = prefix
        L = self.lib
        getattr(L, f"{p}half_to_float").argtypes = [C.c_uint16]
        getattr(L, f"{p}half_to_float").restype = C.c_float
        getattr(L, f"{p}attention").argtypes = [_u16p, _f32p, _sz, _sz, _sz, _sz, C.c_float, _f32p]
        getattr(L, f"{p}select_shared_blocks").argtypes = [
            _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _i64p, C.POINTER(_sz), C.c_void_p]
        getattr(L, f"{p}sparse_units").argtypes = [
            C.POINTER(Unit), _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, C.c_float, C.c_int]
        getattr(L, f"{p}build_reps_per_block").argtypes = [
            _f32p, _u16p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _f32p, C.c_int]
        getattr(L, f"{p}sparse_step").argtypes = [
            _u16p, _i32p, _sz, _f32p, _f32p, _i32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz,
            _sz, _sz, _sz, C.c_float, C.c_int, _i64p, _f32p]

    def attention(self, kv, q, tokens, qh, kh, d, scale):
        out = np.zeros(qh * d, np.float32)
        rc = getattr(self.lib, f"{self.prefix}attention")(
            np.ascontiguousarray(kv, np.uint16), np.ascontiguousarray(q, np.float32),
            tokens, qh, kh, d, float(scale), out)
        if rc != 0:
            raise ValueError("invalid GQA attention dimensions")
        return out.reshape(qh, d)

    def select_shared_blocks(self, q, reps, qh, blocks, d, budget, init, local,
                             with_scores=True):
        ids = np.zeros(max(budget, 1), np.int64)
        n = _sz(0)
        scores = np.zeros(blocks, np.float32)
        rc = getattr(self.lib, f"{self.prefix}select_shared_blocks")(
            np.ascontiguousarray(q, np.float32), np.ascontiguousarray(reps, np.float32),
            qh, blocks, d, budget, init, local, ids, C.byref(n),
            scores.ctypes.data if with_scores else None)
        if rc != 0:
            raise ValueError("invalid representative selection dimensions")
        return ids[: n.value].copy(), scores

    def select_grouped(self, q, reps, qh, group, blocks, d, budget, init, local):
        """Per-group selection via the shared selector on each group's slice."""
        q = np.ascontiguousarray(q, np.float32).reshape(qh, d)
        reps = np.ascontiguousarray(reps, np.float32).reshape(qh, blocks, d)
        ids, scores = [], []
        for g in range(qh // group):
            i, s = self.select_shared_blocks(q[g * group:(g + 1) * group].copy(),
                                             reps[g * group:(g + 1) * group].copy(),
                                             group, blocks, d, budget, init, local)
            ids.append(i)
            scores.append(s)
        return np.stack(ids), np.stack(scores)

    def build_representatives(self, prompt_q, kv, tokens, qh, kh, d, block_tokens,
                              window, topk):
        blocks = tokens // block_tokens if block_tokens else 0
        values = np.zeros(max(qh * blocks * d, 1), np.float32)
        offsets = np.zeros(max(qh * blocks * topk, 1), np.int64)
        fn = getattr(self.lib, f"{self.prefix}build_representatives")
        # keep the contiguous copies alive for the call
        pq = np.ascontiguousarray(prompt_q, np.float32)
        kvc = np.ascontiguousarray(kv, np.uint16)
        args = [pq.ctypes.data, kvc.ctypes.data]
        if self.prefix == "sao_":
            fn.argtypes = [C.c_void_p, C.c_void_p] + [_sz] * 7 + [C.c_void_p] * 3
            rc = fn(*args, tokens, qh, kh, d, block_tokens, window, topk,
                    values.ctypes.data, offsets.ctypes.data, None)
        else:
            fn.argtypes = [C.c_void_p, C.c_void_p] + [_sz] * 7 + [C.c_void_p] * 2
            rc = fn(*args, tokens, qh, kh, d, block_tokens, window, topk,
                    values.ctypes.data, offsets.ctypes.data)
        if rc != 0:
            raise ValueError("invalid local-causal representative dimensions")
        return (values[: qh * blocks * d].reshape(qh, blocks, d),
                offsets[: qh * blocks * topk].reshape(qh, blocks, topk))

    def sparse_units(self, units, qh, kh, d, budget, init, local, scale, threads):
        """Run a ctypes array of Unit (arrays it points to kept alive by the
        caller): per unit select over its KV head's group, packed gather,
        attention; `threads` OpenMP threads over the units."""
        rc = getattr(self.lib, f"{self.prefix}sparse_units")(
            units, len(units), qh, kh, d, 32, budget, init, local, float(scale), int(threads))
        if rc != 0:
            raise ValueError("sparse units step failed")

    def build_reps_per_block(self, prompt_q, kv, blocks, qh, kh, d, window, topk, threads):
        """Representatives [QH][blocks][D] of consecutive 32-token blocks, each
        block built alone (the online seal's call); OpenMP over blocks."""
        values = np.zeros((qh, blocks, d), np.float32)
        rc = getattr(self.lib, f"{self.prefix}build_reps_per_block")(
            np.ascontiguousarray(prompt_q, np.float32).reshape(-1),
            np.ascontiguousarray(kv, np.uint16).reshape(-1), blocks, qh, kh, d, 32, window, topk,
            values.reshape(-1), int(threads))
        if rc != 0:
            raise ValueError("invalid representative dimensions")
        return values

    def sparse_step(self, pool, table, reps, query, tail_block, tail_len, qh, kh, d,
                    block_tokens, blocks, budget, init, local, scale, threads):
        layers = query.shape[0]
        ids = np.zeros((layers, kh, budget), np.int64)
        out = np.zeros((layers, qh, d), np.float32)
        rc = getattr(self.lib, f"{self.prefix}sparse_step")(
            np.ascontiguousarray(pool.reshape(-1), np.uint16),
            np.ascontiguousarray(table, np.int32), table.shape[1],
            np.ascontiguousarray(reps, np.float32), np.ascontiguousarray(query, np.float32),
            np.ascontiguousarray(tail_block, np.int32), tail_len, layers, qh, kh, d,
            block_tokens, blocks, budget, init, local, float(scale), int(threads),
            ids.reshape(-1), out.reshape(-1))
        if rc != 0:
            raise ValueError("sparse step failed")
        return ids, out


class Port(_Lib):
    """The plain-C restatement (always available once built)."""

    def __init__(self):
        super().__init__(PORT_LIB, "sao_")
        L = self.lib
        L.sao_float_to_half_rne.argtypes = [C.c_float]
        L.sao_float_to_half_rne.restype = C.c_uint16
        L.sao_ref_float_to_half.argtypes = [C.c_float]
        L.sao_ref_float_to_half.restype = C.c_uint16
        L.sao_half_to_float_n.argtypes = [_u16p, _f32p, _sz]
        L.sao_float_to_half_rne_n.argtypes = [_f32p, _u16p, _sz]
        L.sao_c1_fixture.argtypes = [_u16p, _f32p]
        L.sao_c21_fixture.argtypes = [_u16p, _f32p, _f32p]
        L.sao_gather_packed.argtypes = [_u16p, _i64p, _sz, _sz, _u16p, _sz, _sz, _u16p]
        L.sao_fnv_offsets.argtypes = [_i64p, _sz]
        L.sao_fnv_offsets.restype = C.c_uint64
        L.sao_lifecycle_run.argtypes = [_sz] * 8 + [C.c_void_p, C.c_void_p, C.c_void_p]

    def top4_first_max(self, scores):
        s = np.ascontiguousarray(scores, np.float32)
        out = np.zeros(4, np.int64)
        self.lib.sao_top4_first_max.argtypes = [_f32p, _sz, _i64p]
        self.lib.sao_top4_first_max(s, s.size, out)
        return out

    def received_mass(self, prompt_q, kv, tokens, qh, kh, d, block_tokens, window, topk):
        """Per-(head, token) received mass of the representative build."""
        blocks = tokens // block_tokens
        received = np.zeros(qh * tokens, np.float32)
        values = np.zeros(max(qh * blocks * d, 1), np.float32)
        offsets = np.zeros(max(qh * blocks * topk, 1), np.int64)
        pq = np.ascontiguousarray(prompt_q, np.float32)
        kvc = np.ascontiguousarray(kv, np.uint16)
        fn = self.lib.sao_build_representatives
        fn.argtypes = [C.c_void_p, C.c_void_p] + [_sz] * 7 + [C.c_void_p] * 3
        rc = fn(pq.ctypes.data, kvc.ctypes.data, tokens, qh, kh, d, block_tokens, window, topk,
                values.ctypes.data, offsets.ctypes.data, received.ctypes.data)
        if rc != 0:
            raise ValueError("invalid local-causal representative dimensions")
        return received.reshape(qh, tokens)

    def half_to_float(self, h):
        h = np.ascontiguousarray(h, np.uint16)
        out = np.empty(h.size, np.float32)
        self.lib.sao_half_to_float_n(h.reshape(-1), out, h.size)
        return out.reshape(h.shape)

    def float_to_half_rne(self, f):
        f = np.ascontiguousarray(f, np.float32)
        out = np.empty(f.size, np.uint16)
        self.lib.sao_float_to_half_rne_n(f.reshape(-1), out, f.size)
        return out.reshape(f.shape)

    def c1_fixture(self):
        kv = np.zeros(128 * 2 * 8 * 128, np.uint16)
        q = np.zeros(16 * 128, np.float32)
        self.lib.sao_c1_fixture(kv, q)
        return kv, q

    def c21_fixture(self):
        kv = np.zeros(512 * 2 * 8 * 128, np.uint16)
        pq = np.zeros(16 * 512 * 128, np.float32)
        q = np.zeros(16 * 128, np.float32)
        self.lib.sao_c21_fixture(kv, pq, q)
        return kv, pq, q

    def gather_packed(self, store, ids, block_tokens, tail, tail_tokens, token_values):
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.zeros((len(ids) * block_tokens + tail_tokens) * token_values, np.uint16)
        tail = np.ascontiguousarray(tail if tail is not None else np.zeros(1), np.uint16)
        self.lib.sao_gather_packed(np.ascontiguousarray(store.reshape(-1), np.uint16), ids,
                                   len(ids), block_tokens, tail.reshape(-1), tail_tokens,
                                   token_values, out)
        return out

    def fnv_offsets(self, offsets):
        o = np.ascontiguousarray(offsets, np.int64).reshape(-1)
        return int(self.lib.sao_fnv_offsets(o, o.size))

    def head_norm_rope(self, rows, weight, position, theta, eps):
        """Rows [..., 128] FP32 normalised and rotated (see sao_head_norm_rope)."""
        r = np.array(rows, np.float32, copy=True)
        w = np.ascontiguousarray(weight, np.float32)
        P = C.c_void_p
        self.lib.sao_head_norm_rope.argtypes = [P, _sz, P, C.c_int, C.c_float, C.c_float]
        self.lib.sao_head_norm_rope.restype = None
        self.lib.sao_head_norm_rope(r.ctypes.data, r.size // 128, w.ctypes.data, int(position),
                                    float(theta), float(eps))
        return r

    def slot_correct(self, selected, counts, slots):
        """compare_prediction per unit (see sao_slot_correct): returns the
        corrected slots, misses, replacement slots and (hits, misses)."""
        sel = np.ascontiguousarray(selected, np.int32)
        units, budget = sel.shape
        cnt = np.ascontiguousarray(counts, np.int32).reshape(units)
        sl = np.array(slots, np.int32, copy=True).reshape(units, budget)
        mi = np.empty_like(sl)
        re = np.empty_like(sl)
        st = np.empty((units, 2), np.int32)
        P = C.c_void_p
        self.lib.sao_slot_correct.argtypes = [P] * 6 + [_sz, _sz]
        self.lib.sao_slot_correct.restype = None
        self.lib.sao_slot_correct(sel.ctypes.data, cnt.ctypes.data, sl.ctypes.data, mi.ctypes.data,
                                  re.ctypes.data, st.ctypes.data, units, budget)
        return sl, mi, re, st

    def dense_block_mass(self, keys, query, block_tokens, scale):
        """audit_dense_selection's per-block mass (see sao_dense_block_mass):
        keys [tokens][head_dim] FP16 (as uint16 or float16), query
        [heads][head_dim] FP32; returns float64 [ceil(tokens / block_tokens)]."""
        k = np.ascontiguousarray(keys).view(np.uint16) if np.asarray(keys).dtype == np.float16 \
            else np.ascontiguousarray(keys, np.uint16)
        tokens, d = k.shape
        q = np.ascontiguousarray(query, np.float32).reshape(-1, d)
        out = np.zeros(max(1, -(-tokens // block_tokens)), np.float64)
        P = C.c_void_p
        fn = self.lib.sao_dense_block_mass
        fn.argtypes = [P, _sz, _sz, P, _sz, _sz, _sz, C.c_float, P]
        fn.restype = None
        fn(k.ctypes.data, d, tokens, q.ctypes.data, q.shape[0], d, block_tokens, float(scale),
           out.ctypes.data)
        return out[:-(-tokens // block_tokens)]

    def audit_selection(self, block_mass, selected, budget, init, local, extra_mass=0.0):
        """(selected_mass, recall) of one selection (see sao_audit_selection)."""
        m = np.ascontiguousarray(block_mass, np.float64)
        sel = np.ascontiguousarray(selected, np.int32).reshape(-1)
        a, r = C.c_double(), C.c_double()
        P = C.c_void_p
        fn = self.lib.sao_audit_selection
        fn.argtypes = [P, _sz, P, _sz, _sz, _sz, _sz, C.c_double, P, P]
        fn.restype = None
        fn(m.ctypes.data, m.size, sel.ctypes.data, sel.size, budget, init, local,
           float(extra_mass), C.byref(a), C.byref(r))
        return a.value, r.value

    def lifecycle_run(self, layers, q_heads, kv_heads, head_dim, block_tokens, local_tokens,
                      decode_tokens, initial_blocks, with_store=False, with_indices=False):
        class Res(C.Structure):
            _fields_ = [("sealed_total", _sz), ("representative_audits", _sz),
                        ("tail_tokens_layer0", _sz), ("generation_layer0", _sz),
                        ("capacity_blocks", _sz)]
        res = Res()
        capacity = initial_blocks + (decode_tokens + 31) // 32 + 1
        token_values = 2 * kv_heads * head_dim
        store = (np.zeros(layers * capacity * block_tokens * token_values, np.uint16)
                 if with_store else None)
        max_seals = layers * (decode_tokens // block_tokens + 2)
        idx = np.full(max_seals * q_heads * 4, -1, np.int64) if with_indices else None
        rc = self.lib.sao_lifecycle_run(
            layers, q_heads, kv_heads, head_dim, block_tokens, local_tokens, decode_tokens,
            initial_blocks, store.ctypes.data if store is not None else None,
            idx.ctypes.data if idx is not None else None, C.byref(res))
        if rc != 0:
            raise ValueError("invalid lifecycle parameters")
        out = {k: getattr(res, k) for k, _ in Res._fields_}
        out["store"] = store
        if idx is not None:
            out["rep_indices"] = idx[: res.sealed_total * q_heads * 4].reshape(-1, q_heads, 4)
        return out


class Reference(_Lib):
    """The reference's own functions compiled from its sources."""

    def __init__(self):
        super().__init__(REF_LIB, "saref_")
        self.lib.saref_float_to_half.argtypes = [C.c_float]
        self.lib.saref_float_to_half.restype = C.c_uint16
        self.lib.saref_max_threads.restype = C.c_int

    def float_to_half(self, value: float) -> int:
        return int(self.lib.saref_float_to_half(value))


def port() -> Port:
    return Port()


def reference() -> Reference | None:
    """The compiled reference, or None when it was not built."""
    return Reference() if REF_LIB.exists() else None
