"""Seeded inputs of the golden cases, shared by make_golden.py and the tests.

Every input is regenerated from a fixed numpy seed; golden_ref.npz stores the
reference's outputs and a SHA-256 of each input, so a change in how an input
is generated shows up as a checksum mismatch rather than as a parity failure.
"""
from __future__ import annotations

import hashlib

import numpy as np

SCALE = np.float32(1.0) / np.sqrt(np.float32(128))

ATTENTION = [(1, 4, 2), (33, 8, 2), (70, 16, 4), (64, 4, 1)]          # tokens, qh, kh
SELECTION = [(16, 16, 16, 4, 1, 1, False), (8, 2, 40, 10, 1, 2, False),
             (4, 4, 30, 7, 0, 0, True), (4, 2, 5, 5, 1, 1, False)]     # qh, group, blocks, budget, init, local, ties
REPRESENTATIVES = [(32, 8, 2, 32, 4), (64, 4, 4, 5, 3), (96, 2, 1, 32, 32)]  # tokens, qh, kh, window, topk


def fp16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(
        np.float16).view(np.uint16)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def attention_case(i):
    tokens, qh, kh = ATTENTION[i]
    rng = np.random.default_rng(100 + i)
    kv = fp16(rng, tokens * 2 * kh * 128)
    q = rng.standard_normal(qh * 128, dtype=np.float32)
    return kv, q, tokens, qh, kh


def selection_case(i):
    qh, group, blocks, budget, init, local, ties = SELECTION[i]
    rng = np.random.default_rng(200 + i)
    q = rng.standard_normal((qh, 128), dtype=np.float32)
    reps = rng.standard_normal((qh, blocks, 128), dtype=np.float32) * np.float32(0.5)
    if ties:
        reps[:, 1::3] = reps[:, 0:1]
    return q, reps, qh, group, blocks, budget, init, local


def representatives_case(i):
    tokens, qh, kh, window, topk = REPRESENTATIVES[i]
    rng = np.random.default_rng(300 + i)
    kv = fp16(rng, tokens * 2 * kh * 128)
    pq = fp16(rng, qh * tokens * 128).view(np.float16).astype(np.float32)
    return kv, pq, tokens, qh, kh, window, topk
