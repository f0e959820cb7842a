"""sa_attention_packed_noalloc gives the workspace entry point's results.

The allocation-free entry point exists for callers that cannot call
cudaMalloc when they need attention (a server whose HBM is already reserved
for its KV pool, a decode loop that must not synchronise the device, a host
language without a device allocator). It keeps its split-K scratch in a
static 2 MiB device array instead of a caller workspace. This file is
collected last (conftest orders test_zz_* after the rest) and passes both
alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import cosine, fp16_normal

pytestmark = pytest.mark.gpu

SCALE = 1.0 / np.sqrt(128.0)


def _noalloc(pkg):
    lib = pkg.load()
    fn = lib.sa_attention_packed_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                   C.c_float, C.c_void_p, C.c_int, C.c_void_p]
    return fn


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(pkg, cuda):
    fn = _noalloc(pkg)
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row with different shapes: the second reuses the static
    # scratch left by the first (its arrival counters must start from zero).
    for tokens, qh, kh, out_fp16 in [(4100, 32, 8, False), (777, 16, 8, True)]:
        rng = np.random.default_rng(tokens)
        kv = torch.from_numpy(fp16_normal(rng, tokens * 2 * kh * 128).view(np.int16)).to(cuda)
        q = torch.from_numpy(rng.standard_normal(qh * 128, dtype=np.float32)).to(cuda)
        want = pkg.attention(kv, q, tokens, qh, kh, 128, SCALE, out_fp16=out_fp16).float()
        got = torch.empty(qh, 128, device=cuda, dtype=torch.float16 if out_fp16 else torch.float32)
        status = fn(kv.data_ptr(), q.data_ptr(), tokens, qh, kh, 128, SCALE, got.data_ptr(),
                    int(out_fp16), stream)
        assert status == 0, pkg.load().sa_last_error()
        torch.cuda.synchronize()
        got = got.float().cpu().numpy()
        want = want.cpu().numpy()
        tol, cos_min = (2e-3, 0.99999) if out_fp16 else (2e-5, 0.999999)
        assert np.abs(got - want).max() <= tol
        assert cosine(got, want) >= cos_min


def test_noalloc_refuses_problems_beyond_its_scratch(pkg, cuda):
    fn = _noalloc(pkg)
    tokens, qh, kh = 1 << 20, 64, 8  # workspace far above 2 MiB
    need = pkg.load().sa_attention_workspace_size(tokens, qh, kh)
    assert need > (2 << 20)
    kv = torch.zeros(8, dtype=torch.int16, device=cuda)  # never read: refused before launch
    q = torch.zeros(qh * 128, device=cuda)
    out = torch.empty(qh * 128, device=cuda)
    status = fn(kv.data_ptr(), q.data_ptr(), tokens, qh, kh, 128, SCALE, out.data_ptr(), 0,
                torch.cuda.current_stream().cuda_stream)
    assert status == pkg.SA_ERR_CAPACITY
    assert "2 MiB" in pkg.load().sa_last_error().decode()


def _bound_cases(pkg, qh, kh):
    """Token counts (multiples of 32) whose workspace is the largest at or
    below the 2 MiB array and the smallest above it, for this device's plan."""
    size = pkg.load().sa_attention_workspace_size
    below = above = None
    for entries in list(range(1, 4096)) + list(range(4096, 40000, 3)):
        need = size(entries * 32, qh, kh)
        if need <= (2 << 20):
            # inputs of at most ~1.3 GB for the case that runs
            if entries < 20000 and (below is None or need >= below[1]):
                below = (entries * 32, need)
        elif above is None or need < above[1]:
            above = (entries * 32, need)
    return below, above


def test_noalloc_at_its_scratch_bound(pkg, cuda):
    """The largest workspace that fits the array runs and matches the
    workspace entry point; the smallest that does not is refused, so a
    capacity check off by the array's alignment slack would show here."""
    fn = _noalloc(pkg)
    qh, kh = 64, 8
    below, above = _bound_cases(pkg, qh, kh)
    assert below is not None and above is not None
    stream = torch.cuda.current_stream().cuda_stream
    tokens = below[0]
    assert below[1] > (2 << 20) * 0.85  # close to the bound (the plan's partials come in steps)
    gen = torch.Generator(device=cuda).manual_seed(tokens)
    kv = torch.randn(tokens * 2 * kh * 128, generator=gen, device=cuda).half().view(torch.int16)
    q = torch.randn(qh * 128, generator=gen, device=cuda)
    want = pkg.attention(kv, q, tokens, qh, kh, 128, SCALE).float().cpu().numpy()
    out = torch.empty(qh, 128, device=cuda)
    status = fn(kv.data_ptr(), q.data_ptr(), tokens, qh, kh, 128, SCALE, out.data_ptr(), 0, stream)
    assert status == 0, pkg.load().sa_last_error()
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.abs(got - want).max() <= 2e-5 and cosine(got, want) >= 0.999999
    status = fn(kv.data_ptr(), q.data_ptr(), above[0], qh, kh, 128, SCALE, out.data_ptr(), 0,
                stream)
    assert status == pkg.SA_ERR_CAPACITY, (above, status)


def test_noalloc_refuses_other_head_dims(pkg, cuda):
    fn = _noalloc(pkg)
    qh, kh, tokens = 16, 8, 64
    kv = torch.zeros(tokens * 2 * kh * 64, dtype=torch.int16, device=cuda)
    q = torch.zeros(qh * 64, device=cuda)
    out = torch.empty(qh * 64, device=cuda)
    status = fn(kv.data_ptr(), q.data_ptr(), tokens, qh, kh, 64, 0.125, out.data_ptr(), 0,
                torch.cuda.current_stream().cuda_stream)
    assert status == pkg.SA_ERR_UNSUPPORTED
