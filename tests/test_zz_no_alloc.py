"""gpu_attention_static: the attention entry point that allocates nothing.

It serves callers that may not allocate device memory once they are running
(a host whose pool manager owns all GPU memory, a loop that cannot absorb
cudaFree's device-wide synchronisation). Its split-K scratch is a fixed device
array inside the library. This test calls it through the C ABI twice in a row,
with different inputs and lengths, and compares each result with the existing
gpu_attention entry point within the attention tolerance used by the other GPU
tests (2e-5); it also checks that the tracked allocation count does not move
and that sizes beyond the array's limit are refused without a launch. The file
is named so that pytest collects it last.
"""
import ctypes
from ctypes import c_int, c_void_p

import numpy as np
import pytest

import cmachine_b200 as cm
from cmachine_b200 import ptr

pytestmark = pytest.mark.gpu

TOL = 2e-5


def entry():
    L = cm.lib()
    fn = L.gpu_attention_static
    fn.restype = c_int
    fn.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int]
    return L, fn


def upload(L, a):
    p = L.gpu_alloc(a.nbytes)
    L.gpu_write(p, ptr(a), a.nbytes)
    return p


def test_static_scratch_attention_matches_gpu_attention_twice():
    L, static = entry()
    g = L.gpu_open()
    capacity = 1100
    buffers = []
    for call, (seed, length) in enumerate([(1, 1037), (2, 300)]):
        rng = np.random.default_rng(seed)
        q = rng.standard_normal(12 * 128).astype(np.float32)
        keys = rng.standard_normal((2, capacity, 128)).astype(np.float32)
        values = rng.standard_normal((2, capacity, 128)).astype(np.float32)
        dq, dk, dv = upload(L, q), upload(L, keys), upload(L, values)
        scores = L.gpu_alloc(12 * capacity * 4)
        expected_d, got_d = L.gpu_alloc(12 * 128 * 4), L.gpu_alloc(12 * 128 * 4)
        buffers += [dq, dk, dv, scores, expected_d, got_d]
        L.gpu_attention(g, expected_d, dq, dk, dv, scores, 12, 2, 128, capacity, length)
        L.gpu_sync()
        live = L.gpu_live_bytes()
        assert static(got_d, dq, dk, dv, 12, 2, 128, capacity, length) == 0
        L.gpu_sync()
        assert L.gpu_live_bytes() == live  # nothing was allocated
        expected = np.empty(12 * 128, np.float32)
        got = np.empty(12 * 128, np.float32)
        L.gpu_read(ptr(expected), expected_d, expected.nbytes)
        L.gpu_read(ptr(got), got_d, got.nbytes)
        err = float(np.max(np.abs(got - expected)))
        print(f"call {call + 1}: length {length}, max |static - gpu_attention| = {err:.3e}")
        assert err <= TOL
    for p in buffers:
        L.gpu_free(p)
    L.gpu_close(g)


def test_static_scratch_attention_refuses_oversize():
    L, static = entry()
    # More KV heads than the array holds, a head size other than 128, a bad length:
    # all refused on the host before any launch (null pointers are never touched).
    assert static(None, None, None, None, 40, 5, 128, 16, 8) == -1
    assert static(None, None, None, None, 12, 2, 64, 16, 8) == -1
    assert static(None, None, None, None, 12, 2, 128, 16, 17) == -1
    assert static(None, None, None, None, 12, 2, 128, 16, 0) == -1
