"""gpu_attention_static: the attention entry point that allocates nothing.

It serves callers that may not allocate device memory once they are running:
a host whose pool manager owns all GPU memory, or a loop that cannot absorb
cudaFree's device-wide synchronisation. Its split-K scratch is a fixed device
array inside the library.

The test calls it through the C ABI twice in a row per case, with different
inputs and lengths, and checks each result
  - against a float64 NumPy attention within 2e-5 (the bound of the other
    attention tests), and
  - against the existing gpu_attention entry point within the same bound.
Cases: the Qwen geometry (12 query heads over 2 KV heads) and the largest
geometry the array holds (32 query heads over 4 KV heads, 8 per KV head), at
lengths up to the capacity. Free device memory (cudaMemGetInfo, through
gpu_free_bytes) must not move across the calls once the first call on the
device has loaded the array, and sizes beyond the array's limit are refused
without a launch. The file is named so that pytest collects it last.
"""
import math
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


def float64_attention(q, keys, values, qheads, kvheads, length):
    group = qheads // kvheads
    qd = q.astype(np.float64).reshape(qheads, 128)
    out = np.empty((qheads, 128))
    for h in range(qheads):
        k = keys[h // group, :length].astype(np.float64)
        v = values[h // group, :length].astype(np.float64)
        s = k @ qd[h] / math.sqrt(128)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v
    return out.reshape(-1)


@pytest.mark.parametrize("qheads,kvheads,capacity,lengths", [
    (12, 2, 1100, (1037, 300)),
    (32, 4, 4100, (4100, 4099)),  # every KV head slot of the array, length at capacity
])
def test_static_scratch_attention_twice(qheads, kvheads, capacity, lengths):
    L, static = entry()
    g = L.gpu_open()
    buffers = []
    warmed = False
    for call, length in enumerate(lengths):
        rng = np.random.default_rng(100 * qheads + call)
        q = rng.standard_normal(qheads * 128).astype(np.float32)
        keys = rng.standard_normal((kvheads, capacity, 128)).astype(np.float32)
        values = rng.standard_normal((kvheads, capacity, 128)).astype(np.float32)
        dq, dk, dv = upload(L, q), upload(L, keys), upload(L, values)
        scores = L.gpu_alloc(qheads * capacity * 4)
        expected_d, got_d = L.gpu_alloc(qheads * 128 * 4), L.gpu_alloc(qheads * 128 * 4)
        buffers += [dq, dk, dv, scores, expected_d, got_d]
        L.gpu_attention(g, expected_d, dq, dk, dv, scores, qheads, kvheads, 128, capacity, length)
        L.gpu_sync()
        if not warmed:
            # The first call on this device may load the array (lazy module
            # loading); callers make it at start-up. Later calls allocate nothing.
            assert static(got_d, dq, dk, dv, qheads, kvheads, 128, capacity, length) == 0
            L.gpu_sync()
            warmed = True
        free_before, live_before = L.gpu_free_bytes(), L.gpu_live_bytes()
        assert static(got_d, dq, dk, dv, qheads, kvheads, 128, capacity, length) == 0
        L.gpu_sync()
        assert L.gpu_free_bytes() == free_before  # no device allocation of any kind
        assert L.gpu_live_bytes() == live_before
        expected = np.empty(qheads * 128, np.float32)
        got = np.empty(qheads * 128, np.float32)
        L.gpu_read(ptr(expected), expected_d, expected.nbytes)
        L.gpu_read(ptr(got), got_d, got.nbytes)
        ref = float64_attention(q, keys, values, qheads, kvheads, length)
        err64 = float(np.max(np.abs(got - ref)))
        err = float(np.max(np.abs(got - expected)))
        print(f"{qheads}/{kvheads} heads, call {call + 1}, length {length}: max |static - float64| = {err64:.3e}, "
              f"max |static - gpu_attention| = {err:.3e}")
        assert err64 <= TOL
        assert err <= TOL
    for p in buffers:
        L.gpu_free(p)
    L.gpu_close(g)


def test_static_scratch_attention_refuses_oversize():
    L, static = entry()
    # More KV heads than the array holds, a head size other than 128, more than
    # 8 query heads per KV head, a bad length: all refused on the host before
    # any launch (null pointers are never touched).
    assert static(None, None, None, None, 40, 5, 128, 16, 8) == -1
    assert static(None, None, None, None, 12, 2, 64, 16, 8) == -1
    assert static(None, None, None, None, 36, 4, 128, 16, 8) == -1
    assert static(None, None, None, None, 12, 2, 128, 16, 17) == -1
    assert static(None, None, None, None, 12, 2, 128, 16, 0) == -1
