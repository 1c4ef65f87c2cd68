"""GPU known-answer and tolerance tests of the primitive ABI (include/gpu.h).

The first test restates the reference's own GPU primitive assay
(tests/gpu_mechanics.c:8-44): exact matvec {5,5,1}, GQA attention within 2e-5
of a double-precision evaluation, RoPE within 2e-5, top-2 ties resolved to
{0, 511}. The others compare each primitive with a float64 numpy evaluation
at the Qwen2.5-1.5B shapes.
"""
import ctypes
import math

import numpy as np
import pytest

import cmachine_b200 as cm
from cmachine_b200 import ptr

pytestmark = pytest.mark.gpu


def dev(a: np.ndarray):
    L = cm.lib()
    a = np.ascontiguousarray(a)
    p = L.gpu_alloc(max(a.nbytes, 4))
    L.gpu_write(p, ptr(a), a.nbytes)
    return p


def host(p, n, dtype=np.float32):
    out = np.empty(n, dtype)
    cm.lib().gpu_read(ptr(out), p, out.nbytes)
    return out


def test_reference_primitive_assay():
    L = cm.lib()
    g = L.gpu_open()
    w = np.array([1, 2, 3, 4, 4, 3, 2, 1, -1, 0, 1, 2], np.float32)
    x = np.array([1, -1, 2, 0], np.float32)
    dw = L.gpu_weight(ptr(w), 1, 12)
    dx = L.gpu_weight(ptr(x), 1, 4)
    dy = L.gpu_alloc(12)
    L.gpu_matvec(g, dw, 4, 3, dx, dy)
    assert list(host(dy, 3)) == [5.0, 5.0, 1.0]
    for p in (dw, dx, dy):
        L.gpu_free(p)

    q = np.array([((i % 5) - 2) / 4 for i in range(16)], np.float32)
    keys = np.zeros((2, 5, 4), np.float32)
    values = np.zeros((2, 5, 4), np.float32)
    for h in range(2):
        for t in range(3):
            for d in range(4):
                keys[h, t, d] = (h + t - d) / 8
                values[h, t, d] = (h * 3 + t + d) / 4
    dq = L.gpu_weight(ptr(q), 1, 16)
    dk, dv = L.gpu_alloc(keys.nbytes), L.gpu_alloc(values.nbytes)
    scores, out = L.gpu_alloc(4 * 5 * 4), L.gpu_alloc(16 * 4)
    L.gpu_zero(dk, keys.nbytes)
    L.gpu_zero(dv, values.nbytes)
    for t in range(3):
        rk = np.ascontiguousarray(keys[:, t, :]).reshape(-1)
        rv = np.ascontiguousarray(values[:, t, :]).reshape(-1)
        a, b = L.gpu_weight(ptr(rk), 1, 8), L.gpu_weight(ptr(rv), 1, 8)
        L.gpu_cache(dk, a, 2, 4, 5, t)
        L.gpu_cache(dv, b, 2, 4, 5, t)
        L.gpu_free(a)
        L.gpu_free(b)
    L.gpu_attention(g, out, dq, dk, dv, scores, 4, 2, 4, 5, 3)
    actual = host(out, 16)
    err = 0.0
    for h in range(4):
        p = [math.exp(sum(float(q[h * 4 + d]) * float(keys[h // 2, t, d]) for d in range(4)) / 2) for t in range(3)]
        s = sum(p)
        for d in range(4):
            expected = sum(p[t] / s * float(values[h // 2, t, d]) for t in range(3))
            err = max(err, abs(actual[h * 4 + d] - expected))
    assert err < 2e-5

    L.gpu_rope(dq, 4, 4, 7, 1e6)
    actual = host(dq, 16)
    err = 0.0
    for h in range(4):
        for d in range(2):
            angle = 7 / (1e6 ** (2.0 * d / 4))
            a, b = float(q[h * 4 + d]), float(q[h * 4 + d + 2])
            err = max(err, abs(actual[h * 4 + d] - (a * math.cos(angle) - b * math.sin(angle))))
            err = max(err, abs(actual[h * 4 + d + 2] - (b * math.cos(angle) + a * math.sin(angle))))
    assert err < 2e-5
    for p in (dq, dk, dv, scores, out):
        L.gpu_free(p)

    logits = np.zeros(600, np.float32)
    logits[0] = logits[511] = 5
    dl = L.gpu_weight(ptr(logits), 1, 600)
    top = L.gpu_top2(g, dl, 600)
    assert (top.first, top.second) == (0, 511)
    L.gpu_free(dl)
    L.gpu_close(g)


@pytest.mark.parametrize("dtype", [1, 2])
@pytest.mark.parametrize("shape", [(1536, 1536), (1536, 256), (1536, 8960), (8960, 1536), (1536, 151936), (12, 8), (4, 3)])
def test_matvec_matches_float64(dtype, shape):
    L = cm.lib()
    inp, out = shape
    rng = np.random.default_rng(inp * 7 + out)
    w = (rng.standard_normal((out, inp)) * 0.02).astype(np.float32)
    x = rng.standard_normal(inp).astype(np.float32)
    if dtype == 2:
        bits = (w.view(np.uint32) + 0x7FFF + ((w.view(np.uint32) >> 16) & 1)) >> 16
        w16 = bits.astype(np.uint16)
        w = (w16.astype(np.uint32) << 16).view(np.float32)
        dw = L.gpu_alloc(w16.nbytes)
        L.gpu_write(dw, ptr(w16), w16.nbytes)
        L.qwen_b200_register_matrix(dw, out, inp, 1)
    else:
        dw = dev(w)
    g = L.gpu_open()
    dx, dy = dev(x), L.gpu_alloc(out * 4)
    L.gpu_matvec(g, dw, inp, out, dx, dy)
    y = host(dy, out)
    ref = w.astype(np.float64) @ x.astype(np.float64)
    bound = 3e-5 * np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64)) + 1e-6
    assert np.all(np.abs(y - ref) <= bound)
    if dtype == 2:
        L.qwen_b200_unregister_matrix(dw)
    for p in (dw, dx, dy):
        L.gpu_free(p)
    L.gpu_close(g)


@pytest.mark.parametrize("length", [1, 7, 33, 512, 4097])
def test_gqa_attention_split_matches_float64(length):
    L = cm.lib()
    rng = np.random.default_rng(length)
    capacity = length + 5
    q = rng.standard_normal(12 * 128).astype(np.float32)
    keys = rng.standard_normal((2, capacity, 128)).astype(np.float32)
    values = rng.standard_normal((2, capacity, 128)).astype(np.float32)
    g = L.gpu_open()
    dq, dk, dv = dev(q), dev(keys), dev(values)
    scores, out = L.gpu_alloc(12 * capacity * 4), L.gpu_alloc(12 * 128 * 4)
    L.gpu_attention(g, out, dq, dk, dv, scores, 12, 2, 128, capacity, length)
    got = host(out, 12 * 128).reshape(12, 128)
    qd = q.astype(np.float64).reshape(12, 128)
    for h in range(12):
        k = keys[h // 6, :length].astype(np.float64)
        v = values[h // 6, :length].astype(np.float64)
        s = k @ qd[h] / math.sqrt(128)
        p = np.exp(s - s.max())
        ref = (p / p.sum()) @ v
        assert np.max(np.abs(got[h] - ref)) < 2e-5
    for p in (dq, dk, dv, scores, out):
        L.gpu_free(p)
    L.gpu_close(g)


def test_elementwise_primitives():
    L = cm.lib()
    rng = np.random.default_rng(3)
    n = 8960
    x = rng.standard_normal(n).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    dx, dy, dw, do = dev(x), dev(y), dev(w), L.gpu_alloc(n * 4)
    # swiglu: g / (1 + exp(-g)) * u
    L.gpu_swiglu(dx, dy, n)
    ref = x.astype(np.float64) / (1 + np.exp(-x.astype(np.float64))) * y
    assert np.max(np.abs(host(dx, n) - ref)) < 1e-5
    L.gpu_write(dx, ptr(x), x.nbytes)
    # rms: (x * r) * w
    L.gpu_rms(do, dx, dw, n, 1e-6)
    r = 1 / math.sqrt(float(np.mean(x.astype(np.float64) ** 2)) + 1e-6)
    assert np.max(np.abs(host(do, n) - x * r * w)) < 1e-5
    # add, bias, multiply, identical_finite
    L.gpu_add(dx, dy, n)
    assert np.array_equal(host(dx, n), x + y)
    g = L.gpu_open()
    assert L.gpu_identical_finite(g, dx, dx, n) == 1
    assert L.gpu_identical_finite(g, dx, dy, n) == 0
    L.gpu_multiply(do, dx, dy, n)
    assert np.array_equal(host(do, n), (x + y) * y)
    for p in (dx, dy, dw, do):
        L.gpu_free(p)
    L.gpu_close(g)


def test_top2_random_and_ties():
    L = cm.lib()
    rng = np.random.default_rng(5)
    g = L.gpu_open()
    for n in (1, 2, 255, 256, 151936, 300001):
        x = rng.standard_normal(n).astype(np.float32)
        if n > 10:
            x[n // 3] = x[n // 2] = x.max() + 1  # tie for first: lower id wins
        d = dev(x)
        top = L.gpu_top2(g, d, n)
        order = np.lexsort((np.arange(n), -x.astype(np.float64)))
        assert top.first == order[0]
        if n > 1:
            assert top.second == order[1]
        L.gpu_free(d)
    L.gpu_close(g)


def test_byte_codec_and_ring_attention_primitives():
    """gpu_encode_current bit for bit against the reference codec
    (src/byte_codec.h:5-9, via the oracle) including a zero row and a refused
    non-finite row; gpu_byte_attention and gpu_ring_attention (gathered rows,
    reservoir weights) within the attention tolerance of the oracle's CPU
    restatement of src/qwen_cache.inc:20-43."""
    import ctypes
    from checkers import ORACLE, codec_rows, load
    L = cm.lib()
    O = load(ORACLE)
    O.orc_ring_attention.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 3
    rng = np.random.default_rng(9)
    capacity, length = 300, 260
    key, value = L.gpu_alloc(2 * capacity * 128), L.gpu_alloc(2 * capacity * 128)
    scales, invalid = L.gpu_alloc(4 * capacity * 4), L.gpu_alloc(4)
    L.gpu_zero(key, 2 * capacity * 128)
    L.gpu_zero(value, 2 * capacity * 128)
    L.gpu_zero(scales, 4 * capacity * 4)
    want_codes = np.zeros((2, 2, capacity, 128), np.int8)
    want_scales = np.zeros((4, capacity), np.float32)
    for p in range(length):
        k = (rng.standard_normal(256) * (0.1 + p % 7)).astype(np.float32)
        v = (rng.standard_normal(256) * (0.5 + p % 3)).astype(np.float32)
        if p == 3:
            k[:] = 0
        dk, dv = dev(k), dev(v)
        assert L.gpu_encode_current(key, value, scales, dk, dv, capacity, p, invalid) == 0
        for kind, x in enumerate((k, v)):
            c, s = codec_rows(x.reshape(2, 128))
            want_codes[kind, :, p] = c
            want_scales[kind * 2:kind * 2 + 2, p] = s
        L.gpu_free(dk)
        L.gpu_free(dv)
    bad = np.ones(256, np.float32)
    bad[17] = np.nan
    db = dev(bad)
    assert L.gpu_encode_current(key, value, scales, db, db, capacity, length, invalid) == -1
    L.gpu_free(db)
    got_k = host(key, 2 * capacity * 128, np.int8).reshape(2, capacity, 128)
    got_v = host(value, 2 * capacity * 128, np.int8).reshape(2, capacity, 128)
    got_s = host(scales, 4 * capacity).reshape(4, capacity)
    assert np.array_equal(got_k[:, :length], want_codes[0, :, :length])
    assert np.array_equal(got_v[:, :length], want_codes[1, :, :length])
    assert np.array_equal(got_s[:, :length].view(np.uint32), want_scales[:, :length].view(np.uint32))
    assert want_scales[0, 3] == 1.0  # a zero row keeps scale 1

    q = rng.standard_normal(12 * 128).astype(np.float32)
    dq, out = dev(q), L.gpu_alloc(12 * 128 * 4)
    kh = np.ascontiguousarray(got_k)
    vh = np.ascontiguousarray(got_v)
    sh = np.ascontiguousarray(got_s)
    g = L.gpu_open()
    cases = [("byte", np.arange(length, dtype=np.int32), np.zeros(length, np.float32), 0),
             ("ring", rng.permutation(length)[:200].astype(np.int32), np.zeros(200, np.float32), 0),
             ("ring-weighted", rng.permutation(length)[:217].astype(np.int32),
              np.where(np.arange(217) % 3 == 0, 0.7, 0.0).astype(np.float32), 1)]
    for name, order, weights, weighted in cases:
        n = len(order)
        if name == "byte":
            L.gpu_byte_attention(g, out, dq, key, value, scales, None, None, capacity, n)
        else:
            do, dw = dev(order), dev(weights)
            L.gpu_ring_attention(g, out, dq, key, value, scales, None, None, do, dw, capacity, n, weighted)
            L.gpu_sync()
            L.gpu_free(do)
            L.gpu_free(dw)
        want = np.empty(12 * 128, np.float32)
        O.orc_ring_attention(ptr(want), ptr(q), ptr(kh), ptr(vh), ptr(sh), ptr(order), ptr(weights), capacity, n,
                             weighted)
        err = float(np.max(np.abs(host(out, 12 * 128) - want)))
        print(f"{name}: {n} rows, max |gpu - oracle| = {err:.2e}")
        assert err < 2e-5, name
    for p in (key, value, scales, invalid, dq, out):
        L.gpu_free(p)
    L.gpu_close(g)
