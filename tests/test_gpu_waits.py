"""Bounded waits: a wait that can never complete runs out, reports, and leaves
the GPU usable.

qwen_b200_wait_limit shortens the limit of every kernel wait to 20 ms. Then
qwen_b200_pipeline_check runs the decode GEMVs' shared-memory ring on one CTA
with its producer told to issue nothing: every consumer's first stage wait
runs out, the kernel returns and the fault word comes back with the full-wait
bit. The next call, with the producer working, completes with no fault bit and
y = W x against float64. After the default limit is restored, a decode token
on a 2-layer model still matches the oracle.
"""
import time

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, CpuDecoder

pytestmark = pytest.mark.gpu


def dev(L, a):
    p = L.gpu_alloc(a.nbytes)
    L.gpu_write(p, cm.ptr(a), a.nbytes)
    return p


def test_starved_wait_runs_out_and_next_call_is_clean():
    L = cm.lib()
    rows = 40
    rng = np.random.default_rng(3)
    w = rng.standard_normal((rows, 1536)).astype(np.float32)
    x = rng.standard_normal(1536).astype(np.float32)
    dw, dx, dy = dev(L, w), dev(L, x), L.gpu_alloc(rows * 4)
    try:
        assert L.qwen_b200_wait_limit(100) == -1  # below the 1 ms floor
        assert L.qwen_b200_wait_limit(20_000_000) == 0
        t0 = time.perf_counter()
        bits = L.qwen_b200_pipeline_check(dw, rows, dx, dy, 1)
        waited = time.perf_counter() - t0
        assert bits == 1, bits  # the consumers' full-stage wait ran out
        assert waited >= 0.015
        assert L.qwen_b200_pipeline_check(dw, rows, dx, dy, 0) == 0
        y = np.empty(rows, np.float32)
        L.gpu_read(cm.ptr(y), dy, y.nbytes)
        ref = w.astype(np.float64) @ x.astype(np.float64)
        bound = 3e-5 * np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64)) + 1e-6
        assert np.all(np.abs(y - ref) <= bound)
    finally:
        assert L.qwen_b200_wait_limit(0) == 0
        for p in (dw, dx, dy):
            L.gpu_free(p)
    # The context is still usable: a fused decode token matches the oracle.
    shape = cm.qwen_shape(2, 64)
    model = cm.Model(shape, 9, cm.TEST_LAW, 0)
    s = cm.Session(model, 8)
    o = CpuDecoder(ORACLE, shape, 9, cm.TEST_LAW, False, 8)
    try:
        for t in (5, 77):
            assert s.push(t) == 0
            _, want = o.push(t)
            assert float(np.max(np.abs(s.logits() - want))) <= 1e-3
    finally:
        o.close()
        s.free()
        model.free()
