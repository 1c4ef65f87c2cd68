"""The session host (cmachine_b200/host/qwen_host.c) on the CPU.

oracle/_ref/libqwen_host_cpu.so links this repository's host with the
reference's CPU primitive fake (tests/gpu_stub.c), the way the reference's
model-free lane runs its lifecycle assay (tests/state_mechanics.c). These tests
restate that assay's checks for the decode-path API: exact K/V and logit
equality after nested rollback and replay, foreign and stale handles, the
64-frame overflow, capacity refusal, observer port coverage, token abort,
reset, and cache-callback layers.
"""
import ctypes
from ctypes import POINTER, c_float, c_int, c_uint64, c_void_p

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ROOT

HOST_CPU = ROOT / "oracle" / "_ref" / "libqwen_host_cpu.so"
pytestmark = pytest.mark.skipif(not HOST_CPU.exists(), reason="reference sources not built here")

TINY = cm.Shape(8, 3, 4, 2, 2, 12, 16, 32, 1e-6, 1e6)


@pytest.fixture(scope="module")
def L():
    return cm.load_library(HOST_CPU)


@pytest.fixture
def model(L):
    m = cm.Model(TINY, 5, cm.TEST_LAW, 0, fused=False, library=L)
    yield m
    m.free()


def prefix(s):
    assert s.reset() == 0
    for t in (2, 3, 4):
        assert s.push(t) == 0


def equal(a, b):
    va, vb = a.view(), b.view()
    assert (va.position, va.pending, va.delivered) == (vb.position, vb.pending, vb.delivered)
    assert va.phase == 1 and vb.phase == 1
    assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32))
    for layer in range(a.model.shape.layers):
        for kind in (0, 1):
            assert np.array_equal(a.kv(layer, kind).view(np.uint32), b.kv(layer, kind).view(np.uint32))


def test_nested_stack_rollback_replays_exactly(model):
    a, b = cm.Session(model, 32), cm.Session(model, 32)
    prefix(a)
    prefix(b)
    st, outer = a.stack_push()
    assert st == 0
    assert a.push(9) == 0
    st, inner = a.stack_push()
    assert st == 0
    assert a.push(10) == 0 and a.push(11) == 0
    assert a.stack_rollback(outer) == -1          # not the top frame
    assert a.stack_rollback(inner) == 0
    assert a.push(12) == 0
    assert a.stack_rollback(outer) == 0
    assert a.view().depth == 0
    assert a.push(7) == 0 and b.push(7) == 0
    equal(a, b)
    assert a.stack_rollback(outer) == -1          # stale handle


def test_stack_overflow_is_refused_without_change(model):
    s = cm.Session(model, 32)
    prefix(s)
    frames = []
    for _ in range(64):
        st, f = s.stack_push()
        assert st == 0
        frames.append(f)
    before = bytes(s._buf)
    st, _ = s.stack_push()
    assert st == -1
    assert bytes(s._buf) == before
    for f in reversed(frames):
        assert s.stack_commit(f) == 0
    assert s.view().depth == 0


def test_foreign_and_stale_checkpoints_are_refused(model):
    a, b = cm.Session(model, 32), cm.Session(model, 32)
    st, c = a.checkpoint()
    assert st == -1                               # no token boundary yet
    prefix(a)
    prefix(b)
    st, ca = a.checkpoint()
    st2, cb = b.checkpoint()
    assert st == 0 and st2 == 0
    assert b.restore(ca) == -1                    # foreign session
    assert a.restore(ca) == 0
    st, cnew = a.checkpoint()
    assert a.restore(ca) == -1                    # superseded serial
    assert a.restore(cnew) == 0
    assert a.reset() == 0
    assert a.restore(cnew) == -1                  # older epoch


def test_capacity_refusal_is_atomic(model):
    s = cm.Session(model, 3)
    for t in (1, 2, 3):
        assert s.push(t) == 0
    before = bytes(s._buf)
    assert s.push(4) == -1
    assert bytes(s._buf) == before
    assert s.push(-1) == -1 and s.push(16) == -1


def test_observer_sees_every_port_once(model):
    s = cm.Session(model, 32)
    seen = {}

    def observer(position, layer, port, data):
        assert (position, layer) == (3, 1)
        assert port not in seen
        seen[port] = data.size

    prefix(s)
    s.observe(observer, 3, 1)
    assert s.push(9) == 0
    assert sorted(seen) == sorted(cm.PORT_NAMES)
    assert seen["mlp_gate"] == TINY.intermediate and seen["key"] == TINY.kvheads * TINY.head


def test_token_abort_restores_the_parent(model):
    s = cm.Session(model, 32)
    prefix(s)
    v0 = s.view()
    assert s.begin_token(6) == 0
    assert s.advance_layer() == 0
    assert s.abort_token() == 0
    v1 = s.view()
    assert (v1.position, v1.pending, v1.lineage_id, v1.phase) == (v0.position, v0.pending, v0.lineage_id, 0)
    assert s.abort_token() == -1
    # The aborted token leaves no trace: replaying it equals a clean push.
    t = cm.Session(model, 32)
    prefix(t)
    assert s.push(6) == 0 and t.push(6) == 0
    equal(s, t)


def test_phase_guards(model):
    s = cm.Session(model, 32)
    assert s.advance_layer() == -1 and s.finish_token() == -1
    prefix(s)
    assert s.begin_token(1) == 0
    assert s.begin_token(1) == -1                 # already inside a token
    assert s.finish_token() == -1                 # layers not done
    while s.view().layer < TINY.layers:
        assert s.advance_layer() == 0
    assert s.advance_layer() == -1
    assert s.finish_token() == 0


STEP = ctypes.CFUNCTYPE(c_int, c_void_p, c_int, c_int, POINTER(c_float), POINTER(c_float), POINTER(c_float),
                        POINTER(c_float), POINTER(c_float))
REWIND = ctypes.CFUNCTYPE(None, c_void_p, c_int, c_uint64, c_uint64)


def test_cache_callback_layers(L):
    calls, rewinds = [], []
    fail = {"layer": -1}
    width = TINY.qheads * TINY.head

    @STEP
    def step(ctx, layer, position, q, k, v, out, scores):
        calls.append((layer, position))
        if layer == fail["layer"]:
            return -77
        ctypes.memmove(out, q, width * 4)         # identity "attention": out = q
        return 0

    @REWIND
    def rewind(ctx, position, owner, epoch):
        rewinds.append((position, epoch))

    m = cm.Model(TINY, 5, cm.TEST_LAW, 0, fused=False, library=L)
    s = cm.Session(m, 32, mask=0b010, step=step, rewind=rewind)
    assert s.view().dense_layers == 2
    for t in (2, 3):
        assert s.push(t) == 0
    assert calls == [(1, 0), (1, 1)]
    fail["layer"] = 1
    assert s.push(4) == -1                        # qwen_push reports the failed layer as -1
    assert s.view().phase == 2 and s.view().layer == 1
    assert s.abort_token() == 0
    assert rewinds[-1] == (2, s.view().epoch)
    fail["layer"] = -1
    assert s.push(4) == 0 and s.view().position == 3
    assert s.reset() == 0
    assert rewinds[-1] == (0, s.view().epoch)
    s.free()
    m.free()


def test_push_batch_refuses_without_the_batched_engine(model):
    """qwen_push_batch needs a BF16 model with the fused decoder; anything else is
    refused with nothing changed (the CPU build has no fused decoder)."""
    a, b = cm.Session(model, 32), cm.Session(model, 32)
    prefix(a)
    before = bytes(a._buf)
    assert cm.push_batch([a, b], [1, 2]) == -1
    assert cm.push_batch([a, a], [1, 2]) == -1
    assert bytes(a._buf) == before


def test_prefill_equals_pushes_and_refuses_unchanged(model):
    """qwen_prefill without the batched engine is n qwen_push calls: identical
    bits and lineage count; refusals (token out of range, capacity, an open
    token) leave the session unchanged."""
    a, b = cm.Session(model, 32), cm.Session(model, 32)
    prefix(a)
    prefix(b)
    tokens = [5, 1, 7, 15, 2, 9]
    latest = b.view().lineage_id  # lineage ids are process-wide: b's prefix took the latest
    assert a.prefill(tokens) == 0
    assert a.view().lineage_id - latest == len(tokens)
    for t in tokens:
        assert b.push(t) == 0
    equal(a, b)
    before = bytes(a._buf)
    assert a.prefill([1, model.shape.vocab]) == -1
    assert a.prefill([-1]) == -1
    assert a.prefill([1] * (32 - a.view().position + 1)) == -1
    assert bytes(a._buf) == before
    assert a.begin_token(3) == 0
    assert a.prefill([1]) == -1
    a.free(); b.free()
