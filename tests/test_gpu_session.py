"""GPU tests of the session state machine on the fused path: replay
determinism (the reference's exact-equality assay, tests/state_mechanics.c:28-36),
fused versus primitive layers, graph replay versus layer-by-layer calls,
chained generation, observer port coverage, checkpoint and stack rollback."""
import numpy as np
import pytest

import cmachine_b200 as cm

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    m = cm.Model(cm.qwen_shape(2, 1024), 31, cm.TEST_LAW, 0)
    yield m
    m.free()


def equal(a: cm.Session, b: cm.Session):
    va, vb = a.view(), b.view()
    assert (va.position, va.pending, va.delivered) == (vb.position, vb.pending, vb.delivered)
    assert va.phase == 1 and vb.phase == 1
    assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32))
    for layer in range(a.model.shape.layers):
        for kind in (0, 1):
            assert np.array_equal(a.kv(layer, kind).view(np.uint32), b.kv(layer, kind).view(np.uint32))


def test_two_sessions_bit_identical(model):
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    for t in (5, 9, 100, 151935, 7):
        assert a.push(t) == 0 and b.push(t) == 0
    equal(a, b)
    a.free(); b.free()


def test_layer_by_layer_equals_graph_token(model):
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    for t in (3, 4, 5):
        assert a.push(t) == 0
        assert b.begin_token(t) == 0
        for _ in range(model.shape.layers):
            assert b.advance_layer() == 0
        assert b.finish_token() == 0
    equal(a, b)
    a.free(); b.free()


def persistent_pair(model, capacity):
    a, b = cm.Session(model, capacity), cm.Session(model, capacity)
    assert a.persistent(1) == 1 and b.persistent(0) == 0
    return a, b


def test_persistent_token_equals_graph(model):
    """One persistent launch per token and the per-stage token graph give the
    same bits (logits, K/V, chained generation)."""
    fresh = cm.Session(model, 64)
    assert fresh.persistent() == 0  # the token graph by default
    assert fresh.persistent(1) == 1
    assert model.L.qwen_b200_launches_per_token(fresh.runner) == 1
    fresh.free()
    a, b = persistent_pair(model, 64)
    for t in (5, 9, 100, 151935, 7):
        assert a.push(t) == 0 and b.push(t) == 0
    equal(a, b)
    sa, ia = a.generate(20)
    sb, ib = b.generate(20)
    assert sa == 0 and sb == 0 and ia == ib
    equal(a, b)
    a.free(); b.free()


@pytest.mark.parametrize("profile,position", [(0, 700), (0, 1500), (2, 3000)])
def test_persistent_long_context_equals_graph(profile, position):
    """Seeded caches beyond one attention cluster's rows (the 64-CTA split) and
    the BF16 profile: the persistent kernel equals the graph bit for bit."""
    m = cm.Model(cm.qwen_shape(2, 4096), 37, cm.TEST_LAW, profile)
    a, b = persistent_pair(m, position + 40)
    L = m.L
    for i, s in enumerate((a, b)):
        v = s.view()
        count = m.shape.layers * m.shape.kvheads * v.capacity * m.shape.head
        L.qwen_b200_seeded_fill(cm.c_void_p(v.keys), 1, 7, 500, count, 0.0, 0.5)
        L.qwen_b200_seeded_fill(cm.c_void_p(v.values), 1, 7, 501, count, 0.0, 0.5)
        assert L.qwen_b200_session_set_cursor(s.handle, position, 4242) == 0
    for t in (11, 12, 13):
        assert a.push(t) == 0 and b.push(t) == 0
    equal(a, b)
    sa, ia = a.generate(30)
    sb, ib = b.generate(30)
    assert sa == 0 and sb == 0 and ia == ib
    equal(a, b)
    a.free(); b.free(); m.free()


def test_generate_equals_advance(model):
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    for t in (2, 3, 4):
        assert a.push(t) == 0 and b.push(t) == 0
    status, ids = a.generate(12)
    assert status == 0
    ref = []
    for _ in range(12):
        assert b.advance() == 0
        ref.append(b.pending)
    assert ids == ref
    equal(a, b)
    a.free(); b.free()


def test_observer_ports_and_primitive_layer(model):
    """An armed observer runs the primitive layer; all 14 ports fire once and the
    result stays within tolerance of the fused path."""
    seen = {}
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    for t in (2, 3, 4):
        assert a.push(t) == 0 and b.push(t) == 0
    a.observe(lambda pos, layer, port, data: seen.setdefault(port, (pos, layer, data.size)), 3, 1)
    assert a.push(9) == 0 and b.push(9) == 0
    assert sorted(seen) == sorted(cm.PORT_NAMES)
    assert all(v[0] == 3 and v[1] == 1 for v in seen.values())
    assert np.max(np.abs(a.logits() - b.logits())) < 1e-3
    a.free(); b.free()


def test_checkpoint_restore_replays_exactly(model):
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    for t in (2, 3, 4):
        assert a.push(t) == 0 and b.push(t) == 0
    status, ckpt = a.checkpoint()
    assert status == 0
    assert a.push(77) == 0 and a.push(78) == 0
    assert a.restore(ckpt) == 0
    assert a.push(9) == 0 and b.push(9) == 0
    equal(a, b)
    status, frame = a.stack_push()
    assert status == 0
    assert a.advance() == 0 and a.advance() == 0
    assert a.stack_rollback(frame) == 0
    assert a.advance() == 0 and b.advance() == 0
    equal(a, b)
    a.free(); b.free()


def test_capacity_and_token_refusals(model):
    s = cm.Session(model, 3)
    assert s.push(-1) == -1 and s.push(model.shape.vocab) == -1
    for t in (1, 2, 3):
        assert s.push(t) == 0
    before = s.view()
    assert s.push(4) == -1
    after = s.view()
    assert (before.position, before.pending, before.lineage_id) == (after.position, after.pending, after.lineage_id)
    s.free()
