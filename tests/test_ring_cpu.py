"""The bounded byte-codec cache (include/bounded_cache.h) against the reference's own.

oracle/_ref/libref_ring.so is the reference's src/bounded_cache.h, unchanged, over
the reference's C host (src/qwen.c) and CPU primitives (tests/gpu_stub.c), with the
codec and ring attention its mechanics test supplies. oracle/_ref/libqwen_host_cpu.so
is this repository's ring module (cmachine_b200/host/bounded_cache.c) and session
host over the same CPU primitives. Both run the same seeded 28-layer model (hidden
1536, 12/2 heads of 128, a small MLP and vocabulary so the CPU finishes in
seconds) through the same operations, and after every operation the tests compare,
bit for bit: the arena bytes, slot positions, cursor / evictions / RNG state, the
retained-row order and weights, the logits, and the session's position, pending
token, depth, epoch and lineage id. The scenario restates the reference's
tests/bounded_mechanics.c (60 tokens at (2, 4, 3) -> 54 evictions, 9 retained
rows; nested mark / rollback / replay; an injected failure on a token whose
sample slot was occupied; refusals; reset) and adds a seeded random stream.
"""
import ctypes
from ctypes import POINTER, Structure, byref, c_float, c_int, c_uint, c_uint64, c_ulonglong, c_void_p

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ROOT

REF_RING = ROOT / "oracle" / "_ref" / "libref_ring.so"
HOST_CPU = ROOT / "oracle" / "_ref" / "libqwen_host_cpu.so"
pytestmark = pytest.mark.skipif(not (REF_RING.exists() and HOST_CPU.exists()), reason="reference sources not built here")

SHAPE = cm.Shape(1536, 28, 12, 2, 128, 8, 64, 4096, 1e-6, 1e6)
SEED = 11


class OrcShape(Structure):
    _fields_ = [(n, c_int) for n in ("hidden", "layers", "qheads", "kvheads", "head", "intermediate", "vocab",
                                     "max_position")] + [("epsilon", c_float), ("theta", c_float)]


class RrState(Structure):
    _fields_ = [("cursor", c_int), ("population", c_uint64), ("rng", c_uint64)] + [
        (n, c_int) for n in ("write_slot", "sample_slot", "active", "capacity", "transaction")] + [
        (n, c_ulonglong) for n in ("calls", "published", "restores", "main_tokens")] + [
        (n, c_int) for n in ("position", "pending", "delivered", "phase", "layer")] + [("depth", c_uint)] + [
        (n, c_uint64) for n in ("epoch", "lineage", "session_id", "top_frame")] + [("top_first", c_int),
                                                                                  ("top_second", c_int)]


class RefRing:
    """The reference's ring, driven through ref_ring.c."""

    def __init__(self, logical, anchors, recent, sample):
        L = self.L = ctypes.CDLL(str(REF_RING))
        L.orc_model_create.restype = c_void_p
        L.orc_model_create.argtypes = [POINTER(OrcShape), c_uint64, c_void_p, c_int]
        L.rr_open.restype = c_void_p
        L.rr_open.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int]
        for name in ("rr_push", "rr_begin"):
            getattr(L, name).argtypes = [c_void_p, c_int]
        for name in ("rr_advance_layer", "rr_finish", "rr_abort", "rr_reset"):
            getattr(L, name).argtypes = [c_void_p]
        L.rr_mark.argtypes = [c_void_p, POINTER(c_uint64)]
        L.rr_rollback.argtypes = L.rr_commit.argtypes = [c_void_p, c_uint64]
        L.rr_fail.argtypes = [c_void_p, c_int, c_int]
        L.rr_state.argtypes = [c_void_p, POINTER(RrState)]
        L.rr_positions.argtypes = L.rr_arena.argtypes = L.rr_logits.argtypes = [c_void_p, c_void_p]
        L.rr_order.argtypes = [c_void_p, c_void_p, c_void_p]
        L.rr_arena_bytes.restype = ctypes.c_size_t
        L.rr_arena_bytes.argtypes = [c_void_p]
        shape = OrcShape(*[getattr(SHAPE, n) for n, _ in OrcShape._fields_])
        self.model = L.orc_model_create(byref(shape), SEED, ctypes.addressof(cm.TEST_LAW), 0)
        self.h = L.rr_open(self.model, logical, anchors, recent, sample, 0)
        self.rows = anchors + recent + sample
        st = RrState()
        L.rr_state(self.h, byref(st))
        self.lineage0 = st.lineage  # ids are process-wide counters: compare increments

    def push(self, t): return self.L.rr_push(self.h, t)
    def begin(self, t): return self.L.rr_begin(self.h, t)
    def advance_layer(self): return self.L.rr_advance_layer(self.h)
    def finish(self): return self.L.rr_finish(self.h)
    def abort(self): return self.L.rr_abort(self.h)
    def reset(self): return self.L.rr_reset(self.h)
    def fail(self, layer, position): self.L.rr_fail(self.h, layer, position)

    def mark(self):
        f = c_uint64(0)
        return self.L.rr_mark(self.h, byref(f)), f.value

    def rollback(self, f): return self.L.rr_rollback(self.h, f)
    def commit(self, f): return self.L.rr_commit(self.h, f)

    def snapshot(self):
        st = RrState()
        self.L.rr_state(self.h, byref(st))
        pos = np.zeros(self.rows, np.int32)
        self.L.rr_positions(self.h, pos.ctypes.data)
        order = np.zeros(self.rows, np.int32)
        weights = np.zeros(self.rows, np.float32)
        self.L.rr_order(self.h, order.ctypes.data, weights.ctypes.data)
        arena = np.zeros(self.L.rr_arena_bytes(self.h), np.uint8)
        self.L.rr_arena(self.h, arena.ctypes.data)
        logits = np.zeros(SHAPE.vocab, np.float32)
        self.L.rr_logits(self.h, logits.ctypes.data)
        return dict(view=(st.cursor, st.population, st.rng), slots=(st.write_slot, st.sample_slot), active=st.active,
                    transaction=st.transaction, session=(st.position, st.pending, st.depth, st.epoch,
                                                         st.lineage - self.lineage0, st.phase, st.top_frame != 0),
                    positions=pos, order=order[:st.active], weights=weights[:st.active].view(np.uint32),
                    arena=arena, logits=logits.view(np.uint32))


class OurRing:
    """This repository's ring module on the CPU primitives."""

    def __init__(self, L, logical, anchors, recent, sample):
        self.model = cm.Model(SHAPE, SEED, cm.TEST_LAW, 0, fused=False, library=L)
        self.ring = cm.Ring(self.model, logical, anchors, recent, sample)
        self.lineage0 = self.ring.session.view().lineage_id

    def __getattr__(self, name):
        return getattr(self.ring, name)

    def snapshot(self):
        r, s = self.ring, self.ring.session
        v, sv = r.view(), s.view()
        order, weights = r.order()
        return dict(view=(v.cursor, v.population, v.rng), slots=(v.write_slot, v.sample_slot), active=v.active,
                    transaction=v.transaction, session=(sv.position, sv.pending, sv.depth, sv.epoch,
                                                        sv.lineage_id - self.lineage0, sv.phase, sv.top_frame != 0),
                    positions=r.positions(), order=order, weights=weights.view(np.uint32), arena=r.arena(),
                    logits=r.logits().view(np.uint32))


def same(a, b, where, skip=()):
    for key in a:
        if key in skip:
            continue
        x, y = a[key], b[key]
        ok = np.array_equal(x, y) if isinstance(x, np.ndarray) else x == y
        assert ok, f"{where}: {key} differs: ours {x if not isinstance(x, np.ndarray) else x[:12]} " \
                   f"reference {y if not isinstance(y, np.ndarray) else y[:12]}"


@pytest.fixture(scope="module")
def L():
    return cm.load_library(HOST_CPU)


def both(L, logical, anchors, recent, sample):
    return OurRing(L, logical, anchors, recent, sample), RefRing(logical, anchors, recent, sample)


def test_reference_mechanics_scenario(L):
    ours, ref = both(L, 1024, 2, 4, 3)
    for i in range(60):
        assert ours.push(i % 16) == 0 and ref.push(i % 16) == 0
        same(ours.snapshot(), ref.snapshot(), f"token {i}")
    s = ours.snapshot()
    assert s["view"][1] == 54 and s["active"] == 9  # tests/bounded_mechanics.c:24
    before = ours.snapshot()
    # nested overwrite, rollback and replay
    for R in (ours, ref):
        st, parent = R.mark()
        assert st == 0 and R.push(7) == 0
        st, child = R.mark()
        assert st == 0 and R.push(8) == 0
        assert R.rollback(child) == 0 and R.push(9) == 0 and R.rollback(parent) == 0
    same(ours.snapshot(), ref.snapshot(), "after nested rollback")
    after = ours.snapshot()
    for key in ("arena", "positions", "view", "logits"):
        assert np.array_equal(before[key], after[key]) if isinstance(before[key], np.ndarray) else before[key] == after[key]
    # replay is exact, a stale handle is refused
    for R in (ours, ref):
        st, parent = R.mark()
        assert st == 0 and R.push(7) == 0 and R.push(8) == 0 and R.rollback(parent) == 0
        assert R.rollback(parent) == -1
    same(ours.snapshot(), ref.snapshot(), "after replay")
    # an injected failure on a token whose sample slot was occupied restores everything
    tested = False
    for attempt in range(128):
        snap = ours.snapshot()
        (sa, pa), (sb, pb) = ours.mark(), ref.mark()
        assert sa == 0 and sb == 0
        assert ours.begin(5) == 0 and ref.begin(5) == 0
        v = ours.ring.view()
        replacement = v.sample_slot >= 0 and v.cut0_sample_position >= 0
        # Inside a token the arena may differ: the reference copies the sampled
        # row layer by layer (src/bounded_cache.h:65), this module for every
        # layer when the token opens. Token boundaries compare the arena.
        same(ours.snapshot(), ref.snapshot(), f"attempt {attempt} begun", skip=("arena",))
        assert ours.abort() == 0 and ref.abort() == 0
        if replacement:
            pos = snap["session"][0]
            for R in (ours, ref):
                R.fail(27, pos)
                assert R.push(5) == -77
            same(ours.snapshot(), ref.snapshot(), "after injected failure")
            restored = ours.snapshot()
            for key in ("arena", "positions", "view", "logits", "session"):
                a, b = snap[key], restored[key]
                if key == "session":  # position, pending, epoch, lineage (the mark stays open)
                    a, b = a[:2] + a[3:5], b[:2] + b[3:5]
                assert np.array_equal(a, b) if isinstance(a, np.ndarray) else a == b, key
            tested = True
            assert ours.push(5) == 0 and ref.push(5) == 0
            assert ours.rollback(pa) == 0 and ref.rollback(pb) == 0
            same(ours.snapshot(), ref.snapshot(), "after retry and rollback")
            break
        assert ours.commit(pa) == 0 and ref.commit(pb) == 0
        assert ours.push(5) == 0 and ref.push(5) == 0
        same(ours.snapshot(), ref.snapshot(), f"attempt {attempt} committed")
    assert tested
    # refusals at depth two, then reset empties the cache
    for R in (ours, ref):
        st1, p = R.mark()
        st2, c = R.mark()
        assert st1 == 0 and st2 == 0
        assert R.mark()[0] == -1
        assert R.commit(c) == 0 and R.commit(p) == 0
        assert R.reset() == 0
    same(ours.snapshot(), ref.snapshot(), "after reset")
    s = ours.snapshot()
    assert s["view"] == (0, 0, 7) and np.all(s["positions"] == -1)
    ours.close()


def test_seeded_stream_with_marks_aborts_and_failures(L):
    rng = np.random.default_rng(2026)
    ours, ref = both(L, 2048, 3, 8, 5)
    frames = []  # (ours, ref) ids
    for step in range(70):
        op = rng.choice(["push"] * 6 + ["mark", "rollback", "commit", "abort", "fail"])
        pos = ours.snapshot()["session"][0]
        tok = int(rng.integers(0, SHAPE.vocab))
        if op == "push" or (op in ("rollback", "commit") and not frames):
            assert ours.push(tok) == ref.push(tok) == 0
        elif op == "mark":
            a, b = ours.mark(), ref.mark()
            assert a[0] == b[0]
            if a[0] == 0:
                frames.append((a[1], b[1]))
        elif op == "rollback":
            a, b = frames.pop()
            assert ours.rollback(a) == ref.rollback(b) == 0
        elif op == "commit":
            a, b = frames.pop()
            assert ours.commit(a) == ref.commit(b) == 0
        elif op == "abort":
            assert ours.begin(tok) == ref.begin(tok) == 0
            layers = int(rng.integers(0, 28))
            for _ in range(layers):
                assert ours.advance_layer() == ref.advance_layer() == 0
            assert ours.abort() == ref.abort() == 0
        else:
            layer = int(rng.integers(0, 28))
            ours.fail(layer, pos)
            ref.fail(layer, pos)
            assert ours.push(tok) == ref.push(tok) == -77
        same(ours.snapshot(), ref.snapshot(), f"step {step} ({op})")
    ours.close()
