"""Python mirror of the cmachine Qwen2.5 session API on the B200 library.

The product is libcmachine_b200.so (C ABI: include/gpu.h, include/qwen.h,
include/qwen_b200.h). This module loads it with ctypes and mirrors the
reference's C entry points (src/qwen.h) one to one -- qwen_push,
qwen_begin_token, qwen_advance_layer, qwen_finish_token, checkpoints, the
nested stack, reset -- with the same return codes, so that tests and the
benchmark drive exactly the calls a C host makes. There is no Python or CPU
fallback: a missing library raises at import of `lib()`.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_float, c_int, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libcmachine_b200.so"


class Shape(Structure):
    """QwenB200Shape (include/qwen_b200.h)."""
    _fields_ = [(n, c_int) for n in ("hidden", "layers", "qheads", "kvheads", "head", "intermediate", "vocab",
                                     "max_position")] + [("epsilon", c_float), ("theta", c_float)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class Fill(Structure):
    _fields_ = [("offset", c_float), ("scale", c_float)]


class FillLaw(Structure):
    """TcmFillLaw (include/tcm_seeded.h)."""
    _fields_ = [("matrix", Fill), ("norm", Fill), ("bias", Fill)]


class Top2(Structure):
    """TcmTop2 (include/gpu.h)."""
    _fields_ = [("first", c_int), ("second", c_int), ("first_value", c_float), ("second_value", c_float)]

    def tuple(self):
        return (self.first, self.second, self.first_value, self.second_value)


class SessionView(Structure):
    _fields_ = [(n, c_int) for n in ("position", "capacity", "pending", "layer", "phase", "delivered",
                                     "dense_layers", "fused")] + [
        ("depth", ctypes.c_uint), ("session_id", c_uint64), ("epoch", c_uint64), ("lineage_id", c_uint64),
        ("checkpoint_serial", c_uint64), ("top_frame", c_uint64), ("top", Top2), ("keys", c_void_p),
        ("values", c_void_p), ("x", c_void_p), ("logits", c_void_p), ("allocated_bytes", c_size_t),
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("attention", c_void_p)]


def qwen_shape(layers: int = 28, max_position: int = 32768) -> Shape:
    """Qwen2.5-1.5B geometry (hidden 1536, 12/2 heads of 128, MLP 8960, vocab 151936)."""
    return Shape(1536, layers, 12, 2, 128, 8960, 151936, max_position, 1e-6, 1e6)


# Random-init laws: the benchmark's (linear/embedding N(0, 0.02), biases 0,
# norms 1) and the parity tests' (nonzero biases, non-unit norms).
BENCH_LAW = FillLaw(Fill(0.0, 0.02), Fill(1.0, 0.0), Fill(0.0, 0.0))
TEST_LAW = FillLaw(Fill(0.0, 0.02), Fill(1.0, 0.1), Fill(0.0, 0.05))

class RingView(Structure):
    """QwenB200RingView (host/session_view.c): the bounded cache's state."""
    _fields_ = [("cursor", c_int), ("population", c_uint64), ("rng", c_uint64)] + [
        (n, c_int) for n in ("write_slot", "sample_slot", "active", "capacity", "transaction", "fused", "layers",
                             "reservoir_count")] + [
        (n, ctypes.c_ulonglong) for n in ("calls", "published", "restores", "main_tokens")] + [
        (n, c_size_t) for n in ("arena_bytes", "gpu_bytes", "host_bytes")] + [
        ("arena", c_void_p), ("positions", c_void_p), ("order", c_void_p), ("weights", c_void_p),
        ("cut0_sample_position", c_int)]


OBSERVER = ctypes.CFUNCTYPE(None, c_void_p, c_int, c_int, c_int, POINTER(c_float), c_size_t)
PORT_NAMES = ["input", "query", "key", "value", "attention", "mlp_input", "mlp_gate", "mlp_up", "mlp_return",
              "output", "attention_write", "raw_receiver", "consumed_attention_write", "consumed_mlp_write"]

_LIB = None
TP_HANDLE_BYTES = 256  # QWEN_B200_TP_HANDLE_BYTES (include/qwen_b200.h)


def tp_gather(dist, handle: bytes) -> bytes:
    """Every rank's tensor-parallel handle, concatenated in rank order, over a
    torch.distributed process group of any backend (the handles are small
    host byte strings)."""
    assert len(handle) == TP_HANDLE_BYTES
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, handle)
    assert all(isinstance(h, bytes) and len(h) == TP_HANDLE_BYTES for h in out)
    return b"".join(out)


def tp_shares(total: int, world: int):
    """[begin, end) of each rank's share of `total` rows, as the kernels split
    the vocabulary (floor(rank * total / world))."""
    return [(r * total // world, (r + 1) * total // world) for r in range(world)]


def _declare(L, strict: bool = True):
    P = c_void_p
    sig = {
        # include/gpu.h
        "gpu_open": (P, []), "gpu_close": (None, [P]), "gpu_alloc": (P, [c_size_t]), "gpu_free": (None, [P]),
        "gpu_zero": (None, [P, c_size_t]), "gpu_copy": (None, [P, P, c_size_t]),
        "gpu_read": (None, [P, P, c_size_t]), "gpu_write": (None, [P, P, c_size_t]), "gpu_sync": (None, []),
        "gpu_live_bytes": (c_size_t, []), "gpu_peak_bytes": (c_size_t, []), "gpu_free_bytes": (c_size_t, []),
        "gpu_weight": (P, [P, c_uint32, c_size_t]),
        "gpu_matvec": (None, [P, P, c_int, c_int, P, P]),
        "gpu_rms": (None, [P, P, P, c_int, c_float]), "gpu_rms_scale": (None, [P, P, P, c_int, c_float, P]),
        "gpu_multiply": (None, [P, P, P, c_int]), "gpu_plane": (None, [P, P, P, P, c_int, c_float, c_float]),
        "gpu_plane_scaled": (None, [P, P, P, P, c_int, c_float, c_float, P]),
        "gpu_linear2": (None, [P, P, P, c_int, c_float, c_float, P]),
        "gpu_identical_finite": (c_int, [P, P, P, c_int]), "gpu_add": (None, [P, P, c_int]),
        "gpu_bias": (None, [P, P, c_int]), "gpu_rope": (None, [P, c_int, c_int, c_int, c_float]),
        "gpu_cache": (None, [P, P, c_int, c_int, c_int, c_int]),
        "gpu_attention": (None, [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int]),
        "gpu_swiglu": (None, [P, P, c_int]), "gpu_gate_anchor": (None, [P, P, P, P, P, c_int]),
        "gpu_gate_swiglu": (None, [P, P, P, P, P, P, P, c_int]), "gpu_top2": (Top2, [P, P, c_int]),
        "gpu_weight_configure": (None, [c_int]),
        "gpu_owned_weight": (P, [P, P, c_uint32, c_size_t, c_int, c_int, c_int]),
        "gpu_owned_weight_bytes": (c_size_t, [P, c_size_t]), "gpu_owned_embedding": (None, [P, P, c_int, c_int]),
        "gpu_weight_release": (None, []),
        "gpu_weight_info": (None, [POINTER(c_size_t), POINTER(c_size_t), POINTER(c_size_t), POINTER(c_int),
                                   POINTER(ctypes.c_ulonglong), POINTER(ctypes.c_ulonglong),
                                   POINTER(ctypes.c_ulonglong)]),
        "gpu_encode_current": (c_int, [P, P, P, P, P, c_int, c_int, P]),
        "gpu_byte_attention": (None, [P, P, P, P, P, P, P, P, c_int, c_int]),
        "gpu_ring_attention": (None, [P, P, P, P, P, P, P, P, P, P, c_int, c_int, c_int]),
        "gpu_attention_static": (c_int, [P, P, P, P, c_int, c_int, c_int, c_int, c_int]),
        # include/bounded_cache.h
        "ring_open": (c_int, [P, P, P, c_int, c_int, c_int, c_int, c_int]),
        "ring_begin": (c_int, [P, c_int]), "ring_abort": (c_int, [P]), "ring_finish": (c_int, [P]),
        "ring_push": (c_int, [P, c_int]), "ring_mark": (c_int, [P, POINTER(c_uint64)]),
        "ring_rollback": (c_int, [P, c_uint64]), "ring_commit": (c_int, [P, c_uint64]), "ring_close": (None, [P]),
        "ring_step": (c_int, [P, c_int, c_int, P, P, P, P, P]),
        # include/qwen.h
        "qwen_model_init_seeded": (c_int, [P, POINTER(Shape), c_uint64, POINTER(FillLaw), c_int, c_int]),
        "qwen_model_free": (None, [P]),
        "qwen_session_init": (c_int, [P, P, c_int]),
        "qwen_session_init_layout": (c_int, [P, P, c_int, c_uint64, P, P, P]),
        "qwen_session_free": (None, [P]), "qwen_abort_token": (c_int, [P]), "qwen_push": (c_int, [P, c_int]),
        "qwen_begin_token": (c_int, [P, c_int]), "qwen_advance_layer": (c_int, [P]),
        "qwen_finish_token": (c_int, [P]), "qwen_advance": (c_int, [P]), "qwen_checkpoint": (c_int, [P, P]),
        "qwen_restore": (c_int, [P, P]), "qwen_stack_push": (c_int, [P, POINTER(c_uint64)]),
        "qwen_stack_rollback": (c_int, [P, c_uint64]), "qwen_stack_commit": (c_int, [P, c_uint64]),
        "qwen_reset": (c_int, [P]), "qwen_port_name": (ctypes.c_char_p, [c_int]),
        "qwen_generate": (c_int, [P, c_int, POINTER(c_int)]),
        "qwen_complete_token": (c_int, [P]),
        "qwen_push_batch": (c_int, [P, c_int, P]),
        "qwen_prefill": (c_int, [P, P, c_int]),
        "qwen_b200_batch_prefill": (c_int, [P, P, P, c_int, c_int, P]),
        # include/qwen_b200.h
        "qwen_b200_decoder_weight_bytes": (c_size_t, [P]),
        "qwen_b200_launches_per_token": (c_int, [P]),
        "qwen_b200_persistent": (c_int, [P, c_int]),
        "qwen_b200_persistent_tune": (c_int, [P, c_int, c_int]),
        "qwen_b200_time_stage": (c_float, [P, c_int, c_int, c_int, c_int]),
        "qwen_b200_trace": (c_int, [P, c_int]),
        "qwen_b200_trace_read": (c_int, [P, P, c_size_t]),
        "qwen_b200_enqueue": (c_int, [P, c_int, c_int, c_int]),
        "qwen_b200_last": (c_int, [P, POINTER(Top2)]),
        "qwen_b200_generate": (c_int, [P, c_int, c_int, c_int, POINTER(c_int), POINTER(Top2)]),
        "qwen_b200_token": (c_int, [P, c_int, c_int, POINTER(Top2)]),
        "qwen_b200_mark": (None, [c_int]), "qwen_b200_elapsed_ms": (c_float, [c_int, c_int]),
        "qwen_b200_set_device": (None, [c_int]), "qwen_b200_sm_count": (c_int, []),
        "qwen_b200_seeded_fill": (None, [P, c_int, c_uint64, c_uint32, c_size_t, c_float, c_float]),
        "qwen_b200_register_matrix": (None, [P, c_int, c_int, c_int]),
        "qwen_b200_complete": (c_int, [P, POINTER(Top2)]), "qwen_b200_can_complete": (c_int, [P]),
        "qwen_b200_ring_rows": (None, [P, c_int, c_int, P, c_int, c_int, c_int]),
        "qwen_b200_batch_create": (P, [P]), "qwen_b200_batch_free": (None, [P]), "qwen_b200_batch_max": (c_int, []),
        "qwen_b200_batch_launches_per_step": (c_int, [P]),
        "qwen_b200_batch_step": (c_int, [P, c_int, P, P, P, P]),
        "qwen_b200_batch_enqueue": (c_int, [P, c_int, P, P, P, c_int]),
        "qwen_b200_batch_read": (c_int, [P, c_int, c_int, P, P]),
        "qwen_b200_batch_matmul": (c_int, [P, c_int, c_int, P, c_int, P, c_int]),
        "qwen_b200_batch_time_stage": (c_float, [P, c_int, P, P, P, c_int, c_int, c_int]),
        "qwen_b200_batch_trace_stage": (c_int, [P, c_int, P, P, P, c_int, c_int, P, c_int]),
        "qwen_b200_batch_tune": (c_int, [P, c_int, c_int]),
        "qwen_b200_batch_cluster_capacity": (c_int, [c_int]),
        "qwen_b200_batch_clusters": (c_int, [P, POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
        "qwen_b200_session_set_cursor": (c_int, [P, c_int, c_int]),
        "qwen_session_tp_open": (c_int, [P, c_int, c_int, P]), "qwen_session_tp_connect": (c_int, [P, P]),
        "qwen_session_tp_close": (c_int, [P]), "qwen_b200_tp_world": (c_int, [P]),
        "qwen_b200_wait_limit": (c_int, [ctypes.c_ulonglong]),
        "qwen_b200_pipeline_check": (c_int, [P, c_int, P, P, c_int]),
        "qwen_b200_unregister_matrix": (None, [P]),
        # host/session_view.c
        "qwen_b200_model_size": (c_size_t, []), "qwen_b200_session_size": (c_size_t, []),
        "qwen_b200_checkpoint_size": (c_size_t, []),
        "qwen_b200_session_view": (None, [P, POINTER(SessionView)]),
        "qwen_b200_session_set_delivered": (None, [P, c_int]),
        "qwen_b200_session_observe": (None, [P, OBSERVER, P, c_int, c_int]),
        "qwen_b200_model_weight_bytes": (c_size_t, [P]), "qwen_b200_model_decoder": (P, [P]),
        "qwen_b200_model_weight": (P, [P, c_int, c_int]), "qwen_b200_model_matrix_dtype": (c_int, [P]),
        "qwen_b200_session_runner": (P, [P]),
        "qwen_b200_ring_size": (c_size_t, []), "qwen_b200_ring_view": (None, [P, POINTER(RingView)]),
        "qwen_b200_ring_fail": (None, [P, c_int, c_int]),
    }
    for name, (res, args) in sig.items():
        try:
            fn = getattr(L, name)
        except AttributeError:
            if strict:
                raise
            continue
        fn.restype = res
        fn.argtypes = args
    return L


def load_library(path) -> ctypes.CDLL:
    """Another build of the same C ABI (e.g. the session host linked against a
    CPU primitive fake for host-logic tests); symbols it lacks stay undeclared."""
    return _declare(ctypes.CDLL(str(path)), strict=False)


def lib():
    """The loaded library; raises if it was not built (no fallback path)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m cmachine_b200.build`")
        _LIB = _declare(ctypes.CDLL(str(LIB_PATH)))
    return _LIB


def ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


class Model:
    """A seeded random-init Qwen2.5-architecture model resident on the GPU."""

    def __init__(self, shape: Shape, seed: int, law: FillLaw = BENCH_LAW, profile: int = 0, fused: bool = True,
                 library=None):
        L = self.L = library or lib()
        self.shape, self.seed, self.law, self.profile = shape, seed, law, profile
        self._buf = ctypes.create_string_buffer(L.qwen_b200_model_size())
        self.handle = ctypes.cast(self._buf, c_void_p)
        if L.qwen_model_init_seeded(self.handle, ctypes.byref(shape), seed, ctypes.byref(law), profile, int(fused)):
            raise ValueError("qwen_model_init_seeded refused the shape")
        self._live = True

    @property
    def weight_bytes(self) -> int:
        return self.L.qwen_b200_model_weight_bytes(self.handle)

    def free(self):
        if self._live:
            self.L.qwen_model_free(self.handle)
            self._live = False


class BatchSession(Structure):
    """QwenB200BatchSession (include/qwen_b200.h)."""
    _fields_ = [("keys", c_void_p), ("values", c_void_p), ("capacity", c_int), ("logits", c_void_p), ("x", c_void_p)]


def push_batch(sessions, tokens) -> int:
    """qwen_push_batch: one batched step, session i takes tokens[i]."""
    L = sessions[0].L
    n = len(sessions)
    handles = (c_void_p * n)(*[s.handle.value for s in sessions])
    toks = (c_int * n)(*tokens)
    return L.qwen_push_batch(ctypes.cast(handles, c_void_p), n, ctypes.cast(toks, c_void_p))


class Checkpoint:
    def __init__(self, L=None):
        L = L or lib()
        self._buf = ctypes.create_string_buffer(L.qwen_b200_checkpoint_size())
        self.handle = ctypes.cast(self._buf, c_void_p)


class Session:
    """A decode session; methods return the C entry point's status code."""

    def __init__(self, model: Model, capacity: int, mask: int = 0, step=None, rewind=None):
        L = self.L = model.L
        self.model = model
        self._buf = ctypes.create_string_buffer(L.qwen_b200_session_size())
        self.handle = ctypes.cast(self._buf, c_void_p)
        self._callbacks = (step, rewind)
        as_ptr = lambda f: ctypes.cast(f, c_void_p) if f is not None else None
        if L.qwen_session_init_layout(self.handle, model.handle, capacity, mask, as_ptr(step), as_ptr(rewind), None):
            raise ValueError("qwen_session_init refused")
        self._live = True
        self._observer = None

    # -- the reference's entry points (src/qwen.h:186-204)
    def push(self, token: int) -> int: return self.L.qwen_push(self.handle, token)
    def begin_token(self, token: int) -> int: return self.L.qwen_begin_token(self.handle, token)
    def advance_layer(self) -> int: return self.L.qwen_advance_layer(self.handle)
    def finish_token(self) -> int: return self.L.qwen_finish_token(self.handle)
    def advance(self) -> int: return self.L.qwen_advance(self.handle)
    def abort_token(self) -> int: return self.L.qwen_abort_token(self.handle)
    def reset(self) -> int: return self.L.qwen_reset(self.handle)

    def checkpoint(self):
        c = Checkpoint(self.L)
        return self.L.qwen_checkpoint(self.handle, c.handle), c

    def restore(self, c: Checkpoint) -> int: return self.L.qwen_restore(self.handle, c.handle)

    def stack_push(self):
        frame = c_uint64(0)
        return self.L.qwen_stack_push(self.handle, ctypes.byref(frame)), frame.value

    def stack_rollback(self, frame: int) -> int: return self.L.qwen_stack_rollback(self.handle, frame)
    def stack_commit(self, frame: int) -> int: return self.L.qwen_stack_commit(self.handle, frame)

    def prefill(self, tokens) -> int:
        """qwen_prefill: n prompt tokens at once (batched tensor-core steps on a BF16 model)."""
        arr = (c_int * len(tokens))(*[int(t) for t in tokens])
        return self.L.qwen_prefill(self.handle, arr, len(tokens))

    def generate(self, n: int):
        ids = (c_int * n)()
        status = self.L.qwen_generate(self.handle, n, ids)
        return status, list(ids)

    def set_delivered(self, delivered: int = 1): self.L.qwen_b200_session_set_delivered(self.handle, delivered)

    def observe(self, fn, position: int, layer: int):
        """Arm the observer: fn(position, layer, port_name, np.ndarray copy)."""
        L = self.L

        def trampoline(_ctx, pos, lay, port, data, count):
            host = np.empty(count, np.float32)
            L.gpu_read(ptr(host), ctypes.cast(data, c_void_p), count * 4)
            fn(pos, lay, PORT_NAMES[port], host)

        self._observer = OBSERVER(trampoline)
        L.qwen_b200_session_observe(self.handle, self._observer, None, position, layer)

    # -- state readback
    def view(self) -> SessionView:
        v = SessionView()
        self.L.qwen_b200_session_view(self.handle, ctypes.byref(v))
        return v

    @property
    def position(self) -> int: return self.view().position

    @property
    def pending(self) -> int: return self.view().pending

    @property
    def top(self): return self.view().top.tuple()

    def logits(self) -> np.ndarray:
        v = self.view()
        out = np.empty(self.model.shape.vocab, np.float32)
        self.L.gpu_read(ptr(out), c_void_p(v.logits), out.nbytes)
        return out

    def hidden(self) -> np.ndarray:
        v = self.view()
        out = np.empty(self.model.shape.hidden, np.float32)
        self.L.gpu_read(ptr(out), c_void_p(v.x), out.nbytes)
        return out

    def kv(self, layer: int, kind: int) -> np.ndarray:
        """K (kind 0) or V (kind 1) rows 0..position-1 of a dense layer: [kvheads][position][head]."""
        v, s = self.view(), self.model.shape
        out = np.empty((s.kvheads, v.position, s.head), np.float32)
        base = (v.values if kind else v.keys) + layer * s.kvheads * v.capacity * s.head * 4
        for h in range(s.kvheads):
            if v.position:
                self.L.gpu_read(ptr(out[h]), c_void_p(base + h * v.capacity * s.head * 4), v.position * s.head * 4)
        return out

    def write_kv(self, layer: int, kind: int, rows: np.ndarray):
        """Write K (kind 0) or V (kind 1) rows 0..n-1 of a dense layer from [kvheads][n][head]."""
        v, s = self.view(), self.model.shape
        rows = np.ascontiguousarray(rows, np.float32)
        n = rows.shape[1]
        assert n <= v.capacity
        base = (v.values if kind else v.keys) + layer * s.kvheads * v.capacity * s.head * 4
        for h in range(s.kvheads):
            self.L.gpu_write(c_void_p(base + h * v.capacity * s.head * 4), ptr(rows[h]), n * s.head * 4)

    def set_cursor(self, position: int, pending: int) -> int:
        """Place the cursor after `position` cached rows written by write_kv (qwen_b200_session_set_cursor)."""
        return self.L.qwen_b200_session_set_cursor(self.handle, position, pending)

    def kv_rows(self):
        """This token's K and V rows of the last layer computed: ([kvheads * head], [kvheads * head])."""
        v, s = self.view(), self.model.shape
        k, vv = np.empty(s.kvheads * s.head, np.float32), np.empty(s.kvheads * s.head, np.float32)
        self.L.gpu_read(ptr(k), c_void_p(v.k), k.nbytes)
        self.L.gpu_read(ptr(vv), c_void_p(v.v), vv.nbytes)
        return k, vv

    def complete_token(self) -> int: return self.L.qwen_complete_token(self.handle)

    # -- tensor-parallel decode over several GPUs (one process per GPU)
    def tp_open(self, rank: int, world: int):
        """qwen_session_tp_open: (status, this rank's handle bytes)."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        status = self.L.qwen_session_tp_open(self.handle, rank, world, ctypes.cast(buf, c_void_p))
        return status, buf.raw

    def tp_connect(self, handles: bytes) -> int:
        """qwen_session_tp_connect with every rank's handle, in rank order."""
        buf = ctypes.create_string_buffer(handles, len(handles))
        return self.L.qwen_session_tp_connect(self.handle, ctypes.cast(buf, c_void_p))

    def tp_close(self) -> int: return self.L.qwen_session_tp_close(self.handle)

    @property
    def tp_world(self) -> int: return self.L.qwen_b200_tp_world(self.runner)

    @property
    def runner(self): return self.L.qwen_b200_session_runner(self.handle)

    def persistent(self, mode: int = -1) -> int:
        """Whole-token execution of the fused runner: 1 persistent kernel, 0 token graph, -1 query."""
        return self.L.qwen_b200_persistent(self.runner, mode)

    def free(self):
        if self._live:
            self.L.qwen_session_free(self.handle)
            self._live = False


class Ring:
    """A bounded anchors/recent/reservoir byte-codec cache over its own session
    (include/bounded_cache.h); methods return the C entry point's status code."""

    def __init__(self, model: Model, logical: int, anchors: int, recent: int, sample: int, full: int = 0):
        L = self.L = model.L
        self.model = model
        self.session = Session.__new__(Session)
        self.session.L, self.session.model = L, model
        self.session._buf = ctypes.create_string_buffer(L.qwen_b200_session_size())
        self.session.handle = ctypes.cast(self.session._buf, c_void_p)
        self.session._callbacks, self.session._observer = (None, None), None
        self._buf = ctypes.create_string_buffer(L.qwen_b200_ring_size())
        self.handle = ctypes.cast(self._buf, c_void_p)
        if L.ring_open(self.handle, self.session.handle, model.handle, logical, anchors, recent, sample, full):
            raise ValueError("ring_open refused the sizes or the model")
        self.session._live = True
        self._live = True

    def push(self, token: int) -> int: return self.L.ring_push(self.handle, token)
    def begin(self, token: int) -> int: return self.L.ring_begin(self.handle, token)
    def abort(self) -> int: return self.L.ring_abort(self.handle)
    def finish(self) -> int: return self.L.ring_finish(self.handle)
    def advance_layer(self) -> int: return self.session.advance_layer()

    def mark(self):
        frame = c_uint64(0)
        return self.L.ring_mark(self.handle, ctypes.byref(frame)), frame.value

    def rollback(self, frame: int) -> int: return self.L.ring_rollback(self.handle, frame)
    def commit(self, frame: int) -> int: return self.L.ring_commit(self.handle, frame)
    def fail(self, layer: int, position: int): self.L.qwen_b200_ring_fail(self.handle, layer, position)

    def reset(self) -> int:
        """The bounded serve's reset: qwen_reset, then zero logits (src/qwen_bounded_serve.c:58)."""
        e = self.session.reset()
        if not e:
            self.L.gpu_zero(c_void_p(self.session.view().logits), self.model.shape.vocab * 4)
        return e

    def view(self) -> RingView:
        v = RingView()
        self.L.qwen_b200_ring_view(self.handle, ctypes.byref(v))
        return v

    def positions(self) -> np.ndarray:
        v = self.view()
        return np.ctypeslib.as_array(ctypes.cast(v.positions, POINTER(c_int)), (v.capacity,)).copy()

    def order(self):
        v = self.view()
        if not v.active:
            return np.zeros(0, np.int32), np.zeros(0, np.float32)
        o = np.ctypeslib.as_array(ctypes.cast(v.order, POINTER(c_int)), (v.active,)).copy()
        w = np.ctypeslib.as_array(ctypes.cast(v.weights, POINTER(c_float)), (v.active,)).copy()
        return o, w

    def arena(self) -> np.ndarray:
        v = self.view()
        out = np.empty(v.arena_bytes, np.uint8)
        self.L.gpu_read(ptr(out), c_void_p(v.arena), v.arena_bytes)
        return out

    def logits(self) -> np.ndarray: return self.session.logits()

    def close(self):
        if self._live:
            self.L.ring_close(self.handle)
            self.session.free()
            self._live = False
