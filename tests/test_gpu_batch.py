"""Batched decode of independent sessions on the tcgen05 tensor cores.

1. The tensor-core GEMM (qwen_b200_batch_matmul: BF16 weights, activations as
   two BF16 halves, FP32 accumulation in tensor memory, split K) against a
   float64 evaluation, within 3e-5 of sum |w| |x| per output, at the decoder's
   shapes (q/k/v, O, gate/up, down) and batch sizes 1..64.
2. qwen_push_batch against the oracle (the reference CPU FP32 path restated):
   sessions with different prompt lengths step together, each logit within the
   BF16 profile's bound (3e-2), K/V rows within the same bound, greedy choices
   equal wherever the oracle's top-2 gap exceeds twice the bound; 2 and 28
   layers.
3. A session's results do not depend on the rest of the batch (bit for bit), a
   rollback replays bit for bit, and chained device-fed steps
   (qwen_b200_batch_enqueue) equal step-by-step pushes bit for bit.
4. The tensor-core attention kernel against the CUDA-core one on the same
   caches (1 to 8,190 rows), at two work-item sizes.
"""
import ctypes

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, CpuDecoder

pytestmark = pytest.mark.gpu

BF16_TOL = 3e-2


def bf16_round(w: np.ndarray) -> np.ndarray:
    u = w.astype(np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("rows,inp,n,splits", [(2048, 1536, 64, 9), (1536, 1536, 7, 12), (17920, 1536, 64, 1),
                                              (1536, 8960, 64, 12), (384, 1536, 1, 1), (256, 8960, 33, 5)])
def test_tensor_core_matmul_matches_float64(rows, inp, n, splits):
    L = cm.lib()
    rng = np.random.default_rng(rows + inp + n)
    w16 = bf16_round(rng.standard_normal((rows, inp)) * 0.02)
    w = (w16.astype(np.uint32) << 16).view(np.float32)
    x = rng.standard_normal((n, inp)).astype(np.float32)
    dw, dx, dy = L.gpu_alloc(w16.nbytes), L.gpu_alloc(x.nbytes), L.gpu_alloc(n * rows * 4)
    L.gpu_write(dw, cm.ptr(w16), w16.nbytes)
    L.gpu_write(dx, cm.ptr(x), x.nbytes)
    assert L.qwen_b200_batch_matmul(dw, rows, inp, dx, n, dy, splits) == 0
    y = np.empty((n, rows), np.float32)
    L.gpu_read(cm.ptr(y), dy, y.nbytes)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    bound = 3e-5 * (np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T) + 1e-6
    err = np.abs(y - ref)
    print(f"{rows}x{inp} n={n} splits={splits}: max err {err.max():.2e}, max err/bound {(err / bound).max():.3f}")
    assert np.all(err <= bound)
    for p in (dw, dx, dy):
        L.gpu_free(p)


def tokens(seed, n, vocab):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def run_batch_parity(layers, seed, prompt_lengths, steps, capacity):
    shape = cm.qwen_shape(layers, 4096)
    model = cm.Model(shape, seed, cm.TEST_LAW, 2)
    sessions = [cm.Session(model, capacity) for _ in prompt_lengths]
    oracles = [CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, True, capacity) for _ in prompt_lengths]
    prompts = [tokens(seed * 100 + i, n, shape.vocab) for i, n in enumerate(prompt_lengths)]
    worst, agree, forced = 0.0, 0, 0
    tops = [None] * len(sessions)
    try:
        for step in range(steps):
            batch = []
            for i, s in enumerate(sessions):
                if step < len(prompts[i]):
                    batch.append(prompts[i][step])
                else:
                    top = tops[i]
                    if top[2] - top[3] > 2 * BF16_TOL:
                        assert s.pending == top[0]
                        agree += 1
                    else:
                        forced += 1
                    batch.append(top[0])  # teacher-forced on the oracle's choice
            assert cm.push_batch(sessions, batch) == 0
            for i, (s, o) in enumerate(zip(sessions, oracles)):
                tops[i], lo = o.push(batch[i])
                worst = max(worst, float(np.max(np.abs(s.logits() - lo))))
        kv_worst = 0.0
        for s, o in zip(sessions, oracles):
            for layer in range(layers):
                for kind in (0, 1):
                    kv_worst = max(kv_worst, float(np.max(np.abs(s.kv(layer, kind) - o.kv(layer, kind)))))
        return worst, kv_worst, agree, forced
    finally:
        for o in oracles:
            o.close()
        for s in sessions:
            s.free()
        model.free()


def test_batch_two_layers_matches_oracle():
    worst, kv, agree, forced = run_batch_parity(2, 81, [1, 5, 17, 33, 2, 60, 9, 40], 72, 80)
    print(f"batch 8, 2 layers: max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")
    assert worst <= BF16_TOL and kv <= BF16_TOL


def test_batch_full_depth_matches_oracle():
    worst, kv, agree, forced = run_batch_parity(28, 82, [3, 8, 1, 12], 14, 16)
    print(f"batch 4, 28 layers: max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")
    assert worst <= BF16_TOL and kv <= BF16_TOL


def test_tensor_core_attention_matches_cuda_core_attention():
    """The batched attention on tensor-core fragments (the default: TF32 hi/lo
    operand splits, 256-row items, a separate merge) against the CUDA-core
    flash-decoding kernel, on the same seeded caches: contexts from 1 row to
    8,190 (partial 16-row stages, one and many items per session), one step
    of a 2-layer model. Logits agree to the path's FP32 rounding level (the
    attention output enters the O projection as BF16 hi/lo, about 2^-17)."""
    L = cm.lib()
    shape = cm.qwen_shape(2, 9216)
    model = cm.Model(shape, 84, cm.TEST_LAW, 2)
    lengths = [1, 7, 16, 17, 255, 256, 257, 1000, 3001, 4096, 5000, 8190]
    n = len(lengths)
    rng = np.random.default_rng(84)
    sessions = []
    for i, ln in enumerate(lengths):
        s = cm.Session(model, ln + 2)
        v = s.view()
        count = shape.layers * shape.kvheads * v.capacity * shape.head
        L.qwen_b200_seeded_fill(ctypes.c_void_p(v.keys), 1, 77, 200 + 2 * i, count, 0.0, 0.8)
        L.qwen_b200_seeded_fill(ctypes.c_void_p(v.values), 1, 77, 201 + 2 * i, count, 0.0, 0.8)
        assert L.qwen_b200_session_set_cursor(s.handle, ln, int(rng.integers(0, shape.vocab))) == 0
        sessions.append(s)
    batch = L.qwen_b200_batch_create(L.qwen_b200_model_decoder(model.handle))
    try:
        views = [s.view() for s in sessions]
        bs = (cm.BatchSession * n)(*[cm.BatchSession(v.keys, v.values, v.capacity, v.logits, v.x) for v in views])
        cp = (ctypes.c_int * n)(*[v.position for v in views])
        ct = (ctypes.c_int * n)(*[v.pending for v in views])
        tops = (cm.Top2 * n)()
        out = {}
        for kernel, rows in ((1, 1024), (0, 256), (0, 512)):
            assert L.qwen_b200_batch_tune(batch, 1, kernel) == 0
            assert L.qwen_b200_batch_tune(batch, 0, rows) == 0
            assert L.qwen_b200_batch_enqueue(batch, n, bs, ct, cp, 1) == 0
            assert L.qwen_b200_batch_read(batch, n, 1, tops, None) == 0
            out[(kernel, rows)] = [s.logits().copy() for s in sessions]
        ref = out[(1, 1024)]
        scale = max(float(np.max(np.abs(r))) for r in ref)
        for key in ((0, 256), (0, 512)):
            err = max(float(np.max(np.abs(a - b))) for a, b in zip(out[key], ref))
            print(f"attention kernel {key}: max|dlogit| {err:.3e} (logit scale {scale:.3e})")
            assert err <= 1e-4 * max(scale, 1.0)
        assert L.qwen_b200_batch_tune(batch, 1, 2) == -1
    finally:
        L.qwen_b200_batch_free(batch)
        for s in sessions:
            s.free()
        model.free()


def test_batch_composition_rollback_and_chained_steps():
    shape = cm.qwen_shape(2, 4096)
    model = cm.Model(shape, 83, cm.TEST_LAW, 2)
    L = model.L
    alone = cm.Session(model, 64)
    crowd = [cm.Session(model, 64) for _ in range(64)]
    try:
        prompt = tokens(83, 6, shape.vocab)
        others = [tokens(900 + i, 6, shape.vocab) for i in range(63)]
        for t in range(6):
            assert cm.push_batch([alone], [prompt[t]]) == 0
            assert cm.push_batch(crowd, [prompt[t]] + [o[t] for o in others]) == 0
            assert np.array_equal(alone.logits().view(np.uint32), crowd[0].logits().view(np.uint32)), t
        st, ck = alone.checkpoint()
        assert st == 0
        first = []
        for _ in range(3):
            assert cm.push_batch([alone], [alone.pending]) == 0
            first.append(alone.logits().copy())
        assert alone.restore(ck) == 0
        for i in range(3):
            assert cm.push_batch([alone], [alone.pending]) == 0
            assert np.array_equal(alone.logits().view(np.uint32), first[i].view(np.uint32)), i
        # chained device-fed steps equal step-by-step pushes
        assert alone.restore(ck) == 0
        batch = L.qwen_b200_batch_create(L.qwen_b200_model_decoder(model.handle))
        assert batch
        v = alone.view()
        bs = (cm.BatchSession * 1)(cm.BatchSession(v.keys, v.values, v.capacity, v.logits, v.x))
        toks, pos = (ctypes.c_int * 1)(alone.pending), (ctypes.c_int * 1)(alone.position)
        assert L.qwen_b200_batch_enqueue(batch, 1, bs, toks, pos, 3) == 0
        hist = (cm.Top2 * 3)()
        last = (cm.Top2 * 1)()
        assert L.qwen_b200_batch_read(batch, 1, 3, last, hist) == 0
        assert np.array_equal(alone.logits().view(np.uint32), first[2].view(np.uint32))
        ids = [hist[i].first for i in range(3)]
        assert alone.restore(ck) == 0
        want = []
        for _ in range(3):
            assert cm.push_batch([alone], [alone.pending]) == 0
            want.append(alone.pending)
        assert ids == want
        L.qwen_b200_batch_free(batch)
    finally:
        alone.free()
        for s in crowd:
            s.free()
        model.free()


def run_prefill_parity(layers, seed, head, prompt_n, follow, capacity):
    """Pushes `head` tokens, prefills `prompt_n` (qwen_prefill: batched causal
    steps of up to 64 tokens), then `follow` greedy pushes; the oracle takes the
    same tokens one by one."""
    shape = cm.qwen_shape(layers, 4096)
    model = cm.Model(shape, seed, cm.TEST_LAW, 2)
    s = cm.Session(model, capacity)
    o = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, True, capacity)
    try:
        for t in tokens(seed * 10, head, shape.vocab):
            assert s.push(t) == 0
            o.push(t, readout=False)
        prompt = tokens(seed * 10 + 1, prompt_n, shape.vocab)
        latest = s.view().lineage_id
        assert s.prefill(prompt) == 0
        for t in prompt[:-1]:
            o.push(t, readout=False)
        top, lo = o.push(prompt[-1])
        v = s.view()
        assert v.position == head + prompt_n and v.phase == 1
        assert v.lineage_id - latest == prompt_n
        worst = float(np.max(np.abs(s.logits() - lo)))
        if top[2] - top[3] > 2 * BF16_TOL:
            assert s.pending == top[0]
        kv = 0.0
        for layer in range(layers):
            for kind in (0, 1):
                kv = max(kv, float(np.max(np.abs(s.kv(layer, kind) - o.kv(layer, kind)))))
        for _ in range(follow):
            t = top[0]  # teacher-forced on the oracle's choice
            assert s.push(t) == 0
            top, lo = o.push(t)
            worst = max(worst, float(np.max(np.abs(s.logits() - lo))))
        return worst, kv
    finally:
        o.close()
        s.free()
        model.free()


def test_prefill_chunks_match_oracle():
    """75 tokens after 5 pushes: a 64-token chunk and an 11-token chunk."""
    worst, kv = run_prefill_parity(2, 91, 5, 75, 4, 100)
    print(f"prefill 2 layers: max|dlogit|={worst:.3e} max|dkv|={kv:.3e}")
    assert worst <= BF16_TOL and kv <= BF16_TOL


def test_prefill_full_depth_matches_oracle():
    worst, kv = run_prefill_parity(28, 92, 0, 10, 2, 16)
    print(f"prefill 28 layers: max|dlogit|={worst:.3e} max|dkv|={kv:.3e}")
    assert worst <= BF16_TOL and kv <= BF16_TOL


def test_prefill_of_fp32_model_is_pushes():
    """The FP32 profile has no batched engine: qwen_prefill is n pushes, bit for bit."""
    shape = cm.qwen_shape(2, 4096)
    model = cm.Model(shape, 93, cm.TEST_LAW, 0)
    a, b = cm.Session(model, 64), cm.Session(model, 64)
    try:
        prompt = tokens(930, 20, shape.vocab)
        assert a.prefill(prompt) == 0
        for t in prompt:
            assert b.push(t) == 0
        assert a.view().position == b.view().position == 20 and a.pending == b.pending
        assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32))
        for layer in range(2):
            for kind in (0, 1):
                assert np.array_equal(a.kv(layer, kind).view(np.uint32), b.kv(layer, kind).view(np.uint32))
    finally:
        a.free(); b.free(); model.free()
