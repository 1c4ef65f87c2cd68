"""GPU parity against the oracle at the benchmark configurations' real cache
lengths.

Prefilling thousands of positions token by token on the CPU oracle would take
minutes per case, so both sides receive the same seeded K/V context instead
(orc_write_kv / Session.write_kv, then the cursor placed after it) and decode a
few teacher-forced tokens from there. Everything the decode step computes is
then compared: the logits of every token and the K/V rows it appends. The
oracle's attention over such an injected context is pinned bit for bit to the
reference's CPU path by tests/test_oracle.py.

Lengths: 512 and 767 (the FP32 ctx-512 window), 4,096 and 4,607 (the BF16
ctx-4096 window), 6,000 (beyond the 64 x 80 = 5,120 rows the batch-1 attention
clusters stage in shared memory, so the unstaged global-read path carries most
rows), and for the batched engine the 128..8,192 spread of the 64-session
configuration, mixed in one batch.

Tolerances: max |delta logit| <= 1e-3 (FP32 weights) and <= 3e-2 (BF16
weights), K/V rows within the same bound.
"""
import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, CpuDecoder, seeded_context

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BF16_TOL = 3e-2
DECODE = 3


def inject(session, oracle, shape, seed, rows, first_token):
    for layer, pair in enumerate(seeded_context(shape, seed, rows)):
        for kind in (0, 1):
            session.write_kv(layer, kind, pair[kind])
            oracle.write_kv(layer, kind, pair[kind])
    assert session.set_cursor(rows, first_token) == 0
    oracle.set_cursor(rows)


@pytest.mark.parametrize("profile", [0, 2], ids=["fp32", "bf16"])
@pytest.mark.parametrize("rows", [512, 767, 4096, 4607, 6000])
def test_fused_decode_at_context(profile, rows):
    """Batch-1 fused token (q/k/v, cluster attention, O, MLP, readout) after
    `rows` cached positions, 2 layers, against the oracle."""
    tol = FP32_TOL if profile == 0 else BF16_TOL
    shape = cm.qwen_shape(2, 8192)
    seed = 500 + rows + profile
    model = cm.Model(shape, seed, cm.TEST_LAW, profile)
    session = cm.Session(model, rows + DECODE + 1)
    oracle = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, profile == 2, rows + DECODE + 1)
    try:
        token = (rows * 7919) % shape.vocab
        inject(session, oracle, shape, seed, rows, token)
        worst = 0.0
        for _ in range(DECODE):
            assert session.push(token) == 0
            top, logits = oracle.push(token)
            worst = max(worst, float(np.max(np.abs(session.logits() - logits))))
            if top[2] - top[3] > 2 * tol:
                assert session.pending == top[0]
            token = top[0]
        kv_worst = 0.0
        for layer in range(shape.layers):
            for kind in (0, 1):
                got, want = session.kv(layer, kind), oracle.kv(layer, kind)
                assert got.shape[1] == rows + DECODE
                assert np.array_equal(got[:, :rows], want[:, :rows])  # the injected context is untouched
                kv_worst = max(kv_worst, float(np.max(np.abs(got[:, rows:] - want[:, rows:]))))
        print(f"profile {profile} rows {rows}: max|dlogit|={worst:.3e} max|dkv|={kv_worst:.3e}")
        assert worst <= tol, worst
        assert kv_worst <= tol, kv_worst
    finally:
        oracle.close()
        session.free()
        model.free()


BATCH_ROWS = [128, 1000, 4096, 8190, 129, 999, 4097, 6000]


def test_batched_decode_at_mixed_contexts():
    """qwen_push_batch on 8 sessions whose contexts span the 64-session
    configuration's 128..8,192 range in one batch (BF16 weights, 2 layers):
    every session's logits and appended K/V rows against its own oracle
    session."""
    shape = cm.qwen_shape(2, 9216)
    seed = 777
    model = cm.Model(shape, seed, cm.TEST_LAW, 2)
    sessions, oracles = [], []
    try:
        tokens = []
        for i, rows in enumerate(BATCH_ROWS):
            s = cm.Session(model, rows + DECODE + 1)
            o = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, True, rows + DECODE + 1)
            sessions.append(s)
            oracles.append(o)
            tokens.append((rows * 131 + i) % shape.vocab)
            inject(s, o, shape, seed * 100 + i, rows, tokens[-1])
        worst = [0.0] * len(sessions)
        for _ in range(DECODE):
            assert cm.push_batch(sessions, tokens) == 0
            nxt = []
            for i, (s, o) in enumerate(zip(sessions, oracles)):
                top, logits = o.push(tokens[i])
                worst[i] = max(worst[i], float(np.max(np.abs(s.logits() - logits))))
                if top[2] - top[3] > 2 * BF16_TOL:
                    assert s.pending == top[0], (i, s.top, top)
                nxt.append(top[0])
            tokens = nxt
        kv_worst = 0.0
        for s, o, rows in zip(sessions, oracles, BATCH_ROWS):
            for layer in range(shape.layers):
                for kind in (0, 1):
                    got, want = s.kv(layer, kind), o.kv(layer, kind)
                    assert got.shape[1] == rows + DECODE
                    kv_worst = max(kv_worst, float(np.max(np.abs(got[:, rows:] - want[:, rows:]))))
        print("batched max|dlogit| per session:", ", ".join(f"{w:.2e}" for w in worst), f"max|dkv|={kv_worst:.3e}")
        assert max(worst) <= BF16_TOL, worst
        assert kv_worst <= BF16_TOL, kv_worst
    finally:
        for o in oracles:
            o.close()
        for s in sessions:
            s.free()
        model.free()
