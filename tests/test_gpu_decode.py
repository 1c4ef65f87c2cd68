"""GPU parity of the fused decode path against the oracle (the C restatement of
the reference CPU FP32 path, oracle/qwen_oracle.c) on identical seeded weights
and token ids.

Tolerances (stated by the task for this path): max |delta logit| <= 1e-3 for
the FP32 weight profile and <= 3e-2 for the source-BF16 profile; K/V rows
within the same bound. Decoding is teacher-forced (both sides consume the
oracle's tokens); the GPU's own greedy choice must equal the oracle's wherever
the oracle's top-2 gap exceeds twice the tolerance.
"""
import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, CpuDecoder

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BF16_TOL = 3e-2


def tokens(seed: int, n: int, vocab: int):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def run_parity(shape, seed, law, profile, n_prompt, n_decode, capacity, tol, prompt_readout=True):
    model = cm.Model(shape, seed, law, profile)
    session = cm.Session(model, capacity)
    oracle = CpuDecoder(ORACLE, shape, seed, law, profile == 2, capacity)
    worst, agree, forced = 0.0, 0, 0
    try:
        prompt = tokens(seed + 1, n_prompt, shape.vocab)
        for i, t in enumerate(prompt):
            assert session.push(t) == 0
            last = i == len(prompt) - 1
            top, lo = oracle.push(t, readout=prompt_readout or last)
            if top is not None:
                worst = max(worst, float(np.max(np.abs(session.logits() - lo))))
        for _ in range(n_decode):
            gap = top[2] - top[3]
            if gap > 2 * tol:
                assert session.pending == top[0], (session.top, top)
                agree += 1
            else:
                forced += 1
            nxt = top[0]
            assert session.push(nxt) == 0
            top, lo = oracle.push(nxt)
            worst = max(worst, float(np.max(np.abs(session.logits() - lo))))
        kv_worst = 0.0
        for layer in range(shape.layers):
            for kind in (0, 1):
                kv_worst = max(kv_worst, float(np.max(np.abs(session.kv(layer, kind) - oracle.kv(layer, kind)))))
        assert worst <= tol, worst
        assert kv_worst <= tol, kv_worst
        return worst, kv_worst, agree, forced
    finally:
        oracle.close()
        session.free()
        model.free()


def test_two_layer_fp32_prefill64_decode32():
    """The reference's CPU-runnable configuration: 2 layers, FP32, 64 + 32."""
    worst, kv, agree, forced = run_parity(cm.qwen_shape(2, 4096), 11, cm.TEST_LAW, 0, 64, 32, 128, FP32_TOL)
    print(f"fp32 2-layer max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")


def test_two_layer_bf16_prefill64_decode32():
    worst, kv, agree, forced = run_parity(cm.qwen_shape(2, 4096), 12, cm.TEST_LAW, 2, 64, 32, 128, BF16_TOL)
    print(f"bf16 2-layer max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")


def test_two_layer_bench_law_long_context():
    """Split-K attention over >1k cached rows (prefill without oracle readouts)."""
    worst, kv, _, _ = run_parity(cm.qwen_shape(2, 4096), 13, cm.BENCH_LAW, 0, 1100, 4, 1200, FP32_TOL,
                                 prompt_readout=False)
    print(f"fp32 2-layer 1100-token context max|dlogit|={worst:.3e} max|dkv|={kv:.3e}")


def test_full_depth_fp32():
    """All 28 layers of Qwen2.5-1.5B, FP32 weights (the benchmark's profile)."""
    worst, kv, agree, forced = run_parity(cm.qwen_shape(28, 4096), 21, cm.BENCH_LAW, 0, 8, 8, 32, FP32_TOL)
    print(f"fp32 28-layer max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")


def test_full_depth_bf16():
    worst, kv, agree, forced = run_parity(cm.qwen_shape(28, 4096), 22, cm.TEST_LAW, 2, 8, 8, 32, BF16_TOL)
    print(f"bf16 28-layer max|dlogit|={worst:.3e} max|dkv|={kv:.3e} agree={agree} forced={forced}")
