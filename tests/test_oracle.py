"""The oracle pinned to the reference (CPU only).

1. oracle/liboracle.so (this repository's C restatement) reproduces the
   reference's CPU path bit for bit against the committed golden vectors,
   which tests/golden/make_golden.py produced from the reference's own
   src/qwen.c + tests/gpu_stub.c.
2. Where the reference build exists (oracle/_ref/libref_cpu.so), the two agree
   bit for bit on fresh seeds and shapes, including K/V rows.
3. The seeded generator: the C implementation matches an independent Python
   evaluation of the formula in include/tcm_seeded.h.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, REF_CPU, CpuDecoder

GOLDEN = Path(__file__).resolve().parent / "golden"


def law_of(name):
    return cm.BENCH_LAW if name == "bench" else cm.TEST_LAW


@pytest.mark.parametrize("name", ["qwen2layer_fp32_p64_g32", "qwen2layer_bf16_p16_g8"])
def test_oracle_matches_reference_golden_vectors(name):
    g = json.loads((GOLDEN / f"{name}.json").read_text())
    case = g["case"]
    shape = cm.qwen_shape(case["layers"], 4096)
    dec = CpuDecoder(ORACLE, shape, case["seed"], law_of(case["law"]), case["bf16"], case["prompt"] + case["greedy"])
    try:
        for i, step in enumerate(g["steps"]):
            if i >= case["prompt"]:
                assert step["token"] == g["steps"][i - 1]["top"][0]  # greedy continuation
            top, logits = dec.push(step["token"])
            assert [top[0], top[1]] == step["top"]
            assert [top[2], top[3]] == step["values"]
            assert hashlib.sha256(logits.tobytes()).hexdigest() == step["logits_sha256"]
            assert [float(logits[p]) for p in g["probes"]] == step["probes"]
    finally:
        dec.close()


def small_shape(layers=3, vocab=4096, hidden=256, heads=(2, 1), inter=512):
    return cm.Shape(hidden, layers, heads[0], heads[1], 128, inter, vocab, 1024, 1e-6, 1e6)


@pytest.mark.skipif(not REF_CPU.exists(), reason="reference sources not built here")
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("shape_kind", ["small", "gqa6"])
def test_oracle_bit_exact_with_reference_build(bf16, shape_kind):
    shape = small_shape() if shape_kind == "small" else small_shape(2, 8192, 1536, (12, 2), 1024)
    seed = 99 + int(bf16)
    a = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, bf16, 40)
    b = CpuDecoder(REF_CPU, shape, seed, cm.TEST_LAW, bf16, 40)
    try:
        rng = np.random.default_rng(seed)
        token = int(rng.integers(0, shape.vocab))
        for i in range(24):
            ta, la = a.push(token)
            tb, lb = b.push(token)
            assert ta == tb
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
            token = ta[0] if i % 3 else int(rng.integers(0, shape.vocab))
        for layer in range(shape.layers):
            for kind in (0, 1):
                assert np.array_equal(a.kv(layer, kind).view(np.uint32), b.kv(layer, kind).view(np.uint32))
        assert np.array_equal(a.hidden().view(np.uint32), b.hidden().view(np.uint32))
    finally:
        a.close()
        b.close()


@pytest.mark.skipif(not REF_CPU.exists(), reason="reference sources not built here")
@pytest.mark.parametrize("bf16", [False, True])
def test_oracle_bit_exact_with_reference_on_injected_context(bf16):
    """Long-context pin: both checkers get the same 1,500 seeded K/V rows per
    layer through orc_write_kv / orc_set_cursor, then decode 6 tokens. The
    oracle's attention (and everything after it) must equal the reference's
    CPU path bit for bit at that length, which is what the GPU long-context
    parity tests lean on."""
    from checkers import seeded_context
    shape = small_shape(2, 8192, 1536, (12, 2), 1024)
    shape.max_position = 2048
    rows, seed = 1500, 314 + int(bf16)
    a = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, bf16, rows + 8)
    b = CpuDecoder(REF_CPU, shape, seed, cm.TEST_LAW, bf16, rows + 8)
    try:
        for layer, pair in enumerate(seeded_context(shape, seed, rows)):
            for kind in (0, 1):
                a.write_kv(layer, kind, pair[kind])
                b.write_kv(layer, kind, pair[kind])
        a.set_cursor(rows)
        b.set_cursor(rows)
        token = 4321
        for _ in range(6):
            ta, la = a.push(token)
            tb, lb = b.push(token)
            assert ta == tb
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
            token = ta[0]
        for layer in range(shape.layers):
            for kind in (0, 1):
                ka, kb = a.kv(layer, kind), b.kv(layer, kind)
                assert ka.shape[1] == rows + 6
                assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32))
    finally:
        a.close()
        b.close()


# ---------------------------------------------------------------- seeded generator
M64 = (1 << 64) - 1


def mix64(z):
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def seeded(seed, tensor, i, offset, scale):
    base = mix64(seed ^ (((tensor + 1) * 0xD1B54A32D192ED03) & M64))
    total = 0
    for j in range(3):
        u = mix64((base + (3 * i + j + 1) * 0x9E3779B97F4A7C15) & M64)
        total += sum((u >> s) & 0xFFFF for s in (0, 16, 32, 48))
    step = np.float32(scale) * np.float32(1.0 / 65536.0)
    v = np.float32(np.float32(total - 393210) * step)
    return v if offset == 0 else np.float32(np.float32(offset) + v)


def test_seeded_generator_formula():
    shape = small_shape(layers=1, vocab=512)
    dec = CpuDecoder(ORACLE, shape, 1234, cm.TEST_LAW, False, 4)
    try:
        law = cm.TEST_LAW
        for tensor, fill, n in [(0, law.matrix, 5), (1, law.norm, 5), (2 + 5, law.bias, 5), (2 + 2, law.matrix, 5)]:
            for i in (0, 1, 2, 77, n * 31):
                assert dec.weight(tensor, i) == seeded(1234, tensor, i, fill.offset, fill.scale)
    finally:
        dec.close()


def test_seeded_generator_statistics():
    vals = np.array([seeded(5, 9, i, 0.0, 0.02) for i in range(4000)], np.float64)
    assert abs(vals.mean()) < 0.002
    assert abs(vals.std() - 0.02) < 0.001
    assert np.max(np.abs(vals)) <= 6 * 0.02


REF_RING = REF_CPU.parent / "libref_ring.so"


@pytest.mark.skipif(not REF_RING.exists(), reason="reference sources not built here")
def test_oracle_ring_bit_exact_with_reference_ring():
    """The oracle's bounded byte-codec session against the reference's
    src/bounded_cache.h over the reference host (oracle/_ref/libref_ring.so):
    arena bytes, slot positions, cursor / evictions / RNG, order, weights and
    logits bit for bit over 40 tokens at (2, 4, 3), which evicts from token 7 on."""
    import ctypes as C
    from checkers import OracleRing
    from test_ring_cpu import SEED, SHAPE, RefRing
    ours = OracleRing(SHAPE, SEED, cm.TEST_LAW, False, 1024, 2, 4, 3)
    ref = RefRing(1024, 2, 4, 3)
    try:
        for i in range(40):
            token = (i * 7 + 3) % SHAPE.vocab
            top, logits = ours.push(token)
            assert ref.push(token) == 0
            a, b = ours.state(), ref.snapshot()
            assert a["view"] == b["view"] and a["slots"] == b["slots"] and a["active"] == b["active"]
            assert np.array_equal(a["positions"], b["positions"]) and np.array_equal(a["order"], b["order"])
            assert np.array_equal(a["weights"].view(np.uint32), b["weights"])
            assert np.array_equal(a["arena"], b["arena"]), f"token {i}"
            assert np.array_equal(logits.view(np.uint32), b["logits"]), f"token {i}"
        assert a["view"][1] == 34 and a["active"] == 9
    finally:
        ours.close()
