"""The reference's experimental operand APIs served on the B200.

The operand programs of src/qwen.h:20-45,106-183 (QKV and lexical programs,
receiver planes, subspaces, writers, gate laws) run in the reference's own
host, src/qwen.c, over the primitive ABI. oracle/ref_operands.c scripts one
scenario per API after the reference's mechanics tests; it is linked into the
reference host over its CPU primitives (oracle/_ref/libref_cpu.so) and over
this repository's sm_100a primitives (oracle/_ref/libref_gpuhost.so). On a
seeded 2-layer model of Qwen2.5-1.5B widths, every API return code must agree
and every recorded logits vector must agree within the FP32 bound (1e-3).
"""
import ctypes

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import REF_CPU, REF_GPUHOST, load

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not (REF_CPU.exists() and REF_GPUHOST.exists()),
                                                  reason="reference host builds absent")]
SCENARIOS = {"plane": 0, "gate_law": 1, "subspace": 2, "qkv_program": 3, "lexical_program": 4, "writer": 5}
MODELS = {}


def run(path, which, shape):
    L = load(path)
    L.orc_operand_run.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_void_p]
    if path not in MODELS:
        MODELS[path] = (L, L.orc_model_create(ctypes.byref(shape), 77, ctypes.byref(cm.TEST_LAW), 0))
    model = MODELS[path][1]
    out = np.zeros((16, shape.vocab), np.float32)
    codes = np.zeros(256, np.int32)
    n = ctypes.c_int(0)
    k = L.orc_operand_run(model, which, ctypes.c_void_p(out.ctypes.data), 16, ctypes.c_void_p(codes.ctypes.data),
                          ctypes.byref(n))
    assert k > 0
    return out[:k], codes[:n.value]


@pytest.mark.parametrize("name", list(SCENARIOS))
def test_operand_api_on_b200_matches_reference_cpu(name):
    cm.lib()
    shape = cm.qwen_shape(2, 4096)
    cpu, cpu_codes = run(REF_CPU, SCENARIOS[name], shape)
    gpu, gpu_codes = run(REF_GPUHOST, SCENARIOS[name], shape)
    assert cpu_codes.tolist() == gpu_codes.tolist()
    assert cpu.shape == gpu.shape
    worst = float(np.max(np.abs(cpu - gpu)))
    print(f"{name}: {len(cpu)} logits vectors, {len(cpu_codes)} calls, max |dlogit| {worst:.3e}")
    assert worst <= 1e-3
    if name in ("plane", "gate_law", "subspace"):  # the modes really change the layer
        assert any(not np.array_equal(cpu[0], v) for v in cpu[1:])
