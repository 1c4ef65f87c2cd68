"""The reference's unchanged C host on the B200 primitive library.

oracle/_ref/libref_gpuhost.so is the reference's own src/qwen.c and
src/model.c, compiled from its sources and linked against
libcmachine_b200.so: every gpu_* call the reference host makes (src/gpu.h)
lands in this repository's sm_100a kernels. This is the drop-in boundary seen
from the caller's side. The test decodes a 2-layer seeded model through that
host and checks
  - logits against the oracle within the FP32 bound (1e-3), for a prompt and
    greedy continuation;
  - the reference's nested-stack replay (src/qwen.c:416-431): after
    qwen_stack_push, four tokens, qwen_stack_rollback and the same four tokens
    again, logits and top-2 are bit-identical to the first pass.
"""
import ctypes

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, REF_GPUHOST, CpuDecoder

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not REF_GPUHOST.exists(), reason="reference host build absent")]

FP32_TOL = 1e-3


def test_reference_host_over_b200_primitives():
    cm.lib()  # the primitive library the reference host links against
    shape = cm.qwen_shape(2, 4096)
    seed = 4242
    ref = CpuDecoder(REF_GPUHOST, shape, seed, cm.TEST_LAW, False, 64)
    oracle = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, False, 64)
    try:
        tokens = [int(t) for t in np.random.default_rng(seed).integers(0, shape.vocab, 8)]
        worst = 0.0
        for t in tokens:
            top_r, lr = ref.push(t)
            top_o, lo = oracle.push(t)
            worst = max(worst, float(np.max(np.abs(lr - lo))))
        for _ in range(8):
            nxt = top_o[0]
            top_r, lr = ref.push(nxt)
            top_o, lo = oracle.push(nxt)
            worst = max(worst, float(np.max(np.abs(lr - lo))))
        print(f"reference host on B200 primitives: max|dlogit| vs oracle = {worst:.3e}")
        assert worst <= FP32_TOL

        frame = ctypes.c_uint64(0)
        assert ref.L.orc_stack_push(ref.session, ctypes.byref(frame)) == 0
        replay = [top_r[0], 17, 151935, 4096]
        first = [ref.push(t) for t in replay]
        assert ref.L.orc_stack_rollback(ref.session, frame.value) == 0
        again = [ref.push(t) for t in replay]
        for (ta, la), (tb, lb) in zip(first, again):
            assert ta == tb
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    finally:
        ref.close()
        oracle.close()


GPU_MECHANICS = REF_GPUHOST.parent / "gpu-mechanics-b200"


@pytest.mark.skipif(not GPU_MECHANICS.exists(), reason="reference GPU mechanics build absent")
def test_reference_gpu_mechanics_on_b200_primitives():
    """The reference's own GPU test (tests/gpu_mechanics.c, unchanged) linked
    against this library instead of its cuBLAS object: exact matvec {5, 5, 1},
    attention and RoPE within 2e-5 of double precision, top-2 ties to the lower
    id, and checkpoint ownership, all asserted by the reference's code."""
    import json
    import subprocess
    proc = subprocess.run([str(GPU_MECHANICS)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr[-2000:]
    out = json.loads(proc.stdout.strip().splitlines()[-1])
    print(out)
    assert out["matvec_exact"] and out["top2_ties"] and out["checkpoint_ownership"]
    assert out["attention_max_error"] < 2e-5 and out["rope_max_error"] < 2e-5
