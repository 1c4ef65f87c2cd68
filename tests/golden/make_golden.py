"""Regenerates the golden vectors from the reference's own CPU path.

Runs oracle/_ref/libref_cpu.so -- the reference's src/qwen.c + src/model.c +
tests/gpu_stub.c compiled from its sources by oracle/Makefile -- on seeded
weights and token ids and records, per pushed token, the top-2 (ids and
values), the SHA-256 of all vocabulary logits and the logits at fixed probe
ids. Needs the reference sources (this container only):

    make -C oracle ref && python tests/golden/make_golden.py
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE.parent))

import cmachine_b200 as cm  # noqa: E402
from checkers import REF_CPU, CpuDecoder  # noqa: E402

PROBES = [0, 1, 17, 4096, 65535, 100000, 151935]

CASES = {
    # The reference's CPU-runnable configuration: 2-layer Qwen2.5-1.5B geometry,
    # FP32 weights N(0, 0.02), biases 0, norms 1; 64-token prompt + 32 greedy steps.
    "qwen2layer_fp32_p64_g32": dict(layers=2, bf16=False, law="bench", seed=2026, prompt=64, greedy=32),
    # Same geometry, BF16-rounded matrices, parity law (nonzero biases, non-unit norms).
    "qwen2layer_bf16_p16_g8": dict(layers=2, bf16=True, law="test", seed=2027, prompt=16, greedy=8),
}


def law_of(name):
    return cm.BENCH_LAW if name == "bench" else cm.TEST_LAW


def run(case):
    shape = cm.qwen_shape(case["layers"], 4096)
    dec = CpuDecoder(REF_CPU, shape, case["seed"], law_of(case["law"]), case["bf16"], case["prompt"] + case["greedy"])
    prompt = [int(t) for t in np.random.default_rng(case["seed"] + 1).integers(0, shape.vocab, case["prompt"])]
    steps = []
    token = None
    for i in range(case["prompt"] + case["greedy"]):
        token = prompt[i] if i < case["prompt"] else top[0]
        top, logits = dec.push(token)
        steps.append({"token": token, "top": [top[0], top[1]], "values": [top[2], top[3]],
                      "logits_sha256": hashlib.sha256(logits.tobytes()).hexdigest(),
                      "probes": [float(logits[p]) for p in PROBES]})
    dec.close()
    return {"case": case, "probes": PROBES, "steps": steps,
            "source": "reference CPU path (src/qwen.c + tests/gpu_stub.c), built by oracle/Makefile"}


if __name__ == "__main__":
    for name, case in CASES.items():
        (HERE / f"{name}.json").write_text(json.dumps(run(case), indent=0) + "\n")
        print("wrote", name)
