"""The timed single-session run (`tcm-cuda qwen`, the reference's qwen_main,
src/qwen.c:438-503) on the CPU host build (oracle/_ref/tcm-cuda-cpu: this
repository's session host over the reference's CPU primitives).

Checked against the oracle on the same seeded model and prompt: the greedy
token ids and their logits, margins and runner-ups in the tcm-qwen-run-v1 JSON,
the --first-logits dump (bit for bit: both are the reference's CPU arithmetic),
the --checkpoint-test exact replay, and the --trace-* port dumps: 14 ports in
the reference's order, each a raw FP32 file named by occurrence and port, with
a JSONL ledger line each. Also the usage errors.
"""
import json
import subprocess

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ORACLE, ROOT, CpuDecoder

EXE = ROOT / "oracle" / "_ref" / "tcm-cuda-cpu"
pytestmark = pytest.mark.skipif(not EXE.exists(), reason="CPU host build absent")
MODEL = "seeded:8x3x4x2x2x12x16x32:5:0"
PORTS = ["input", "query", "key", "value", "attention", "attention_write", "consumed_attention_write", "raw_receiver",
         "mlp_input", "mlp_gate", "mlp_up", "consumed_mlp_write", "mlp_return", "output"]


def test_qwen_run_matches_oracle(tmp_path):
    prompt = [1, 2, 3, 4, 5]
    (tmp_path / "t.txt").write_text(" ".join(map(str, prompt)) + "\n")
    proc = subprocess.run([str(EXE), "qwen", MODEL, "--tokens-file", str(tmp_path / "t.txt"), "--new-tokens", "6",
                           "--context", "32", "--checkpoint-test", "--first-logits", str(tmp_path / "first.f32"),
                           "--trace-prefix", str(tmp_path / "tr"), "--trace-layer", "1", "--trace-position", "3",
                           "--output", str(tmp_path / "run.json")], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr
    run = json.loads((tmp_path / "run.json").read_text())
    assert run["schema"] == "tcm-qwen-run-v1" and run["prompt_tokens"] == 5 and run["generated_tokens"] == 6
    assert run["checkpoint_tested"] is True and run["checkpoint_exact"] is True and run["trace_ports"] == 14
    shape = cm.Shape(8, 3, 4, 2, 2, 12, 16, 32, 1e-6, 1e6)
    law = cm.FillLaw(cm.Fill(0.0, 0.02), cm.Fill(1.0, 0.0), cm.Fill(0.0, 0.0))
    o = CpuDecoder(ORACLE, shape, 5, law, False, 32)
    try:
        for t in prompt:
            top, logits = o.push(t)
        assert np.array_equal(np.fromfile(tmp_path / "first.f32", np.float32).view(np.uint32), logits.view(np.uint32))
        for step in run["tokens"]:
            assert step["id"] == top[0] and step["runner_up"] == top[1]
            assert step["logit"] == pytest.approx(top[2], rel=1e-6)
            assert step["margin"] == pytest.approx(top[2] - top[3], rel=1e-5, abs=1e-7)
            top, _ = o.push(step["id"])
    finally:
        o.close()
    ledger = [json.loads(line) for line in (tmp_path / "tr.jsonl").read_text().splitlines()]
    assert [e["port"] for e in ledger] == PORTS and [e["occurrence"] for e in ledger] == list(range(14))
    assert all(e["position"] == 3 and e["layer"] == 1 for e in ledger)
    for e in ledger:
        dump = tmp_path / f"tr-{e['occurrence']:04d}-{e['port']}.f32"
        assert np.fromfile(dump, np.float32).size == e["count"]


def test_qwen_run_usage_errors(tmp_path):
    (tmp_path / "t.txt").write_text("1 2 3\n")
    base = [str(EXE), "qwen", MODEL, "--tokens-file", str(tmp_path / "t.txt")]
    for extra in (["--new-tokens", "0"], ["--context", "40000"], ["--bogus", "1"], ["--trace-layer", "1"],
                  ["--new-tokens"]):
        assert subprocess.run(base + extra, capture_output=True, timeout=60).returncode == 2
    assert subprocess.run([str(EXE), "qwen", MODEL], capture_output=True, timeout=60).returncode == 2
