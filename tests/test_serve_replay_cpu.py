"""Protocol replay against the reference's own serving loops (CPU).

oracle/_ref/ref-serve-cpu is the reference's src/qwen_serve.c and
src/qwen_bounded_serve.c, unchanged, over its src/qwen.c and the CPU
primitives of tests/gpu_stub.c (seeded models through wrapped loader calls,
oracle/ref_serve.c). oracle/_ref/tcm-cuda-cpu is this repository's serve
(cmachine_b200/host/serve.c and the session host) over the same CPU
primitives. A scripted session -- appends, generation, state hashes, legacy
checkpoint/restore, nested push/rollback/commit, stack overflow, reset and
malformed commands -- must produce the same replies from both, field for field,
including the SHA-256 state hashes of the K/V cache (or byte-codec arena, ring
positions and RNG) and the logits. Excluded: the memory-accounting fields
(gpu_weight_bytes, gpu_session_bytes, gpu_state_bytes, tracked_gpu_bytes: this
repository's token cut keeps rows, not a whole arena) and the bounded serve's
free-text weight_storage.
"""
import json
import subprocess

import pytest

from checkers import ROOT

OURS = ROOT / "oracle" / "_ref" / "tcm-cuda-cpu"
REF = ROOT / "oracle" / "_ref" / "ref-serve-cpu"
pytestmark = pytest.mark.skipif(not (OURS.exists() and REF.exists()), reason="reference sources not built here")
ACCOUNTING = {"gpu_weight_bytes", "gpu_session_bytes", "gpu_state_bytes", "tracked_gpu_bytes", "weight_storage"}


def replies(exe, model, script, *args):
    proc = subprocess.run([str(exe), "serve", model, *args], input="\n".join(script) + "\n", text=True,
                          capture_output=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines()]


def compare(model, script, *args):
    ours, ref = replies(OURS, model, script, *args), replies(REF, model, script, *args)
    assert len(ours) == len(ref) == len(script) - (1 if script[-1] == "Q" else 0) + 1
    for i, (a, b) in enumerate(zip(ours, ref)):
        assert set(a) == set(b), (i, a, b)
        for key in a:
            if key not in ACCOUNTING:
                assert a[key] == b[key], (i, key, a[key], b[key])
    return ours


def test_dense_session_replays_like_the_reference():
    script = ["A 1 2 3", "G 4", "S", "P", "A 5 6", "S", "B 1", "S", "C", "A 7", "R", "S", "K 9", "P", "P", "A 4",
              "K 3", "B 2", "S", "Z", "S", "A", "A 99", "G 0", "X", "A 1", "G 5", "S", "Q"]
    out = compare("seeded:8x3x4x2x2x12x16x32:5:0", script, "--context", "32")
    states = [r for r in out if r.get("event") == "state"]
    assert len(states) == 7 and states[1]["cache_sha256"] != states[0]["cache_sha256"]
    assert any(r.get("error") for r in out)


def test_bounded_session_replays_like_the_reference():
    """The reference ring needs 28 layers and 12/2 heads of 128 (src/bounded_cache.h:67);
    a narrow MLP and vocabulary keep the CPU run short. Retention (2, 4, 3) evicts
    and samples the reservoir from the seventh token on."""
    script = ["A 1 2 3 4 5 6 7 8 9 10 11 12", "G 6", "S", "P", "A 5 6 7", "S", "B 1", "S", "C", "P", "A 3", "K 2",
              "S", "P", "P", "P", "Z", "S", "A 9 9", "G 12", "S", "Q"]
    out = compare("seeded:1536x28x12x2x128x64x256x96:7:0", script, "--cache-policy", "bounded", "--context", "64",
                  "--anchors", "2", "--recent", "4", "--reservoir", "3")
    states = [r for r in out if r.get("event") == "state"]
    assert states[0]["evictions"] == 11 and states[0]["resident_rows"] == 9
    assert states[2]["cache_sha256"] == states[0]["cache_sha256"]  # the rollback restored the arena
