"""The serving front-end (cmachine_b200/host/serve.c, the reference's line
protocol of src/qwen_serve.c) on the CPU host build (oracle/_ref/tcm-cuda-cpu):
a scripted session on a small seeded model checks every command's reply, the
state hashes across push/rollback and checkpoint/restore, and the error replies
for malformed input."""
import json
import subprocess

import pytest

from checkers import ROOT

SERVE = ROOT / "oracle" / "_ref" / "tcm-cuda-cpu"
pytestmark = pytest.mark.skipif(not SERVE.exists(), reason="reference sources not built here")
TINY = "seeded:8x3x4x2x2x12x16x32:5:0"


def run(commands, *args, model=TINY):
    proc = subprocess.run([str(SERVE), "serve", model, *args], input="\n".join(commands) + "\n", text=True,
                          capture_output=True, timeout=60)
    return proc.returncode, [json.loads(line) for line in proc.stdout.splitlines()], proc.stderr


def test_protocol_session():
    rc, out, err = run(["A 1 2 3", "G 4", "S", "P", "A 5 6", "S", "B 1", "S", "C", "A 7", "R", "S", "Z", "S", "Q"],
                       "--context", "32")
    assert rc == 0, err
    ready, appended, generated, s0, pushed, app2, s1, rolled, s2, ck, app3, restored, s3, reset, s4 = out
    assert ready["event"] == "ready" and ready["capacity"] == 32
    assert appended == {"event": "appended", "count": 3, "position": 3}
    assert generated["event"] == "generated" and generated["count"] == 4 == len(generated["ids"])
    assert generated["position"] == 6 and generated["pending_token"] == generated["ids"][-1]
    assert s0["position"] == 6 and s0["logits_valid"] is True and s0["delivered"] == 1
    assert pushed["event"] == "pushed" and pushed["depth"] == 1 and pushed["position"] == 6
    assert app2["position"] == 8 and s1["stack_depth"] == 1 and s1["cache_sha256"] != s0["cache_sha256"]
    assert rolled["event"] == "rolled_back" and rolled["frame"] == pushed["frame"] and rolled["position"] == 6
    assert s2["cache_sha256"] == s0["cache_sha256"] and s2["stack_depth"] == 0
    assert ck["event"] == "checkpoint" and app3["position"] == 7
    assert restored == {"event": "restored", "position": 6, "pending_token": s0["pending_token"]}
    assert s3["cache_sha256"] == s0["cache_sha256"]
    assert reset == {"event": "reset"}
    assert s4["position"] == 0 and s4["pending_token"] == -1 and s4["epoch"] == s0["epoch"] + 1
    # an empty cache hashes to SHA-256 of no bytes
    assert s4["cache_sha256"] == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"


def test_protocol_errors():
    rc, out, _ = run(["A", "A 16", "A -1", "A 1 x", "G 1", "R", "B 1", "K 1", "B x", "X", "A " + " ".join(["1"] * 33),
                      "A 1", "G 0", "G 5000", "G 33", "C", "Q"], "--context", "32")
    assert rc == 0
    replies = out[1:]
    assert replies[:4] == [{"error": "invalid append or context capacity"}] * 4
    assert replies[4] == {"error": "invalid generation budget or state"}  # nothing appended yet
    assert replies[5] == {"error": "no compatible saved parent"}
    assert replies[6:9] == [{"error": "no compatible top frame"}] * 3
    assert replies[9] == {"error": "unknown command"}
    assert replies[10] == {"error": "invalid append or context capacity"}  # more than the capacity
    assert replies[11]["event"] == "appended"
    assert replies[12:15] == [{"error": "invalid generation budget or state"}] * 3
    assert replies[15]["event"] == "checkpoint"


def test_usage_and_model_errors():
    assert run(["Q"], "--context")[0] == 2
    assert run(["Q"], "--context", "0")[0] == 2
    assert run(["Q"], "--bogus", "1")[0] == 2
    rc, _, err = run(["Q"], model="seeded:nonsense:1:0")
    assert rc == 2 and "invalid seeded model specification" in err
    rc, _, err = run(["Q"], model=str(ROOT / "no-such-bundle.tcm"))
    assert rc == 2 and "cannot open model bundle" in err
