"""The serving executable (cmachine_b200/tcm-cuda, the reference's line
protocol) on the GPU, and TCM1LE bundles end to end:

1. a dense session on a seeded BF16 model: prefill through A, generation,
   push/rollback and checkpoint/restore restore the state hashes;
2. a bounded (byte-codec ring) session: marks roll back to identical hashes;
3. a 28-layer BF16 bundle written from a seeded model's device weights serves
   exactly as the seeded model itself: same cache and logits hashes after the
   same commands (qwen_model_init + the source-BF16 weight profile).
"""
import ctypes
import hashlib
import json
import struct
import subprocess

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ROOT

pytestmark = pytest.mark.gpu
SERVE = ROOT / "cmachine_b200" / "tcm-cuda"


def run(model, commands, *args):
    proc = subprocess.run([str(SERVE), "serve", model, *args], input="\n".join(commands) + "\n", text=True,
                          capture_output=True, timeout=600)
    assert proc.returncode == 0, proc.stderr
    return [json.loads(line) for line in proc.stdout.splitlines()]


def prompt(n, seed=3):
    return " ".join(str(int(t)) for t in np.random.default_rng(seed).integers(0, 151936, n))


def test_dense_session_protocol():
    out = run("seeded:qwen2.5-1.5b@2:7:2", ["A " + prompt(100), "G 8", "S", "P", "A " + prompt(5, 4), "S", "B 1", "S",
                                           "C", "G 3", "R", "S", "Q"], "--context", "256")
    ready, app, gen, s0, pushed, app2, s1, rolled, s2, ck, gen2, restored, s3 = out
    assert ready["event"] == "ready" and app == {"event": "appended", "count": 100, "position": 100}
    assert gen["count"] == 8 and gen["position"] == 107
    assert s0["position"] == 107 and s0["logits_valid"] is True
    assert app2["position"] == 112 and s1["cache_sha256"] != s0["cache_sha256"]
    assert rolled["event"] == "rolled_back" and s2["cache_sha256"] == s0["cache_sha256"]
    assert ck["event"] == "checkpoint" and gen2["count"] == 3
    assert restored["position"] == 107 and s3["cache_sha256"] == s0["cache_sha256"]


def test_bounded_session_protocol():
    out = run("seeded:qwen2.5-1.5b:7:2", ["A " + prompt(60), "G 4", "S", "P", "A " + prompt(20, 5), "S", "B 1", "S",
                                         "Q"], "--cache-policy", "bounded", "--context", "256", "--anchors", "8",
              "--recent", "32", "--reservoir", "16")
    ready, app, gen, s0, pushed, app2, s1, rolled, s2 = out
    assert ready["cache_policy"] == "bounded" and ready["resident_capacity"] == 56
    assert app["position"] == 60 and gen["count"] == 4
    assert s0["resident_rows"] == 56 and s0["evictions"] > 0
    assert s1["cache_sha256"] != s0["cache_sha256"]
    assert rolled["event"] == "rolled_back" and s2["cache_sha256"] == s0["cache_sha256"]
    assert s2["logits_sha256"] == s0["logits_sha256"]


def write_model_bundle(path, model):
    """A TCM1LE bundle (the reference's tensor names, BF16 matrices, FP32
    vectors) holding a seeded model's device weights."""
    L, s = model.L, model.shape
    d, kv, f = s.hidden, s.kvheads * s.head, s.intermediate
    specs = [("model.embed_tokens.weight", -1, 0, (s.vocab, d)), ("model.norm.weight", -1, 1, (d,))]
    suffix = ["input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
              "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.bias",
              "self_attn.v_proj.bias", "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
              "mlp.down_proj.weight"]
    shapes = [(d,), (d,), (d, d), (kv, d), (kv, d), (d,), (kv,), (kv,), (d, d), (f, d), (f, d), (d, f)]
    for layer in range(s.layers):
        for kind in range(12):
            specs.append((f"model.layers.{layer}.{suffix[kind]}", layer, kind, shapes[kind]))
    specs.sort(key=lambda x: x[0])
    offset = 176 + 120 * len(specs)
    records, layout = [], []
    for name, layer, kind, shape in specs:
        dtype = 2 if len(shape) == 2 else 1
        nbytes = int(np.prod(shape)) * (2 if dtype == 2 else 4)
        offset += (-offset) % 8
        records.append(struct.pack("<64sII4QQQ", name.encode(), len(shape), dtype, *(list(shape) + [0] * (4 - len(shape))),
                                   offset, nbytes))
        layout.append((offset, layer, kind, nbytes))
        offset += nbytes
    config = [1536, 28, 12, 2, 128, 8960, 151936, struct.unpack("<I", struct.pack("<f", 1e-6))[0],
              struct.unpack("<I", struct.pack("<f", 1e6))[0], 151935, 32768, 1, 0]
    head = struct.pack("<II16I64s", 2, len(specs), *(config + [0] * 3), hashlib.sha256(b"seeded").hexdigest().encode())
    digest = hashlib.sha256()
    with open(path, "wb") as out:
        out.write(b"TCM1LE\0\0" + bytes(32))
        for block in (head, b"".join(records)):
            out.write(block)
            digest.update(block)
        pos = 176 + 120 * len(specs)
        for off, layer, kind, nbytes in layout:
            pad = bytes(off - pos)
            host = np.empty(nbytes, np.uint8)
            L.gpu_read(cm.ptr(host), ctypes.c_void_p(L.qwen_b200_model_weight(model.handle, layer, kind)), nbytes)
            for block in (pad, host.tobytes()):
                out.write(block)
                digest.update(block)
            pos = off + nbytes
        out.seek(8)
        out.write(digest.digest())


def test_bundle_serves_as_the_seeded_model(tmp_path):
    seed = 11
    model = cm.Model(cm.qwen_shape(28, 32768), seed, cm.BENCH_LAW, 2)
    assert model.L.qwen_b200_model_matrix_dtype(model.handle) == 2
    path = tmp_path / "qwen.tcm"
    write_model_bundle(path, model)
    model.free()
    script = ["A " + prompt(40), "S", "G 3", "S", "P", "A 5 6 7", "B 1", "S", "Q"]
    args = ["--cache-policy", "bounded", "--context", "128", "--anchors", "4", "--recent", "16", "--reservoir", "8"]
    from_bundle = run(str(path), script, *args)
    seeded = run(f"seeded:qwen2.5-1.5b:{seed}:2", script, *args)
    assert from_bundle[0]["model_digest"] == hashlib.sha256(path.read_bytes()[40:]).hexdigest()
    assert from_bundle[0]["weight_profile"] == 2 and from_bundle[0]["gpu_weight_bytes"] == seeded[0]["gpu_weight_bytes"]
    for a, b in zip(from_bundle[1:], seeded[1:]):
        if a.get("event") == "state":
            assert a["cache_sha256"] == b["cache_sha256"] and a["logits_sha256"] == b["logits_sha256"]
        else:
            assert a == b


REF_SERVE = ROOT / "oracle" / "_ref" / "ref-serve-cpu"
# Reply fields that hold floating-point state or memory accounting: the B200
# path computes within FP32 tolerance of the reference's CPU path, not to its bits.
NUMERIC = {"cache_sha256", "logits_sha256", "gpu_weight_bytes", "gpu_session_bytes", "gpu_state_bytes",
           "tracked_gpu_bytes", "weight_storage"}


def ref_run(model, commands, *args):
    proc = subprocess.run([str(REF_SERVE), "serve", model, *args], input="\n".join(commands) + "\n", text=True,
                          capture_output=True, timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines()]


def replay_matches(model, commands, *args):
    ours, ref = run(model, commands, *args), ref_run(model, commands, *args)
    assert len(ours) == len(ref)
    for i, (a, b) in enumerate(zip(ours, ref)):
        assert set(a) == set(b), (i, a, b)
        for key in a:
            if key not in NUMERIC:
                assert a[key] == b[key], (i, key, a[key], b[key])
    return ours, ref


@pytest.mark.skipif(not REF_SERVE.exists(), reason="reference serve build absent")
def test_dense_protocol_replay_against_reference_serve():
    """The same scripted session through the B200 tcm-cuda and the reference's
    own serve loop (src/qwen_serve.c over its CPU FP32 path): every reply field
    but the float hashes and byte counts, generated ids included. 2-layer FP32
    seeded model (full Qwen2.5-1.5B widths)."""
    script = ["A " + prompt(12, 5), "G 6", "S", "P", "A " + prompt(3, 6), "S", "B 1", "S", "C", "A 7", "R", "S",
              "P", "P", "A 4", "K 3", "B 2", "Z", "S", "A 11 12", "G 4", "S", "Q"]
    ours, _ = replay_matches("seeded:qwen2.5-1.5b@2:21:0", script, "--context", "64")
    assert sum(len(r.get("ids", [])) for r in ours) == 10


@pytest.mark.skipif(not REF_SERVE.exists(), reason="reference serve build absent")
def test_bounded_protocol_replay_against_reference_serve():
    """A bounded byte-codec session (retention 2/4/3, evicting and sampling the
    reservoir) through the B200 tcm-cuda and the reference's bounded serve
    (src/qwen_bounded_serve.c + src/bounded_cache.h over its CPU path): cursor,
    evictions, RNG state, resident rows, frames and generated ids must agree.
    28-layer FP32 seeded model, as the reference ring requires."""
    script = ["A " + prompt(9, 8), "G 3", "S", "P", "A 5 6", "S", "B 1", "S", "Q"]
    replay_matches("seeded:qwen2.5-1.5b:22:0", script, "--cache-policy", "bounded", "--context", "64", "--anchors",
                   "2", "--recent", "4", "--reservoir", "3")


CPU_HOST_EXE = ROOT / "oracle" / "_ref" / "tcm-cuda-cpu"


def qwen_run(exe, model, prompt_tokens, tmp_path, tag, *extra):
    tokens = tmp_path / f"{tag}.txt"
    tokens.write_text(" ".join(map(str, prompt_tokens)) + "\n")
    proc = subprocess.run([str(exe), "qwen", model, "--tokens-file", str(tokens), "--output", str(tmp_path / f"{tag}.json"),
                           "--first-logits", str(tmp_path / f"{tag}.f32"), *extra], capture_output=True, text=True,
                          timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return json.loads((tmp_path / f"{tag}.json").read_text()), np.fromfile(tmp_path / f"{tag}.f32", np.float32)


@pytest.mark.parametrize("profile,n_prompt,tol", [(0, 6, 1e-3), (2, 100, 3e-2)], ids=["fp32", "bf16-prefill"])
def test_qwen_run_against_oracle(tmp_path, profile, n_prompt, tol):
    """`tcm-cuda qwen` on the B200 (2-layer seeded model of Qwen2.5-1.5B widths):
    the first-logits dump and every generated token against the oracle, and the
    checkpoint test's exact replay. The BF16 prompt runs through the batched
    prefill."""
    from checkers import ORACLE, CpuDecoder
    prompt_ids = [int(t) for t in np.random.default_rng(31).integers(0, 151936, n_prompt)]
    run, first = qwen_run(SERVE, f"seeded:qwen2.5-1.5b@2:23:{profile}", prompt_ids, tmp_path, "gpu", "--new-tokens",
                          "5", "--context", "128", "--checkpoint-test")
    assert run["checkpoint_exact"] is True and run["generated_tokens"] == 5
    law = cm.FillLaw(cm.Fill(0.0, 0.02), cm.Fill(1.0, 0.0), cm.Fill(0.0, 0.0))
    o = CpuDecoder(ORACLE, cm.qwen_shape(2, 32768), 23, law, profile == 2, 128)
    try:
        for i, t in enumerate(prompt_ids):
            top, logits = o.push(t, readout=i == len(prompt_ids) - 1)
        assert float(np.max(np.abs(first - logits))) <= tol
        for step in run["tokens"]:
            if top[2] - top[3] > 2 * tol:
                assert step["id"] == top[0]
            assert abs(step["logit"] - top[2]) <= tol
            top, _ = o.push(step["id"])
    finally:
        o.close()


@pytest.mark.skipif(not CPU_HOST_EXE.exists(), reason="CPU host build absent")
def test_qwen_run_port_trace_against_cpu_host(tmp_path):
    """--trace-prefix/--trace-layer/--trace-position on the B200: the same 14
    ports, in the same order and sizes, as the session host over the
    reference's CPU primitives, and values within the FP32 bound."""
    prompt_ids = [5, 77, 1234, 99, 42, 7]
    args = ["--new-tokens", "3", "--context", "64", "--trace-layer", "1", "--trace-position", "4"]
    gpu, _ = qwen_run(SERVE, "seeded:qwen2.5-1.5b@2:24:0", prompt_ids, tmp_path, "gpu", "--trace-prefix",
                      str(tmp_path / "g"), *args)
    cpu, _ = qwen_run(CPU_HOST_EXE, "seeded:qwen2.5-1.5b@2:24:0", prompt_ids, tmp_path, "cpu", "--trace-prefix",
                      str(tmp_path / "c"), *args)
    assert gpu["trace_ports"] == cpu["trace_ports"] == 14
    lg = [json.loads(l) for l in (tmp_path / "g.jsonl").read_text().splitlines()]
    lc = [json.loads(l) for l in (tmp_path / "c.jsonl").read_text().splitlines()]
    assert lg == lc
    for e in lg:
        name = f"-{e['occurrence']:04d}-{e['port']}.f32"
        a, b = np.fromfile(str(tmp_path / "g") + name, np.float32), np.fromfile(str(tmp_path / "c") + name, np.float32)
        assert a.size == b.size == e["count"]
        assert float(np.max(np.abs(a - b))) <= 1e-3 * max(1.0, float(np.max(np.abs(b))))
    assert [t["id"] for t in gpu["tokens"]] == [t["id"] for t in cpu["tokens"]]
