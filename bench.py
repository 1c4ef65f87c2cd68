"""Decode benchmark of the B200 Qwen2.5 path.

A step is one batch-1 greedy decode token of full-depth Qwen2.5-1.5B (28
layers, FP32 seeded weights by default) inside a 512-token-prompt, 256-token
decode window: the prompt is prefilled once (untimed), then steps cycle over
positions 512..767 (each 256-step segment restarts from the post-prompt state).

  value : device-timed tokens/s -- chained whole-token CUDA-graph replays, the
          device feeding each top-1 back as the next token, CUDA events on the
          library stream, max over ranks, summed over ranks (weak scaling:
          one independent session per GPU, no collective on the data path).
  e2e   : the same steps through the public C API (qwen_advance): per step one
          pinned host->device copy of the token state, one graph replay and one
          device->host read of the top-2, host synchronised every step.

The default run adds, in the same JSON line, the other configurations the
metric names, each a sub-object with its own value, e2e, roofline and clocks:
  bs64          64 independent sessions per GPU (contexts 128..8192, each a
                uniform-random prompt run through qwen_prefill, untimed), batched
                tcgen05 decode; at N > 1 weak scaling (64 sessions per GPU);
  bs64_strong   N > 1 only: 64 sessions in all, dealt over the N GPUs;
  bf16_ctx4096  BF16 weights, 4096-token prompt, 512-token decode window;
  bf16_ctx4096_tp  N > 1 only: the same single session split over the N GPUs
                (tensor-parallel MLP and readout; value = that session's tokens/s);
  bounded       two bounded byte-codec sessions per GPU (below).
--no-extras skips them; --config runs one configuration alone.

With --config bf16-bounded a step is one token of each of the GPU's bounded
sessions through ring_push (include/bounded_cache.h), which reads the top-2 back
every token by design (abort and recovery are decided per token on the host):
value is CUDA-event time over those steps, e2e the host clock over a second pass.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
       [--config fp32-ctx512 | bf16-ctx4096 | fp32-2layer | bf16-bounded | bf16-batch64] [--no-extras]
Under torchrun (N > 1) every rank runs its own replica; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
from ctypes import c_void_p
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Qwen2.5-1.5B decode tok/s/GPU (bs1, bs64) + % HBM roofline; max |Δlogit|"

CONFIGS = {
    # Full Qwen2.5-1.5B, native FP32 weights, 512-token prompt, 256 greedy steps.
    "fp32-ctx512": dict(layers=28, profile=0, prompt=512, window=256),
    # Full Qwen2.5-1.5B, source-BF16 weights, 4096-token prompt, 512 greedy steps.
    "bf16-ctx4096": dict(layers=28, profile=2, prompt=4096, window=512),
    # The reduced 2-layer model of the reference's CPU-runnable case (64 + 32).
    "fp32-2layer": dict(layers=2, profile=0, prompt=64, window=32),
    # Bounded compressed memory: full Qwen2.5-1.5B, source-BF16 weights, all-layer
    # K/V in the byte codec with 64 anchor, 1024 recent and 1024 reservoir rows,
    # logical context 32768; two sessions per GPU (16 over 8 GPUs), each prefilled
    # past the first 1,024 evictions, then streaming with a mark every 256 tokens
    # (nested to depth 2, the reference ring's limit), a commit 128 tokens later,
    # and one injected layer failure with recovery per 1,024 tokens.
    "bf16-bounded": dict(layers=28, profile=2, ring=(64, 1024, 1024), logical=32768, prefill=2200,
                         sessions=2, mark_every=256, fail_every=1024),
    # Batched decode: full Qwen2.5-1.5B, source-BF16 weights, 64 independent
    # sessions per GPU with contexts drawn uniformly from 128..8192, greedy steps
    # in segments of 64 with a checkpoint at each segment start and a rollback
    # after every second segment; projections on the tcgen05 tensor cores.
    "bf16-batch64": dict(layers=28, profile=2, batch=64, ctx=(128, 8192), segment=64),
}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (read-only queries) for the whole run, each stamped by
    nvidia-smi's own clock; summary(t0, t1) reports the samples that fall in a
    window of the host clock (widened by `pad` seconds on both sides)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.reader = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.reader:
                self.reader.join(timeout=5)
            self.proc = None

    @staticmethod
    def _stamp(text):
        from datetime import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.strptime(text.strip(), fmt).timestamp()
            except ValueError:
                continue
        return None

    def summary(self, t0=None, t1=None, pad=0.25):
        sm, mx, reasons, n_all = [], None, set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in list(self.lines):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            when = self._stamp(parts[0])
            if t0 is not None and (when is None or when < t0 - pad or when > t1 + pad):
                continue
            try:
                sm.append(float(parts[2]))
                mx = float(parts[3])
            except ValueError:
                continue
            for name, flag in zip(names, parts[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window_s": None if t0 is None else round(t1 - t0 + 2 * pad, 3)}


CLOCKS = None  # the run's sampler (started in main before any GPU work)


def clocks_between(t0, t1):
    return CLOCKS.summary(t0, t1) if CLOCKS else {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        return world, rank, local, dist, torch
    return 1, 0, local, None, None


def barrier(dist, torch):
    """All ranks meet; with NCCL the device is drained on both sides."""
    if dist:
        dist.barrier()
        if dist.get_backend() == "nccl":
            torch.cuda.synchronize()


def max_over_ranks(value: float, dist, torch) -> float:
    """The largest value over all ranks (device time of the slowest rank)."""
    if not dist:
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompt_tokens(seed: int, n: int, vocab: int):
    import numpy as np
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


# ---------------------------------------------------------------- CPU baseline (reference path)
def ref_context(cfg) -> int:
    """Cached rows the CPU reference starts from for a configuration: the prompt
    length of a batch-1 workload, the mean context of the batched one."""
    if "prompt" in cfg:
        return cfg["prompt"]
    if "ctx" in cfg:
        return (cfg["ctx"][0] + cfg["ctx"][1]) // 2
    return 0


def context_kv(layers: int, context: int):
    """Seeded K/V rows standing for a `context`-token prompt, shared by the CPU
    sample's sessions and its GPU replay: kv[layer][kind] = [kvheads][context][128]."""
    import numpy as np
    rng = np.random.default_rng(5150 + context)
    return [[(0.5 * rng.standard_normal((2, context, 128))).astype(np.float32) for _ in (0, 1)]
            for _ in range(layers)]


def cpu_reference_rate(layers: int, bf16: bool, seconds: float = 15.0, threads: int | None = None, context: int = 0):
    """The reference's own CPU FP32 C path (src/qwen.c + tests/gpu_stub.c, built
    from its sources into oracle/_ref), one session per host thread. With
    `context`, every session starts after `context` cached rows (seeded K/V rows
    written into the reference session, cursor placed after them), so each
    token's attention reads the workload's cache length; then one prompt token
    and greedy steps. Returns (tokens/s, threads, sample, kind, the first
    thread's logits per greedy step)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import ctypes
    import numpy as np
    import cmachine_b200 as cm
    L, model, kind = reference_model(layers, 2 if bf16 else 0, 2026)
    shape = cm.qwen_shape(layers, 32768)
    n = threads or max(1, min(os.cpu_count() or 1, 32))
    per_token = (1.3 * layers / 28 + 0.05) * (1.0 + context / 16000.0)
    steps = max(2, int(seconds / max(per_token, 1e-3)) // 1)
    steps = min(steps, 12 if layers > 2 else 64)
    results, first_logits = [0] * n, []
    kv = context_kv(layers, context) if context else None

    def worker(i):
        s = L.orc_session_create(model, context + 64)
        if kv:
            for layer in range(layers):
                for kind in (0, 1):
                    L.orc_write_kv(s, layer, kind, context, ctypes.c_void_p(kv[layer][kind].ctypes.data))
            assert L.orc_set_cursor(s, context) == 0
        top = cm.Top2()
        toks = prompt_tokens(90 + i, 1 if kv else 2, shape.vocab)
        out = np.empty(shape.vocab, np.float32)
        for t in toks:
            L.orc_push(s, t, ctypes.byref(top), ctypes.c_void_p(out.ctypes.data))
        done = len(toks)
        for _ in range(steps):
            L.orc_push(s, top.first, ctypes.byref(top), ctypes.c_void_p(out.ctypes.data))
            if i == 0:
                first_logits.append(out.copy())
            done += 1
        results[i] = done
        L.orc_session_free(s)

    t0 = time.perf_counter()
    pool = [threading.Thread(target=worker, args=(i,)) for i in range(n)]
    for th in pool:
        th.start()
    for th in pool:
        th.join()
    wall = time.perf_counter() - t0
    total = sum(results)
    start = f"{context} cached rows (seeded K/V) + 1 prompt token" if context else "2-token prompt"
    sample = (f"{n} threads x ({start} + {steps} greedy decode steps, every push counted), {layers}-layer "
              f"{'BF16' if bf16 else 'FP32'} seeded model, one session per thread")
    return total / wall, n, sample, kind, first_logits


def cpu_reference_ring_rate(cfg, threads: int | None = None):
    """The reference's own bounded cache (src/bounded_cache.h over src/qwen.c and
    tests/gpu_stub.c, oracle/_ref/libref_ring.so) on the host cores, one ring
    session per thread with the benchmark's retention, each pushing a 2-token
    prompt and greedy steps from position 0 (the retained set is still small
    there; at 2,112 retained rows ring attention adds about 1% to a token's
    arithmetic). Returns (tokens/s, threads, sample, kind) or None."""
    sys.path.insert(0, str(ROOT / "tests"))
    import ctypes
    ref = ROOT / "oracle" / "_ref" / "libref_ring.so"
    if not ref.exists():
        return None
    import cmachine_b200 as cm
    from checkers import load
    L = load(ref)
    L.rr_open.restype = ctypes.c_void_p
    L.rr_open.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.rr_push.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.rr_close.argtypes = [ctypes.c_void_p]
    shape = cm.qwen_shape(cfg["layers"], 4096)
    model = L.orc_model_create(ctypes.byref(shape), 2026, ctypes.byref(cm.BENCH_LAW), int(cfg["profile"] == 2))
    n = threads or max(1, min(os.cpu_count() or 1, 16))
    steps, results = 6, [0] * n
    a, r, m = cfg["ring"]

    def worker(i):
        h = L.rr_open(model, 4096, a, r, m, 0)
        for t in prompt_tokens(90 + i, 2 + steps, shape.vocab):
            assert L.rr_push(h, t) == 0
            results[i] += 1
        L.rr_close(h)

    t0 = time.perf_counter()
    pool = [threading.Thread(target=worker, args=(i,)) for i in range(n)]
    for th in pool:
        th.start()
    for th in pool:
        th.join()
    wall = time.perf_counter() - t0
    L.orc_model_free(model)
    sample = (f"{n} threads x 8 ring_push tokens from position 0, 28-layer BF16 seeded model, retention "
              f"({a}, {r}, {m}), one bounded session per thread")
    return sum(results) / wall, n, sample, "reference"


def run_bounded(args, cfg, world, rank, local, dist, torch):
    """Bounded byte-codec sessions (ring_push), two per GPU."""
    import cmachine_b200 as cm
    L = cm.lib()
    L.qwen_b200_set_device(local)
    shape = cm.qwen_shape(cfg["layers"], cfg["logical"])
    model = cm.Model(shape, 2026 + rank, cm.BENCH_LAW, cfg["profile"])
    a, r, m = cfg["ring"]
    rings = [cm.Ring(model, cfg["logical"], a, r, m) for _ in range(cfg["sessions"])]
    assert all(g.view().fused for g in rings)
    for i, g in enumerate(rings):
        for t in prompt_tokens(7 + 16 * rank + i, cfg["prefill"], shape.vocab):
            assert g.push(t) == 0
    state = [dict(count=0, frames=[]) for _ in rings]
    counts = {"tokens": 0, "marks": 0, "commits": 0, "failures": 0}

    def step():
        for g, st in zip(rings, state):
            sv = g.session.view()
            if st["count"] % cfg["fail_every"] == cfg["fail_every"] // 2:
                g.fail(27, sv.position)  # injected failure, then recovery by a retry
                assert g.push(sv.pending) == -77
                counts["failures"] += 1
            assert g.push(sv.pending) == 0
            counts["tokens"] += 1
            st["count"] += 1
            if st["count"] % cfg["mark_every"] == 0 and len(st["frames"]) < 2:
                status, frame = g.mark()
                assert status == 0
                st["frames"].append(frame)
                counts["marks"] += 1
            elif st["count"] % cfg["mark_every"] == cfg["mark_every"] // 2 and st["frames"]:
                assert g.commit(st["frames"].pop()) == 0
                counts["commits"] += 1

    t_warm = time.time()
    for _ in range(max(args.warmup, 3)):
        step()
    L.gpu_sync()
    for key in counts:
        counts[key] = 0
    barrier(dist, torch)
    L.qwen_b200_mark(0)
    for _ in range(args.steps):
        step()
    L.qwen_b200_mark(1)
    L.gpu_sync()
    device_ms = L.qwen_b200_elapsed_ms(0, 1)
    clocks = clocks_between(t_warm, time.time())
    timed = dict(counts)
    barrier(dist, torch)
    device_ms = max_over_ranks(device_ms, dist, torch)
    # End to end: a second pass on the host clock.
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3, dist, torch)
    barrier(dist, torch)

    runner = rings[0].session.runner
    pos = rings[0].session.view().position
    es = 2
    gateup_ms = L.qwen_b200_time_stage(runner, 3, 0, pos - 1, 30)
    gateup_bytes = 2 * shape.intermediate * shape.hidden * es + shape.intermediate * 4
    ring_ms = L.qwen_b200_time_stage(runner, 1, 0, pos - 1, 30)
    peak, peak_kind = measured_peaks()
    achieved = gateup_bytes / (gateup_ms * 1e-3) / 1e9
    active = rings[0].view().active
    ring_bytes = shape.layers * active * 528 + 2 * shape.layers * 2 * 528 + 2 * shape.vocab * 4
    step_bytes = model.weight_bytes + ring_bytes
    tokens = timed["tokens"] * world
    ms_per_token = device_ms / max(timed["tokens"], 1)
    views = [g.view() for g in rings]
    for g in rings:
        g.close()
    model.free()
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("gateup_bf16")
    return {
        "metric": METRIC, "value": round(tokens / (device_ms * 1e-3), 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(device_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16-weights/f32/int8-kv", "data": "synthetic",
        "config": {"workload": "qwen2.5-1.5b-bf16-bounded", "layers": shape.layers, "batch": 1,
                   "sessions_per_gpu": cfg["sessions"], "sessions_total": cfg["sessions"] * world,
                   "retention": {"anchors": a, "recent": r, "reservoir": m}, "logical_context": cfg["logical"],
                   "prefill_tokens": cfg["prefill"], "retained_rows": active,
                   "timed_ops_per_rank": timed, "parallelism": f"replicas{world}",
                   "weights": "seeded N(0,0.02) random init",
                   "l2": "inputs larger than L2 (weights stream from HBM every token)"},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 2), "unit": "tokens/s", "h2d_bytes_per_step": 64 * len(rings),
                "d2h_bytes_per_step": 64 * len(rings)},
        "gpu_launches": (5 * shape.layers + 2) * (timed["tokens"] + timed["failures"]),
        "roofline": {"bound": "hbm", "kernel": "gateup_kernel (RMSNorm + gate/up GEMV + SwiGLU)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": gateup_bytes,
                     "launch_ms": round(gateup_ms, 5)},
        "step_roofline": {"bytes_per_token": int(step_bytes),
                          "achieved_gbs": round(step_bytes / (ms_per_token * 1e6), 1),
                          "frac": round(step_bytes / (ms_per_token * 1e6) / peak, 4)},
        "ring_attention_ms_layer0": round(ring_ms, 5),
        "ring_state": [{"position": v.cursor, "evictions": v.population, "retained": v.active,
                        "restores": v.restores} for v in views],
        "clocks": clocks,
    }


def run_batched(args, cfg, world, rank, local, dist, torch):
    """64 sessions per GPU through the batched tensor-core engine."""
    import ctypes
    import numpy as np
    import cmachine_b200 as cm
    L = cm.lib()
    L.qwen_b200_set_device(local)
    shape = cm.qwen_shape(cfg["layers"], 9216)
    model = cm.Model(shape, 2026 + rank, cm.BENCH_LAW, cfg["profile"])
    n, seg = cfg["batch"], cfg["segment"]
    steps = max(seg, (args.steps // seg) * seg)
    strong = bool(cfg.get("strong"))
    if strong:  # one fixed set of `total` sessions, dealt round-robin over the ranks
        total = cfg["total"]
        every = np.random.default_rng(11).integers(cfg["ctx"][0], cfg["ctx"][1] + 1, total)
        ids = list(range(rank, total, world))
        lengths = [int(every[i]) for i in ids]
        n = len(lengths)
    else:
        rng = np.random.default_rng(11 + rank)
        lengths = [int(v) for v in rng.integers(cfg["ctx"][0], cfg["ctx"][1] + 1, n)]
        ids = [rank * n + i for i in range(n)]
    sessions = []
    t_prefill = time.time()
    for i, ln in zip(ids, lengths):
        s = cm.Session(model, ln + steps // 2 + seg + max(args.warmup, 3) + 2)
        # The context: a uniform-random prompt of ln token ids (seeded per
        # session), run through qwen_prefill (batched causal chunks of 64 tokens
        # on the tensor cores), so every cached K/V row is the model's own.
        prompt = np.random.default_rng(70000 + i).integers(0, shape.vocab, ln)
        assert s.prefill(prompt) == 0
        sessions.append(s)
    L.gpu_sync()
    prefill_s = time.time() - t_prefill
    batch = L.qwen_b200_batch_create(L.qwen_b200_model_decoder(model.handle))
    assert batch
    views = [s.view() for s in sessions]
    bs = (cm.BatchSession * n)(*[cm.BatchSession(v.keys, v.values, v.capacity, v.logits, v.x) for v in views])
    pos = [v.position for v in views]
    tok = [v.pending for v in views]
    tops = (cm.Top2 * n)()

    def segment(k, advance):
        nonlocal pos, tok
        cp, ct = (ctypes.c_int * n)(*pos), (ctypes.c_int * n)(*tok)
        assert L.qwen_b200_batch_enqueue(batch, n, bs, ct, cp, k) == 0
        assert L.qwen_b200_batch_read(batch, n, k, tops, None) == 0
        if advance:  # keep the segment; otherwise roll back to its checkpoint
            pos = [p + k for p in pos]
            tok = [tops[i].first for i in range(n)]

    t_warm = time.time()
    segment(max(args.warmup, 3), False)
    barrier(dist, torch)
    L.qwen_b200_mark(0)
    for c in range(steps // seg):
        segment(seg, c % 2 == 0)
    L.qwen_b200_mark(1)
    L.gpu_sync()
    device_ms = L.qwen_b200_elapsed_ms(0, 1)
    clocks = clocks_between(t_warm, time.time())
    barrier(dist, torch)
    device_ms = max_over_ranks(device_ms, dist, torch)
    mean_pos = sum(pos) / n
    # End to end through qwen_push_batch with session checkpoints.
    e2e_steps = min(steps, 2 * seg)
    handles = sessions
    ck = [s.checkpoint() for s in handles]
    assert all(st == 0 for st, _ in ck)
    barrier(dist, torch)
    t0 = time.perf_counter()
    for c in range(e2e_steps // seg):
        for _ in range(seg):
            assert cm.push_batch(handles, [s.pending for s in handles]) == 0
        if c % 2 == 0:
            for s, (_, cp) in zip(handles, ck):
                assert s.restore(cp) == 0
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3, dist, torch)
    barrier(dist, torch)

    # Stage times of layer 0 at the current cursors; the roofline is the
    # attention kernel's (the step's dominant bytes) and the tensor pipe's.
    cp, ct = (ctypes.c_int * n)(*pos), (ctypes.c_int * n)(*tok)
    names = ["qkv_gemm", "attention", "o_gemm", "gateup_gemm", "down_gemm", "vocab_gemm", "rmsnorm"]
    stage = {nm: L.qwen_b200_batch_time_stage(batch, n, bs, ct, cp, i, 0, 10) for i, nm in enumerate(names)}
    peak, peak_kind = measured_peaks()
    attn_bytes = sum((p + 1) * shape.kvheads * shape.head * 4 * 2 for p in pos)
    attn_gbs = attn_bytes / (stage["attention"] * 1e-3) / 1e9
    kv_step = sum((p + 1) for p in pos) * 57344  # K and V of every layer, once a step
    weight_bytes = model.weight_bytes
    step_bytes = weight_bytes + kv_step
    ms_per_step = device_ms / steps
    gemm_flops = 2 * 2 * 1543569408 * n  # hi and lo halves: two MMAs per product
    layer_gemm_ms = stage["qkv_gemm"] + stage["o_gemm"] + stage["gateup_gemm"] + stage["down_gemm"]
    tflops = (gemm_flops - 2 * 2 * shape.vocab * shape.hidden * n) / shape.layers / (layer_gemm_ms * 1e-3) / 1e12
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tc_peak = float(pk.get("bf16_tflops", 1590.0))
    gateup_bytes = 2 * shape.intermediate * shape.hidden * 2
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():  # ncu DRAM bytes per cache row (a 4,096-row capture), scaled to these rows
        per_row = json.loads(tf.read_text()).get("batch_attn_bytes_per_row")
        traffic = int(per_row * sum(p + 1 for p in pos)) if per_row else None
    per_step_launches = L.qwen_b200_batch_launches_per_step(batch)
    L.qwen_b200_batch_free(batch)
    parity = None
    if getattr(args, "ref_check", False) and world == 1:
        # Session 0's next batched step at its own context, checked by the reference CPU path.
        s0 = sessions[0]
        v0 = s0.view()
        kv = session_kv(s0, shape.layers)
        assert cm.push_batch([s0], [v0.pending]) == 0
        parity = {"max_abs_dlogit": reference_dlogit_at_context(shape.layers, cfg["profile"], 2026 + rank, kv,
                                                                 v0.position, v0.pending, s0.logits()),
                  "context_rows": v0.position, "session": 0,
                  "checker": "reference CPU path given the session's K/V rows (the prefilled context and the "
                             "decoded rows)"}
    for s in sessions:
        s.free()
    model.free()
    tokens_total = steps * (cfg["total"] if strong else n * world)
    return {
        "metric": METRIC, "value": round(tokens_total / (device_ms * 1e-3), 2), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "bf16-weights/f32", "data": "synthetic",
        "config": {"workload": "qwen2.5-1.5b-bf16-batch64", "layers": shape.layers, "batch": n,
                   "sessions_total": cfg["total"] if strong else n * world,
                   "context": "uniform 128..8192 per session (seeded)",
                   "mean_position": round(mean_pos, 1), "segment": seg,
                   "checkpoints": "every segment; rollback after every second segment",
                   "kv_prefill": "uniform-random prompt of each session's context length through qwen_prefill "
                                 "(untimed)", "prefill_s": round(prefill_s, 1),
                   "parallelism": f"replicas{world}", "weights": "seeded N(0,0.02) random init",
                   "l2": "inputs larger than L2 (weights and K/V stream from HBM every step)"},
        "e2e": {"value": round(e2e_steps * tokens_total / steps / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": n * 8, "d2h_bytes_per_step": n * 16},
        "gpu_launches": per_step_launches * (steps + max(args.warmup, 3)),
        "roofline": {"bound": "hbm",
                     "kernel": "batch_attn_tc_kernel + batch_attn_merge_kernel (64 sessions x 2 KV heads, "
                               "split-K flash decoding on TF32 tensor-core fragments)",
                     "achieved": round(attn_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(attn_gbs / peak, 4),
                     "peak_source": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": int(attn_bytes),
                     "launch_ms": round(stage["attention"], 5)},
        "tensor_roofline": {"bound": "tensor", "kernels": "tc_gemm_kernel (q/k/v, O, gate/up, down of one layer)",
                            "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                            "frac": round(tflops / tc_peak, 4),
                            "note": "two BF16 MMAs per product (activation hi and lo halves); the GEMMs are HBM-bound",
                            "gateup_hbm_gbs": round(gateup_bytes / (stage["gateup_gemm"] * 1e-3) / 1e9, 1)},
        "step_roofline": {"bytes_per_step": int(step_bytes), "achieved_gbs": round(step_bytes / (ms_per_step * 1e6), 1),
                          "frac": round(step_bytes / (ms_per_step * 1e6) / peak, 4)},
        "stage_ms_layer0": {k: round(v, 5) for k, v in stage.items()},
        "clocks": clocks,
        **({"parity_at_context": parity} if parity else {}),
    }


REF_MODEL = {}  # the CPU leg's model of the last (layers, profile, seed), kept for the next use


def reference_model(layers: int, profile: int, seed: int):
    """The CPU leg's seeded model (the reference's CPU path from oracle/_ref,
    else the oracle restatement): (library, model, kind). Building a 28-layer
    model takes most of a minute on the host, so the last one is kept for the
    CPU-baseline timing and the parity check of the same configuration."""
    sys.path.insert(0, str(ROOT / "tests"))
    import ctypes
    import cmachine_b200 as cm
    from checkers import ORACLE, REF_CPU, load
    key = (layers, profile, seed)
    if key not in REF_MODEL:
        for L, model, _ in REF_MODEL.values():
            L.orc_model_free(model)
        REF_MODEL.clear()
        path, kind = (REF_CPU, "reference") if REF_CPU.exists() else (ORACLE, "port")
        L = load(path)
        shape = cm.qwen_shape(layers, 32768)
        model = L.orc_model_create(ctypes.byref(shape), seed, ctypes.byref(cm.BENCH_LAW), int(profile == 2))
        REF_MODEL[key] = (L, model, kind)
    return REF_MODEL[key]


def reference_dlogit_at_context(layers: int, profile: int, seed: int, kv, position: int, token: int, gpu_logits):
    """Part of the CPU-baseline leg, as the checker: the reference's own CPU
    path (oracle/_ref, else the oracle restatement) receives the GPU session's
    K/V rows 0..position-1 of every layer (kv[layer][kind], [kvheads][position]
    [head]), places its cursor there and pushes `token`, the token the GPU
    session pushed at `position`; returns max |delta logit| against the GPU's
    logits of that push. This checks the decode step at the workload's real
    context without prefilling it on the CPU."""
    sys.path.insert(0, str(ROOT / "tests"))
    import ctypes
    import numpy as np
    import cmachine_b200 as cm
    L, model, _ = reference_model(layers, profile, seed)
    session = L.orc_session_create(model, position + 1)
    try:
        for layer in range(layers):
            for kind in (0, 1):
                rows = np.ascontiguousarray(kv[layer][kind], np.float32)
                L.orc_write_kv(session, layer, kind, position, ctypes.c_void_p(rows.ctypes.data))
        assert L.orc_set_cursor(session, position) == 0
        top = cm.Top2()
        logits = np.empty(gpu_logits.size, np.float32)
        assert L.orc_push(session, token, ctypes.byref(top), ctypes.c_void_p(logits.ctypes.data)) == 0
        return float(np.max(np.abs(gpu_logits - logits)))
    finally:
        L.orc_session_free(session)


def session_kv(session, layers: int):
    return [[session.kv(layer, kind) for kind in (0, 1)] for layer in range(layers)]


def gpu_dlogit(layers: int, profile: int, ref_logits, context: int = 0):
    """max |delta logit| of the GPU path on the CPU sample's first thread (the
    same context rows, prompt and greedy steps)."""
    import numpy as np
    import cmachine_b200 as cm
    if not ref_logits:
        return None
    model = cm.Model(cm.qwen_shape(layers, 32768), 2026, cm.BENCH_LAW, profile)
    s = cm.Session(model, context + 64)
    worst = 0.0
    toks = prompt_tokens(90, 1 if context else 2, model.shape.vocab)
    if context:
        kv = context_kv(layers, context)
        for layer in range(layers):
            for kind in (0, 1):
                s.write_kv(layer, kind, kv[layer][kind])
        assert s.set_cursor(context, toks[0]) == 0
    for t in toks:
        s.push(t)
    for ref in ref_logits:
        s.push(s.pending)
        worst = max(worst, float(np.max(np.abs(s.logits() - ref))))
    s.free()
    model.free()
    return worst


# ---------------------------------------------------------------- B200 arm
def batch1_config(name: str, cfg, world: int, tp: bool = False):
    """The workload of a batch-1 configuration, as both arms report it."""
    return {"workload": f"qwen2.5-1.5b-{name}", "layers": cfg["layers"], "batch": 1,
            "prompt_tokens": cfg["prompt"], "decode_window": cfg["window"],
            "weights": "seeded N(0,0.02) random init",
            "parallelism": f"tensor{world} (MLP units and readout rows split, peer-memory exchange)" if tp
            else f"replicas{world}",
            "l2": "inputs larger than L2 (weights stream from HBM every step)"}


def run_b200(args, cfg, world, rank, local, dist, torch, tp=False):
    """Batch-1 decode: one independent session per GPU, or with tp one session
    split over all the GPUs (tensor-parallel MLP and readout)."""
    import cmachine_b200 as cm
    L = cm.lib()
    L.qwen_b200_set_device(local)
    shape = cm.qwen_shape(cfg["layers"], 32768)
    salt = 0 if tp else rank  # a tensor-parallel group decodes one model and one prompt
    model = cm.Model(shape, 2026 + salt, cm.BENCH_LAW, cfg["profile"])
    capacity = cfg["prompt"] + cfg["window"] + 1
    s = cm.Session(model, capacity)
    if tp:
        status, handle = s.tp_open(rank, world)
        assert status == 0
        assert s.tp_connect(cm.tp_gather(dist, handle)) == 0
    # The prompt through qwen_prefill (batched causal tensor-core steps on a BF16
    # model; token by token on FP32), timed on the device.
    L.gpu_sync()
    barrier(dist, torch)
    L.qwen_b200_mark(4)
    assert s.prefill(prompt_tokens(7 + salt, cfg["prompt"], shape.vocab)) == 0
    L.qwen_b200_mark(5)
    L.gpu_sync()
    prefill_ms = L.qwen_b200_elapsed_ms(4, 5)
    barrier(dist, torch)
    status, ckpt = s.checkpoint()
    assert status == 0
    p0, pos0, window = s.pending, s.position, cfg["window"]
    runner = s.runner
    if args.token_mode == "persistent":
        assert s.persistent(1) == 1
    per_token_launches = L.qwen_b200_launches_per_token(runner)

    def enqueue_steps(k):
        while k > 0:
            n = min(k, window)
            assert L.qwen_b200_enqueue(runner, p0, pos0, n) == 0
            k -= n

    # Warm-up, then exactly K timed chained steps.
    t_warm = time.time()
    enqueue_steps(max(args.warmup, 3))
    L.gpu_sync()
    barrier(dist, torch)
    L.qwen_b200_mark(0)
    enqueue_steps(args.steps)
    L.qwen_b200_mark(1)
    L.gpu_sync()
    device_ms = L.qwen_b200_elapsed_ms(0, 1)
    clocks = clocks_between(t_warm, time.time())
    barrier(dist, torch)
    top = cm.Top2()
    assert L.qwen_b200_last(runner, top) == 0
    device_ms = max_over_ranks(device_ms, dist, torch)

    # End to end through qwen_advance (host round trip every step).
    assert s.restore(ckpt) == 0
    for _ in range(max(args.warmup, 3)):
        assert s.advance() == 0
    assert s.restore(ckpt) == 0
    barrier(dist, torch)
    L.qwen_b200_mark(2)
    done = 0
    while done < args.steps:
        n = min(args.steps - done, window)
        for _ in range(n):
            assert s.advance() == 0
        done += n
        assert s.restore(ckpt) == 0
    L.qwen_b200_mark(3)
    L.gpu_sync()
    e2e_ms = max_over_ranks(L.qwen_b200_elapsed_ms(2, 3), dist, torch)
    barrier(dist, torch)

    # Roofline of the dominant kernel: the fused gate/up GEMV (half the bytes;
    # with tp this rank's 1/world of its rows).
    es = 2 if cfg["profile"] == 2 else 4
    share = world if tp else 1
    gateup_ms = L.qwen_b200_time_stage(runner, 3, 0, pos0, 30)
    gateup_bytes = (2 * shape.intermediate * shape.hidden * es + shape.intermediate * 4) // share
    peak, peak_kind = measured_peaks()
    achieved = gateup_bytes / (gateup_ms * 1e-3) / 1e9
    weight_bytes = model.weight_bytes
    if tp:  # per GPU: the MLP matrices and the readout rows are split, the rest replicated
        split = (3 * shape.intermediate * shape.hidden * shape.layers + shape.vocab * shape.hidden) * es
        weight_bytes = weight_bytes - split + split // world
    mean_ctx = pos0 + window / 2
    kv_bytes = 2 * shape.layers * shape.kvheads * shape.head * 4 * mean_ctx
    step_bytes = weight_bytes + kv_bytes
    ms_per_step = device_ms / args.steps
    stage_names = ["qkv", "attention", "oproj", "gateup", "down", "readout"]
    stage_ms = {name: round(L.qwen_b200_time_stage(runner, i, 0, pos0, 10), 5) for i, name in enumerate(stage_names)
                if not (tp and i >= 4)}  # the group's exchange stages run only as whole tokens
    barrier(dist, torch)
    if tp:
        assert s.tp_close() == 0
        barrier(dist, torch)
    parity = None
    if getattr(args, "ref_check", False) and world == 1:
        # The GPU's next token at the workload's context, checked by the reference CPU path.
        assert s.restore(ckpt) == 0
        kv = session_kv(s, shape.layers)
        assert s.push(p0) == 0
        parity = {"max_abs_dlogit": reference_dlogit_at_context(shape.layers, cfg["profile"], 2026 + salt, kv, pos0, p0,
                                                                 s.logits()),
                  "context_rows": pos0, "checker": "reference CPU path given the session's K/V rows"}
    s.free()
    model.free()
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"gateup_{'bf16' if es == 2 else 'fp32'}")

    sessions = 1 if tp else world
    line = {
        "metric": METRIC, "value": round(args.steps * sessions / (device_ms * 1e-3), 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "strong" if tp else "weak",
        "vs_baseline": None, "dtype": "bf16-weights/f32" if es == 2 else "f32", "data": "synthetic",
        "config": batch1_config(args.config, cfg, world, tp),
        "execution": {"token": args.token_mode},
        "e2e": {"value": round(args.steps * sessions / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 32},
        "gpu_launches": per_token_launches * args.steps + (args.steps + window - 1) // window,
        "roofline": {"bound": "hbm", "kernel": "gateup_kernel (RMSNorm + gate/up GEMV + SwiGLU)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": gateup_bytes,
                     "launch_ms": round(gateup_ms, 5)},
        "step_roofline": {"bytes_per_step": int(step_bytes), "achieved_gbs": round(step_bytes / (ms_per_step * 1e6), 1),
                          "frac": round(step_bytes / (ms_per_step * 1e6) / peak, 4)},
        "stage_ms_layer0": stage_ms,
        "prefill": {"tokens": cfg["prompt"], "ms": round(prefill_ms, 3),
                    "tokens_per_s": round(cfg["prompt"] / (prefill_ms * 1e-3), 1),
                    "path": "batched tensor-core steps of 64 tokens" if es == 2 else "token by token (FP32 weights)"},
        "clocks": clocks,
        "last_top2": top.tuple(),
    }
    if parity:
        line["parity_at_context"] = parity
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default=DEFAULT_CONFIG)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default configuration only: skip the batch-64, long-context and bounded sub-lines")
    ap.add_argument("--token-mode", choices=["graph", "persistent"], default="graph",
                    help="batch-1 whole-token execution: the per-stage token graph or the persistent kernel")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        if "ring" in cfg:
            got = cpu_reference_ring_rate(cfg)
            if got is None:
                print(json.dumps({"impl": "reference", "unavailable": "the reference ring build (oracle/_ref) is absent"}))
                return
            rate, cores, sample, kind = got
        else:
            rate, cores, sample, kind, _ = cpu_reference_rate(cfg["layers"], cfg["profile"] == 2,
                                                              context=ref_context(cfg))
        print(json.dumps({
            "metric": METRIC, "impl": "reference", "value": round(rate, 4), "unit": "tokens/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 / rate, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16-weights/f32" if cfg["profile"] == 2 else "f32", "data": "synthetic",
            "config": (batch1_config(args.config, cfg, int(os.environ.get("WORLD_SIZE", "1"))) if "prompt" in cfg
                       else {"workload": f"qwen2.5-1.5b-{args.config}", "layers": cfg["layers"], "batch": 1}),
            "cpu_baseline": {"value": round(rate, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(rate, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    world, rank, local, dist, torch = dist_setup(args.gpus)
    global CLOCKS
    CLOCKS = ClockSampler(local).start()
    try:
        args.ref_check = world == 1 and not args.no_cpu_baseline  # the CPU-baseline leg's checker, 1 GPU only
        line = run_workload(args, args.config, world, rank, local, dist, torch, cpu=not args.no_cpu_baseline)
        if args.config == DEFAULT_CONFIG and not args.no_extras:
            # The other configurations the metric names, measured in the same run:
            # 64-session batched decode (weak scaling: 64 sessions per GPU; at N > 1
            # also strong scaling: 64 sessions in all), BF16 long context, and the
            # bounded byte-codec sessions.
            line["bs64"] = compact(run_workload(args, "bf16-batch64", world, rank, local, dist, torch))
            if world > 1:
                strong = dict(CONFIGS["bf16-batch64"], strong=True, total=64)
                line["bs64_strong"] = compact(run_batched(args, strong, world, rank, local, dist, torch))
            line["bf16_ctx4096"] = compact(run_workload(args, "bf16-ctx4096", world, rank, local, dist, torch))
            args.ref_check = False
            line["bounded"] = compact(run_workload(args, "bf16-bounded", world, rank, local, dist, torch))
            if world > 1 and world in (2, 4, 8):
                # Last, so that a failure here costs only this sub-line: one
                # session split over all the GPUs (tensor-parallel MLP and readout).
                sub = argparse.Namespace(**vars(args))
                sub.config = "bf16-ctx4096"
                try:
                    line["bf16_ctx4096_tp"] = compact(run_b200(sub, CONFIGS["bf16-ctx4096"], world, rank, local, dist,
                                                               torch, tp=True))
                except Exception as e:  # every rank runs the same steps, so all fail alike
                    line["bf16_ctx4096_tp"] = {"error": repr(e)[:300]}
    finally:
        CLOCKS.stop()
    if rank == 0:
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


DEFAULT_CONFIG = "fp32-ctx512"


def compact(line):
    """A workload's line as a sub-object of the headline line."""
    return {k: v for k, v in line.items() if k not in ("metric", "higher_is_better", "vs_baseline", "data")}


def run_workload(args, name, world, rank, local, dist, torch, cpu=False):
    """One configuration's line; with cpu, rank 0 of a 1-GPU run adds the
    reference CPU path timed on the host cores."""
    cfg = CONFIGS[name]
    sub = argparse.Namespace(**vars(args))
    sub.config = name
    if "batch" in cfg:
        line = run_batched(sub, cfg, world, rank, local, dist, torch)
        if cpu and rank == 0 and world == 1:
            rate, cores, sample, kind, _ = cpu_reference_rate(cfg["layers"], True, context=ref_context(cfg))
            line["cpu_baseline"] = {"value": round(rate, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
                                    "sample": sample + "; at these sessions' contexts the reference's attention adds "
                                              "about a quarter to each token's arithmetic"}
        return line
    if "ring" in cfg:
        line = run_bounded(sub, cfg, world, rank, local, dist, torch)
        if cpu and rank == 0 and world == 1:
            got = cpu_reference_ring_rate(cfg)
            if got:
                rate, cores, sample, kind = got
                line["cpu_baseline"] = {"value": round(rate, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
                                        "sample": sample}
        return line
    line = run_b200(sub, cfg, world, rank, local, dist, torch)
    if cpu and rank == 0 and world == 1:
        rate, cores, sample, kind, ref_logits = cpu_reference_rate(cfg["layers"], cfg["profile"] == 2,
                                                                   context=ref_context(cfg))
        line["cpu_baseline"] = {"value": round(rate, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
                                "sample": sample}
        line["max_abs_dlogit"] = gpu_dlogit(cfg["layers"], cfg["profile"], ref_logits, context=ref_context(cfg))
    return line


if __name__ == "__main__":
    main()
