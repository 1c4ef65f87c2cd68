"""Timeline of one fused decode token (qwen_b200_trace): where the time goes
between and inside the 141 launches of a token, or between the grid barriers
of the persistent token kernel.

    python -m cmachine_b200.trace_decode --profile 0 --prompt 512 --tokens 8 [--mode graph|persistent]

Persistent kernel: every CTA stamps the GPU global timer at its start, as it
passes each of the six grid barriers of a layer and when its readout rows are
done. Per phase (q/k/v, attention, merge, O, gate/up, down) the report gives the
mean over layers of the time from the previous barrier's release (its first
CTA through) to this one's, and how far apart the CTAs passed it.

Under torchrun with 2, 4 or 8 processes the session is split tensor-parallel
over the GPUs (MLP units and readout rows, peer-memory exchanges in the down
projection and the readout); every rank traces its own kernels and prints its
own report.

Token graph: every CTA of every launch stamps the GPU global timer at entry, when its
dependency on the previous launch was released (griddepcontrol.wait), when its
input vector was ready and when it finished. Per stage kind the report gives the
mean over layers of: the gap from the previous launch's last finish to this
launch's first release (boundary), release to input ready, ready to last
finish, and the whole span; then the token's total.
"""
from __future__ import annotations

import argparse
import ctypes

import numpy as np

import cmachine_b200 as cm

LAUNCHES, CTAS = 160, 320
STAGES = ["qkv", "attention", "oproj", "gateup", "down"]
PHASES = ["qkv", "attention", "merge", "oproj", "gateup", "down"]
MARKS = 512


def report_persistent(buf, layers, sms):
    t = buf[: sms * MARKS].reshape(sms, MARKS).astype(np.float64)
    k_last = 6 * layers
    start = t[:, 0].min()
    arrive = [None] + [t[:, 2 * k - 1] for k in range(1, k_last + 1)]
    passed = [t[:, 0]] + [t[:, 2 * k] for k in range(1, k_last + 1)]
    done = t[:, 2 * k_last + 1].max()
    print(f"persistent token: {(done - start) / 1000:.1f} us from the first CTA's start to the last readout row")
    print(f"{'phase':10s} {'interval':>8s} {'sum':>8s} {'work':>8s} {'barrier':>8s} {'arr spread':>10s}"
          f"   (us, mean over layers; work = previous release to the last arrival,"
          f" barrier = last arrival to the first CTA through)")
    for i, name in enumerate(PHASES):
        ks = [6 * l + i + 1 for l in range(layers)]
        interval = [passed[k].min() - passed[k - 1].min() for k in ks]
        work = [arrive[k].max() - passed[k - 1].min() for k in ks]
        bar = [passed[k].min() - arrive[k].max() for k in ks]
        spread = [arrive[k].max() - arrive[k].min() for k in ks]
        print(f"{name:10s} {np.mean(interval) / 1000:8.2f} {np.sum(interval) / 1000:8.1f} {np.mean(work) / 1000:8.2f}"
              f" {np.mean(bar) / 1000:8.2f} {np.mean(spread) / 1000:10.2f}")
    print(f"{'readout':10s} {(done - passed[k_last].min()) / 1000:8.2f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", type=int, choices=[0, 2], default=0)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--mode", choices=["graph", "persistent"], default="persistent")
    ap.add_argument("--lookahead", type=int, default=-1, help="persistent kernel L2 prefetch distance (KB)")
    ap.add_argument("--time", type=int, default=0, help="then time this many chained greedy tokens (device time)")
    args = ap.parse_args()
    L = cm.lib()
    import os
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if world > 1:
        from datetime import timedelta
        import torch.distributed as dist
        L.qwen_b200_set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    model = cm.Model(cm.qwen_shape(args.layers, 32768), 2026, cm.BENCH_LAW, args.profile)
    s = cm.Session(model, args.prompt + args.tokens + 9 + args.time)
    if world > 1:
        status, handle = s.tp_open(rank, world)
        assert status == 0 and s.tp_connect(cm.tp_gather(dist, handle)) == 0
        dist.barrier()
        print(f"rank {rank}: tensor-parallel over {world} GPUs", flush=True)
    for i in range(args.prompt):
        assert s.push((i * 7919 + 11) % model.shape.vocab) == 0
    runner = s.runner
    persistent = s.persistent(1 if args.mode == "persistent" else 0) == 1
    if persistent and args.lookahead >= 0:
        assert L.qwen_b200_persistent_tune(runner, 0, args.lookahead) == 0
    assert L.qwen_b200_trace(runner, 1) == 0
    status, _ = s.generate(args.tokens)
    assert status == 0
    buf = np.zeros(LAUNCHES * CTAS * 4, np.uint64)
    n = L.qwen_b200_trace_read(runner, ctypes.c_void_p(buf.ctypes.data), buf.size)
    L.qwen_b200_trace(runner, 0)
    if persistent:
        report_persistent(buf, args.layers, L.qwen_b200_sm_count())
        s.free()
        model.free()
        return
    t = buf.reshape(LAUNCHES, CTAS, 4).astype(np.float64)
    per_token = args.layers * 5 + 1
    t0 = np.min(t[0, :, 0][t[0, :, 0] > 0])
    rows = []
    prev_done = None
    for k in range(per_token):
        m = t[k]
        live = m[:, 0] > 0
        entry = m[live, 0] - t0
        rel = m[live, 1] - t0
        ready = m[m[:, 2] > 0, 2] - t0
        done = m[m[:, 3] > 0, 3] - t0
        kind = "readout" if k == per_token - 1 else STAGES[k % 5]
        both = (m[:, 2] > 0) & (m[:, 1] > 0)
        fin = (m[:, 3] > 0) & (m[:, 2] > 0)
        rec = dict(kind=kind, entry0=entry.min(), release0=rel.min(), ready1=ready.max() if ready.size else np.nan,
                   done1=done.max() if done.size else np.nan, release_spread=rel.max() - rel.min(),
                   cta_ready=np.median(m[both, 2] - m[both, 1]) if both.any() else np.nan,
                   cta_work=np.median(m[fin, 3] - m[fin, 2]) if fin.any() else np.nan,
                   done_spread=(done.max() - done.min()) if done.size else np.nan,
                   lead=np.median(m[live, 1] - m[live, 0]) if live.any() else np.nan)
        rec["boundary"] = rec["release0"] - prev_done if prev_done is not None else np.nan
        prev_done = rec["done1"]
        rows.append(rec)
    print(f"rank {rank}: launches recorded: {n}; token span {rows[-1]['done1'] / 1000:.1f} us")
    print(f"{'stage':10s} {'boundary':>9s} {'rel->ready':>10s} {'ready->done':>11s} {'span':>8s} "
          f"{'rel spread':>10s} {'cta ready':>9s} {'cta work':>9s} {'done spread':>11s} {'resident':>8s}"
          f"   (us, mean over layers; resident = a CTA's entry to its release, median)")
    for kind in STAGES + ["readout"]:
        sel = [r for r in rows if r["kind"] == kind]
        b = np.nanmean([r["boundary"] for r in sel]) / 1000
        rr = np.nanmean([r["ready1"] - r["release0"] for r in sel]) / 1000
        rd = np.nanmean([r["done1"] - r["ready1"] for r in sel]) / 1000
        sp = np.nanmean([r["done1"] - r["release0"] for r in sel]) / 1000
        extra = [np.nanmean([r[k] for r in sel]) / 1000
                 for k in ("release_spread", "cta_ready", "cta_work", "done_spread", "lead")]
        print(f"{kind:10s} {b:9.2f} {rr:10.2f} {rd:11.2f} {sp:8.2f} {extra[0]:10.2f} {extra[1]:9.2f} {extra[2]:9.2f}"
              f" {extra[3]:11.2f} {extra[4]:8.2f}")
    if args.time:
        # Chained greedy tokens from the same position, twice (device time between marks 0 and 1).
        pos0 = args.prompt + args.tokens
        for rep in range(2):
            assert L.qwen_b200_enqueue(runner, 1, pos0, 8) == 0
            L.gpu_sync()
            L.qwen_b200_mark(0)
            assert L.qwen_b200_enqueue(runner, 1, pos0, args.time) == 0
            L.qwen_b200_mark(1)
            L.gpu_sync()
            ms = L.qwen_b200_elapsed_ms(0, 1) / args.time
            print(f"{ms * 1000:.1f} us/token ({1000 / ms:.1f} tokens/s) over {args.time} chained tokens")
    if world > 1:
        dist.barrier()
        s.tp_close()
        dist.barrier()
    s.free()
    model.free()


if __name__ == "__main__":
    main()
