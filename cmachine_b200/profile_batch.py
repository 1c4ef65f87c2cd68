"""A short batched decode for profilers (ncu): a seeded BF16 Qwen2.5-architecture
model, `--sessions` sessions with `--context` cached rows each (seeded K/V),
and `--steps` batched greedy steps through the tensor-core engine, so that a
kernel capture sees the step's kernels without a long run first.

    python -m cmachine_b200.profile_batch --layers 2 --sessions 64 --context 512 --steps 2
"""
from __future__ import annotations

import argparse
import ctypes
from ctypes import c_void_p

import cmachine_b200 as cm


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--context", type=int, default=512)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--seed", type=int, default=2026)
    args = ap.parse_args()
    L = cm.lib()
    shape = cm.qwen_shape(args.layers, 9216)
    model = cm.Model(shape, args.seed, cm.BENCH_LAW, 2)
    sessions = []
    for i in range(args.sessions):
        s = cm.Session(model, args.context + args.steps + 1)
        v = s.view()
        count = shape.layers * shape.kvheads * v.capacity * shape.head
        L.qwen_b200_seeded_fill(c_void_p(v.keys), 1, 7, 1000 + 2 * i, count, 0.0, 0.8)
        L.qwen_b200_seeded_fill(c_void_p(v.values), 1, 7, 1001 + 2 * i, count, 0.0, 0.8)
        assert L.qwen_b200_session_set_cursor(s.handle, args.context, (i * 7919 + 11) % shape.vocab) == 0
        sessions.append(s)
    for _ in range(args.steps):
        assert cm.push_batch(sessions, [s.pending for s in sessions]) == 0
    print(f"{args.sessions} sessions x {args.steps} batched steps at context {args.context}: "
          f"pending {[s.pending for s in sessions[:4]]} ...")
    for s in sessions:
        s.free()
    model.free()


if __name__ == "__main__":
    main()
