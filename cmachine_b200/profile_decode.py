"""A short decode run for profilers (ncu): builds a seeded Qwen2.5-architecture
model, prefills a few tokens through qwen_push and generates a few more with
qwen_generate, so that a launch list or a kernel capture sees the same kernels
as a long decode without thousands of launches first. With --context N the
session instead starts at position N over seeded synthetic K/V rows (the
attention then reads N rows, as after an N-token prompt).

    python -m cmachine_b200.profile_decode --layers 28 --profile 0 --prompt 4 --tokens 2
    python -m cmachine_b200.profile_decode --layers 28 --profile 2 --context 4096 --tokens 2
"""
from __future__ import annotations

import argparse
from ctypes import c_void_p

import cmachine_b200 as cm


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--profile", type=int, choices=[0, 2], default=0, help="0 FP32 weights, 2 BF16 weights")
    ap.add_argument("--prompt", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=2)
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--context", type=int, default=0, help="start at this position over seeded K/V instead")
    args = ap.parse_args()
    L = cm.lib()
    model = cm.Model(cm.qwen_shape(args.layers, 32768), args.seed, cm.BENCH_LAW, args.profile)
    session = cm.Session(model, max(args.prompt, args.context) + args.tokens + 1)
    if args.context:
        v = session.view()
        count = model.shape.layers * model.shape.kvheads * v.capacity * model.shape.head
        L.qwen_b200_seeded_fill(c_void_p(v.keys), 1, 7, 1000, count, 0.0, 0.8)
        L.qwen_b200_seeded_fill(c_void_p(v.values), 1, 7, 1001, count, 0.0, 0.8)
        assert L.qwen_b200_session_set_cursor(session.handle, args.context, 11) == 0
    else:
        for i in range(args.prompt):
            assert session.push((i * 7919 + 11) % model.shape.vocab) == 0
    status, ids = session.generate(args.tokens)
    assert status == 0
    print(f"{'context ' + str(args.context) if args.context else 'prompt ' + str(args.prompt)} tokens, generated {ids}")
    session.free()
    model.free()


if __name__ == "__main__":
    main()
