"""Tensor-parallel decode of one session over 2, 4 or 8 GPUs (one process each).

Each rank loads the same seeded model and opens the same session, exports its
exchange handle, gathers the other's over a gloo process group, connects, and
decodes the same prompt and greedy continuation. Checked on every token:
  - rank 0's logits against the oracle (the reference's CPU FP32 path
    restated) within 1e-3 for FP32 weights and 3e-2 for BF16 weights;
  - both ranks hold bit-identical logits, top-2 and K/V rows (the exchange
    adds the partials in rank order on every rank);
  - against the same decode on one GPU within the same bounds (only the order
    of the down projection's sum differs).
Each world size runs where the box has that many GPUs and is skipped otherwise.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, world, port, profile, out):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import hashlib
    from datetime import timedelta

    import torch.distributed as dist

    import cmachine_b200 as cm
    from checkers import ORACLE, CpuDecoder
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    result = {"rank": rank}
    try:
        L = cm.lib()
        L.qwen_b200_set_device(rank)
        shape = cm.qwen_shape(2, 4096)
        seed = 31 + profile
        model = cm.Model(shape, seed, cm.TEST_LAW, profile)
        s = cm.Session(model, 64)
        status, handle = s.tp_open(rank, world)
        assert status == 0, "tp_open"
        assert s.tp_connect(cm.tp_gather(dist, handle)) == 0, "tp_connect"
        assert s.tp_world == world
        dist.barrier()
        # The group's tokens first, back to back on both ranks (the checks on
        # the CPU come after, so no rank lags the other by host work).
        tokens = [int(t) for t in np.random.default_rng(seed).integers(0, shape.vocab, 6)]
        fed, seen, digests = [], [], []
        for i in range(len(tokens) + 10):
            token = tokens[i] if i < len(tokens) else s.pending
            assert s.push(token) == 0, f"push {i}"
            fed.append(token)
            logits = s.logits()
            seen.append(logits)
            digests.append(hashlib.sha256(logits.tobytes() + repr(s.top).encode()).hexdigest())
        kv = hashlib.sha256(b"".join(s.kv(l, k).tobytes() for l in range(shape.layers) for k in (0, 1))).hexdigest()
        dist.barrier()
        assert s.tp_close() == 0
        dist.barrier()
        worst_oracle = worst_single = 0.0
        if rank == 0:
            oracle = CpuDecoder(ORACLE, shape, seed, cm.TEST_LAW, profile == 2, 64)
            single = cm.Session(model, 64)  # the same tokens on this GPU alone
            for token, logits in zip(fed, seen):
                _, want = oracle.push(token)
                worst_oracle = max(worst_oracle, float(np.max(np.abs(logits - want))))
                assert single.push(token) == 0
                worst_single = max(worst_single, float(np.max(np.abs(logits - single.logits()))))
            oracle.close()
            single.free()
        result.update(digests=digests, kv=kv, worst_oracle=worst_oracle, worst_single=worst_single,
                      position=s.position)
        s.free()
        model.free()
    except Exception as e:  # reported to the parent
        result["error"] = repr(e)
    out.put(result)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("profile", [0, 2], ids=["fp32", "bf16"])
def test_tensor_parallel(profile, world):
    if gpu_count() < world:
        pytest.skip(f"tensor-parallel decode over {world} GPUs needs {world} GPUs")
    import torch.multiprocessing as mp
    tol = 1e-3 if profile == 0 else 3e-2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + 10 * world + profile
    procs = [ctx.Process(target=_rank, args=(r, world, port, profile, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=600) for _ in procs), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=120)
    for r in results:
        assert "error" not in r, r
    for p in procs:
        assert p.exitcode == 0
    a = results[0]
    for b in results[1:]:
        assert a["digests"] == b["digests"], f"ranks 0 and {b['rank']} disagree on logits or top-2"
        assert a["kv"] == b["kv"], f"ranks 0 and {b['rank']} disagree on K/V"
    print(f"TP-{world} profile {profile}: max|dlogit| vs oracle {a['worst_oracle']:.3e}, vs one GPU {a['worst_single']:.3e}")
    assert a["worst_oracle"] <= tol
    assert a["worst_single"] <= tol
