"""Host side of tensor-parallel decode, on the CPU.

- Two gloo ranks exchange tensor-parallel handles with cmachine_b200.tp_gather:
  every rank receives every handle, in rank order (what qwen_session_tp_connect
  expects).
- The vocabulary and MLP shares tile their ranges exactly once at 2, 4 and 8
  ranks (the kernels' split: floor(rank * total / world)).
- The session host refuses to open a group where no fused runner exists (the
  host built over the reference's CPU primitives), leaving the session usable.
"""
import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import cmachine_b200 as cm


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mine = bytes([rank + 1]) * 16 + bytes(cm.TP_HANDLE_BYTES - 16)
    out.put((rank, cm.tp_gather(dist, mine)))
    dist.destroy_process_group()


def test_handles_gathered_in_rank_order_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, 29631, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = b"".join(bytes([r + 1]) * 16 + bytes(cm.TP_HANDLE_BYTES - 16) for r in range(2))
    assert got == [(0, want), (1, want)]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shares_tile_vocabulary_and_mlp(world):
    for total in (151936, 8960, 1536, 4099):
        shares = cm.tp_shares(total, world)
        assert shares[0][0] == 0 and shares[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(shares, shares[1:]))
        assert max(e - b for b, e in shares) - min(e - b for b, e in shares) <= 1
    assert all(e - b == 8960 // world for b, e in cm.tp_shares(8960, world))


def test_host_refuses_group_without_fused_runner():
    from checkers import ROOT
    path = ROOT / "oracle" / "_ref" / "libqwen_host_cpu.so"
    if not path.exists():
        pytest.skip("CPU host build absent")
    L = cm.load_library(path)
    shape = cm.Shape(256, 2, 2, 1, 128, 512, 1024, 64, 1e-6, 1e6)
    model = cm.Model(shape, 5, cm.TEST_LAW, 0, fused=False, library=L)
    s = cm.Session(model, 16)
    status, _ = s.tp_open(0, 2)
    assert status == -1
    assert s.tp_connect(bytes(2 * cm.TP_HANDLE_BYTES)) == -1
    assert s.push(3) == 0  # still a working session
    s.free()
    model.free()
