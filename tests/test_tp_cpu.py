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


@pytest.mark.parametrize("elem_bytes", [4, 2], ids=["fp32", "bf16"])
@pytest.mark.parametrize("shards", [1, 2, 4, 8])
def test_down_projection_tiling_covers_every_column_once(elem_bytes, shards):
    """The down kernel's geometry (csrc/decode.cu DownGeo): a rank reads
    F = 8960 / shards columns of each row, RD rows a stage, and its eight
    consumer warps split a stage into PIECES pieces per row or RPW rows per warp.
    Every (row slot, column) of a stage must be read by exactly one warp and lane
    step, every copy must be whole 16-byte vectors at 16-byte-aligned offsets,
    and a stage must stay within the 35 KB the ring was sized for."""
    inter, warps = 8960, 8
    E = 16 // elem_bytes
    RD_base = 1 if elem_bytes == 4 else 2
    F = inter // shards
    RD = RD_base * shards
    PIECES = 1 if RD >= warps else warps // RD
    RPW = RD // warps if RD >= warps else 1
    NVP = F // E // PIECES
    KV = (NVP + 31) // 32
    assert F % (E * PIECES) == 0 and (F * elem_bytes) % 16 == 0
    assert PIECES * RD == warps or RPW * warps == RD
    assert RD * F * elem_bytes <= 35840
    for rank in range(shards):
        assert (rank * F * elem_bytes) % 16 == 0  # the column offset of this rank's copies
    seen = {}
    for warp in range(warps):
        piece = warp % PIECES if PIECES > 1 else 0
        for j in range(RPW):
            slot = warp // PIECES if PIECES > 1 else warp + warps * j
            for lane in range(32):
                for k in range(KV):
                    if lane + 32 * k < NVP:
                        v = piece * NVP + lane + 32 * k
                        for e in range(E):
                            key = (slot, E * v + e)
                            assert key not in seen
                            seen[key] = warp
    assert len(seen) == RD * F
    assert all(0 <= s < RD and 0 <= c < F for s, c in seen)
