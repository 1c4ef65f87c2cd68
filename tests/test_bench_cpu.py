"""The benchmark's host side on the CPU: rank orchestration (barrier and
max-over-ranks) as two gloo ranks, and the reference arm's JSON line on the
reduced 2-layer configuration (the reference's own CPU path)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def _rank(rank, world, port, out):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bench.barrier(dist, torch)
    value = bench.max_over_ranks(float(10 + 5 * rank), dist, torch)
    out.put((rank, value))
    dist.destroy_process_group()


def test_max_over_ranks_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, 29617, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == [(0, 15.0), (1, 15.0)]


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libref_cpu.so").exists(), reason="reference build absent")
def test_reference_arm_line():
    env = dict(os.environ, ORACLE_THREADS="2")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "fp32-2layer",
                           "--steps", "4", "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env,
                          cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    # The reference arm reports the B200 arm's workload object, and its sample
    # decodes at the workload's cache length (the prompt's rows).
    assert line["config"] == bench.batch1_config("fp32-2layer", bench.CONFIGS["fp32-2layer"], 1)
    assert f"threads x ({bench.CONFIGS['fp32-2layer']['prompt']} cached rows" in line["cpu_baseline"]["sample"]


def test_reference_context_per_configuration():
    assert bench.ref_context(bench.CONFIGS["fp32-ctx512"]) == 512
    assert bench.ref_context(bench.CONFIGS["bf16-ctx4096"]) == 4096
    assert bench.ref_context(bench.CONFIGS["bf16-batch64"]) == (128 + 8192) // 2
    kv = bench.context_kv(2, 16)
    assert len(kv) == 2 and kv[1][0].shape == (2, 16, 128) and kv[1][0].dtype.name == "float32"


def test_clock_sampler_window():
    """The run-long sampler keeps only samples stamped inside the asked window
    and reports slowdown reasons seen there."""
    from datetime import datetime
    c = bench.ClockSampler(0)
    t = datetime(2026, 1, 2, 3, 4, 5).timestamp()

    def row(dt, mhz, thermal="Not Active"):
        stamp = datetime.fromtimestamp(t + dt).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return f"{stamp}, 0, {mhz}, 1965, 700.0, 0x0, Not Active, {thermal}, Not Active, Not Active\n"

    c.lines = [row(-5, 900), row(0.1, 1965), row(0.3, 1950), row(0.5, 1965, "Active"), row(9, 800)]
    got = c.summary(t, t + 0.5, pad=0.05)
    assert got["samples"] == 3 and got["sm_mhz"] == 1965 and got["sm_max_mhz"] == 1965
    assert got["reasons"] == ["hw_thermal_slowdown"]
    assert c.summary()["samples"] == 5
