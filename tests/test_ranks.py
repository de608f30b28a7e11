"""The multi-GPU plumbing of bench.py on the CPU: two gloo ranks.

bench.py runs one replica a GPU (no data-path collective); what the ranks
share is the barrier and the max-over-ranks of the step time, and only rank 0
prints.  Those run here over gloo with world size 2 on 127.0.0.1.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, values, out):
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    dist.barrier()
    out[rank] = bench.max_over_ranks(values[rank], dist, "cpu")
    dist.barrier()
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    values = [3.25, 7.5]
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, values, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0] == 7.5 and out[1] == 7.5


def test_single_rank_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(1.5) == 1.5


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs (and prints) the reference arm."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1"],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libsdasm_ref.so").exists(), reason="reference kernels not built")
def test_reference_arm_line():
    """Rank 0's reference line: the driver contract's keys, the arm's kind, a positive rate, the GPU
    arm's config, and every host core in use although the launcher's OMP_NUM_THREADS says 1 (torchrun
    sets it so): the arm sets its thread count from the process's CPU affinity."""
    env = dict(os.environ, RANK="0", WORLD_SIZE="2", LOCAL_RANK="0", OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "0"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["unit"] == "image-steps/s"
    assert line["steps"] == 1 and abs(line["ms_per_step"] - 1e3 / line["value"]) < 1e-6 * line["ms_per_step"]
    import bench

    assert line["config"] == bench.unet_config(2, "")


def _guidance_worker(rank: int, world: int, port: int, out):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT / "stable-diffusion.assembly_b200"))
    import unet as U

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    groups = U.pair_groups(dist, world)
    group = groups[rank // 2]
    half = torch.full((1, 3, 2, 4), float(10 * rank + 1))
    full = torch.zeros(2, 3, 2, 4)
    U.gather_guidance(dist, group, half, full)
    out[rank] = full[:, 0, 0, 0].tolist()
    dist.barrier()
    dist.destroy_process_group()


def test_guidance_pairs_gloo():
    """Four ranks in two guidance pairs: each pair's lower rank holds the unconditional half, its higher
    rank the conditional one, and after the exchange both hold [unconditional, conditional] -- their own
    pair's, never the other pair's."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_guidance_worker, args=(r, 4, port, out)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    assert out[0] == out[1] == [1.0, 11.0]
    assert out[2] == out[3] == [21.0, 31.0]
