"""The multi-GPU bench's host plumbing at world size 2 over gloo on the CPU: replicas share no
data, the timed region is bracketed by barriers, the elapsed time is the max over ranks and
throughput counts every rank's chunks. (The GPU run uses NCCL for the same two calls.)"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from bench import Ranks, throughput

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r = Ranks(world, "cpu")
    r.barrier()
    elapsed = [120.0, 250.0][rank]  # the slower rank sets the job time
    ms = r.max(elapsed)
    out.put((rank, ms, throughput(world, 64, ms)))
    r.barrier()
    dist.destroy_process_group()


def test_two_rank_max_and_throughput():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [250.0, 250.0]
    assert abs(res[0][2] - 2 * 64 / 0.25) < 1e-9


def test_reference_arm_only_rank_zero_prints():
    """Under torchrun the reference (CPU) arm runs on rank 0 only; other ranks exit quietly."""
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], env=env, capture_output=True, text=True, timeout=300)  # fmt: skip
    assert r.returncode == 0 and r.stdout.strip() == ""
