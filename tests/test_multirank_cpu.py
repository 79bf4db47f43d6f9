"""Host logic of the multi-GPU bench path, on CPU with gloo (world size 2).

The decode path shards by sequence with no collective: every rank builds its
own sequences from rank-seeded inputs (weak scaling) and the only
communication is the max over ranks of the timed values.  These tests run the
bench's helpers in two gloo processes and check the reference arm's rule that
only rank 0 works and prints.
"""
from __future__ import annotations

import importlib.util
import os
import socket
import subprocess
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("lf_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench = _bench()
        slowest = bench.max_over_ranks(1.5 + rank, "cpu")
        tails = bench.tails_for(bench.CONFIGS[1], rank)
        out.put((rank, slowest, list(tails)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_rank_sharding_gloo():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, m0, t0), (r1, m1, t1) = results
    assert (r0, r1) == (0, 1)
    assert m0 == m1 == 2.5  # every rank sees the slowest rank's time
    batch = _bench().CONFIGS[1]["batch"]
    assert len(t0) == len(t1) == batch
    assert t0 != t1  # each rank decodes its own sequences


def test_max_over_ranks_without_process_group_is_identity():
    assert _bench().max_over_ranks(3.25, "cpu") == 3.25


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                           "--steps", "1", "--warmup", "0"], env=env, capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""


def _gather_worker(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from logitfill_b200.sharding import assemble_heads, gather_heads, kv_head_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        B, NQ, H, D = 3, 40, 8, 16
        full = torch.arange(B * NQ * D, dtype=torch.float32).reshape(B, NQ, D)
        h0, h1, q0, q1 = kv_head_range(H, NQ, world, rank)
        local = full[:, q0:q1].contiguous()  # this rank's q-heads, as its K3 writes them
        gathered = torch.empty(world, B, q1 - q0, D)
        gather_heads(local, gathered)
        out.put((rank, bool(torch.equal(assemble_heads(gathered), full)), (h0, h1, q0, q1)))
    finally:
        dist.destroy_process_group()


def test_kv_head_gather_gloo():
    """KV-head sharding: each rank's q-heads gathered over the process group
    reassemble the full [B, n_q, D] output in q-head order."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in results] == [True, True]
    assert [r[2] for r in results] == [(0, 4, 0, 20), (4, 8, 20, 40)]


def test_kv_head_range_rules():
    import pytest

    from logitfill_b200.sharding import kv_head_range, shard_levels

    assert kv_head_range(8, 40, 8, 3) == (3, 4, 15, 20)
    assert kv_head_range(4, 28, 1, 0) == (0, 4, 0, 28)
    with pytest.raises(ValueError):
        kv_head_range(8, 40, 3, 0)
    import numpy as np

    levels = [np.arange(8 * 4).reshape(8, 4) % 4, None]
    got = shard_levels(levels, 8, 4, 2)
    assert got[1] is None and got[0].tolist() == (np.arange(8 * 4).reshape(8, 4) % 4)[4:6].tolist()
