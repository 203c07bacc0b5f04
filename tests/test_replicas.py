"""The multi-GPU host logic on CPU: two gloo ranks (spawned processes) split the
streams round-robin, meet at barriers and agree on the max elapsed time; a rank
whose peer never joins gets an error from the short process-group timeout
instead of hanging; the reference arm runs on rank 0 only."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    from nvcr_b200.replicas import Group, rank_environment, streams_of

    env = rank_environment()
    group = Group(env, "gloo", timeout_s=30)
    mine = streams_of(env.rank, env.world, 64)
    group.barrier()
    slowest = group.max(float(10 + env.rank))
    differing = group.sum(float(env.rank + 1))
    group.barrier()
    group.close()
    results.put((env.rank, mine, slowest, differing))


def test_streams_split_round_robin():
    from nvcr_b200.replicas import streams_of

    for world in (1, 2, 4, 8):
        shards = [streams_of(r, world, 64) for r in range(world)]
        assert sorted(s for shard in shards for s in shard) == list(range(64))
        assert all(len(shard) == 64 // world for shard in shards)
        assert all(s % world == r for r, shard in enumerate(shards) for s in shard)
    with pytest.raises(ValueError):
        streams_of(2, 2, 64)


def test_two_gloo_ranks_agree():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(results.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [g[0] for g in got] == [0, 1]
    assert got[0][1] == list(range(0, 64, 2)) and got[1][1] == list(range(1, 64, 2))
    assert got[0][2] == got[1][2] == 11.0  # the max over ranks
    assert got[0][3] == got[1][3] == 3.0   # the sum over ranks


def _lonely(port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="2", RANK="0", LOCAL_RANK="0")
    sys.path.insert(0, str(ROOT))
    from nvcr_b200.replicas import Group, rank_environment

    try:
        Group(rank_environment(), "gloo", timeout_s=3)
        results.put("joined")
    except Exception as error:  # the peer never arrives: rendezvous times out
        results.put(f"error: {type(error).__name__}")


def test_missing_peer_ends_with_an_error():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(free_port(), results))
    p.start()
    outcome = results.get(timeout=120)
    p.join(timeout=60)
    assert outcome.startswith("error"), outcome


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                           "--steps", "1", "--warmup", "0"], env=env, capture_output=True, text=True, timeout=120)
    assert done.returncode == 0
    assert done.stdout.strip() == ""
