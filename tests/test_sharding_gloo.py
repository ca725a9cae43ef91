"""Multi-rank session sharding on CPU: two ``gloo`` ranks on 127.0.0.1.

Covers the N > 1 host logic of the step: every session routes to exactly one
rank under ``shard_of``; each rank drives the packer oracle with only its own
rows; and the end-of-run reduction (max of times, sum of work) that
``bench.py --gpus N`` uses gives the whole-job numbers."""
from __future__ import annotations

import os
import random
import socket

import pytest
import torch.multiprocessing as mp

from tests.conftest import load_package


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _trace(seed: int, n_sessions: int, ticks: int):
    rng = random.Random(seed)
    sids = [f"user-{rng.randrange(10**9)}-{i}" for i in range(n_sessions)]
    trace = []
    for t in range(ticks):
        live = [s for s in sids if rng.random() < 0.8]
        trace.append([(s, 0, 0, t, t) for s in live])  # (session, generation, epoch, frame, seq)
    return sids, trace


def _rank_main(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch.distributed as dist

    from oracle.packer_ref import SlotPolicy

    load_package()
    from gemma4_omni_b200 import sharding

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sids, trace = _trace(7, 200, 12)
        mine = [s for s in sids if sharding.shard_of(s, world) == rank]
        owners = [None] * world
        dist.all_gather_object(owners, mine)
        policy = SlotPolicy(max_sessions=256)
        frames = 0
        for tick in trace:
            rows = sharding.split_rows(tick, world, key=lambda r: r[0])[rank]
            assert [r[0] for r in rows] == [r[0] for r in tick if sharding.shard_of(r[0], world) == rank]
            if rows:
                policy.prepare(rows)
                policy.commit()
                frames += len(rows)
        elapsed = 10.0 + rank  # a stand-in per-rank time
        (t_max,), (total,) = sharding.reduce_over_ranks([elapsed], [frames])
        out.put((rank, owners, frames, t_max, total, sorted(policy.slots_by_key)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_sessions_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    sids, trace = _trace(7, 200, 12)
    owners = res[0][1]
    assert owners == res[1][1]
    assert set(owners[0]).isdisjoint(owners[1]) and set(owners[0]) | set(owners[1]) == set(sids)
    assert 60 < len(owners[0]) < 140  # the hash spreads sessions
    total_frames = sum(len(t) for t in trace)
    assert res[0][2] + res[1][2] == total_frames
    for r in res:
        assert r[3] == 11.0 and r[4] == total_frames  # max time, summed work
    # each rank's packer only ever saw its own sessions
    assert {k[0] for k in res[0][5]} <= set(owners[0]) and {k[0] for k in res[1][5]} <= set(owners[1])


def test_shard_of_is_stable_and_total():
    load_package()
    from gemma4_omni_b200 import sharding

    assert sharding.shard_of(13, 4) == 1
    a = [sharding.shard_of(f"sess-{i}", 8) for i in range(4000)]
    assert a == [sharding.shard_of(f"sess-{i}", 8) for i in range(4000)]
    assert all(0 <= v < 8 for v in a) and min(a.count(k) for k in range(8)) > 400
    assert sharding.local_sessions(range(100), 1, 4, 5) == [1, 5, 9, 13, 17]
    with pytest.raises(ValueError):
        sharding.shard_of("x", 0)
