"""GPU tick dispatcher snapshot and coordinator head order vs the CPU oracle
(bit-exact: same rows, same order, same pops and deferrals, same reason).

Model: tests/kernel/test_shared_listener_tick_dispatcher.py and
tests/kernel/test_listener_micro_batching.py of the reference replay event
traces through the policies; here seeded random traces drive both the oracle
and the GPU path from identical starting state."""
from __future__ import annotations

import copy
import random

import pytest
import torch

from oracle.packer_ref import TickFrame, order_ready_heads, snapshot_ready_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dispatch(pkg):
    from gemma4_omni_b200 import dispatch as d
    return d


def _trace(rng: random.Random, n_sessions: int, ticks: int):
    regs = [f"s{rng.randrange(10**6):06d}-{i}" for i in range(n_sessions)]
    rng.shuffle(regs)
    ingress = {sid: [] for sid in regs}
    for sid in regs:
        t = rng.randrange(0, 4) * 80_000_000
        for f in range(rng.randrange(0, ticks + 2)):
            t += rng.choice([80_000_000, 80_000_000, 79_000_000, 95_000_000, 0])
            ingress[sid].append(TickFrame(sid, f, t + rng.randrange(-3_000_000, 3_000_000)))
    return regs, ingress


@pytest.mark.parametrize("n_sessions,seed", [(0, 1), (1, 2), (7, 3), (300, 4), (1500, 5), (5000, 6)])
def test_snapshot_matches_oracle_over_ticks(dispatch, n_sessions, seed):
    rng = random.Random(seed)
    regs, ingress = _trace(rng, n_sessions, ticks=8)
    ing_gpu, ing_ref = copy.deepcopy(ingress), copy.deepcopy(ingress)
    def_gpu, def_ref = {}, {}
    for tick in range(10):
        paused = {sid for sid in regs if rng.random() < 0.1}
        deadline = tick * 80_000_000 + 40_000_000
        ref = snapshot_ready_rows(regs, paused, ing_ref, def_ref, deadline)
        got = dispatch.snapshot_ready_rows(regs, paused, ing_gpu, def_gpu, deadline)
        assert [(f.session_id, f.frame_id) for f in got] == [(f.session_id, f.frame_id) for f in ref]
        assert {k: (v.frame_id, v.enqueue_ns) for k, v in def_gpu.items()} == \
               {k: (v.frame_id, v.enqueue_ns) for k, v in def_ref.items()}
        assert {k: [f.frame_id for f in q] for k, q in ing_gpu.items()} == \
               {k: [f.frame_id for f in q] for k, q in ing_ref.items()}


def test_snapshot_all_paused_and_all_late(dispatch):
    regs = ["a", "b", "c"]
    ingress = {s: [TickFrame(s, 0, 100)] for s in regs}
    assert dispatch.snapshot_ready_rows(regs, set(regs), ingress, {}, 1000) == []
    assert all(len(q) == 1 for q in ingress.values())
    deferred = {}
    assert dispatch.snapshot_ready_rows(regs, set(), ingress, deferred, 50) == []
    assert sorted(deferred) == regs and all(not q for q in ingress.values())
    rows = dispatch.snapshot_ready_rows(regs, set(), ingress, deferred, 150)
    assert [f.session_id for f in rows] == regs and deferred == {}


def _heads(rng: random.Random, n: int, dup_orders: bool):
    heads = []
    for i in range(n):
        ready = rng.choice([0, 1_000, 2_000, 2_000, 5_000_000]) + rng.randrange(0, 3) * 1_000
        order = rng.randrange(0, 4) if dup_orders else rng.randrange(10**12)
        heads.append((ready, order, f"sess-{rng.randrange(10**6)}-{i}"))
    return heads


@pytest.mark.parametrize("n,seed,dup", [(0, 1, False), (1, 2, False), (2, 3, True), (37, 4, True),
                                        (1000, 5, False), (4097, 6, True), (8192, 7, False)])
def test_order_matches_oracle(dispatch, n, seed, dup):
    rng = random.Random(seed)
    heads = _heads(rng, n, dup)
    for now in (0, 1_500, 2_500_000, 10_000_000):
        for coalesce in (0, 2_000_000):
            for registered in (n, n + 3):
                ref = order_ready_heads(heads, now, coalesce, registered)
                got = dispatch.order_ready_heads(heads, now, coalesce, registered)
                assert got == ref, (now, coalesce, registered)


def test_order_single_head_coalesce_window(dispatch):
    heads = [(1_000, 5, "only")]
    assert dispatch.order_ready_heads(heads, 1_500, 2_000_000, 3) == ([], None)
    assert dispatch.order_ready_heads(heads, 2_001_000, 2_000_000, 3) == (heads, "coalesce_deadline")
    assert dispatch.order_ready_heads(heads, 2_001_000, 2_000_000, 1) == (heads, "batch_full")
    assert dispatch.order_ready_heads(heads, 500, 0, 1) == ([], None)  # not ready yet


def test_order_rejects_more_than_capacity(dispatch):
    heads = [(0, i, f"s{i}") for i in range(dispatch.MAX_SORT_HEADS + 1)]
    with pytest.raises(RuntimeError):
        dispatch.order_ready_heads(heads, 0, 0, len(heads))


def test_order_replays_reference_coordinator_golden(dispatch):
    """lb_order_ready_heads through the reference ListenerMicrobatchCoordinator's
    take_ready trace (tests/golden/packer.npz ``coordinator``): every dispatched
    row order and reason bit-exact."""
    import json
    from pathlib import Path

    import numpy as np
    from helpers import replay_coordinator

    g = json.loads(str(np.load(Path(__file__).resolve().parent / "golden" / "packer.npz")["coordinator"]))
    assert replay_coordinator(g, dispatch.order_ready_heads) > 50
