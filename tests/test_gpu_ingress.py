"""GPU-resident ingress (lb_ingress_*) vs the oracle of the reference's tick
snapshot (SharedListenerTickDispatcher._snapshot_ready_rows,
shared_listener_scheduler.py:486-535) on multi-tick traces with joins,
leaves, pauses and deadline deferrals: rows (session, frame) bit-exact and
every row's PCM identical to the frame submitted."""
from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from oracle.packer_ref import TickFrame, snapshot_ready_rows

pytestmark = pytest.mark.gpu


def _pcm(sid: str, frame: int) -> np.ndarray:
    rng = np.random.default_rng([hash(sid) % (1 << 31), frame])
    return rng.standard_normal(1280).astype(np.float32)


@pytest.mark.parametrize("seed,n_sessions", [(1, 5), (2, 60), (3, 700)])
def test_ingress_matches_oracle_snapshot(pkg, seed, n_sessions):
    from gemma4_omni_b200.ingress import GpuTickIngress

    rng = random.Random(seed)
    ing = GpuTickIngress(max_sessions=n_sessions + 8, ring_frames=8)
    regs: list[str] = []
    paused: set[str] = set()
    queues: dict[str, list] = {}
    deferred: dict = {}
    next_frame: dict[str, int] = {}
    payload: dict[tuple[str, int], np.ndarray] = {}
    counter = 0
    tick_ns = 80_000_000
    for tick in range(14):
        deadline = (tick + 1) * tick_ns
        # session events: joins, leaves, pauses, resumes
        if tick == 0 or rng.random() < 0.5:
            for _ in range(rng.randrange(1, 4) if tick else n_sessions):
                sid = f"s{counter}"
                counter += 1
                regs.append(sid)
                queues[sid] = []
                next_frame[sid] = 0
                ing.register_session(sid, handle=counter)
        for sid in list(regs):
            u = rng.random()
            if u < 0.03:
                regs.remove(sid)
                queues.pop(sid)
                deferred.pop(sid, None)
                paused.discard(sid)
                ing.unregister_session(sid)
            elif u < 0.08 and sid not in paused:
                paused.add(sid)
                ing.pause_session(sid)
            elif u < 0.12 and sid in paused:
                paused.discard(sid)
                ing.resume_session(sid)
        # arrivals: mostly one frame, sometimes none or two; some late
        for sid in regs:
            held = len(queues[sid]) + (sid in deferred)
            for _ in range(rng.choice([0, 1, 1, 1, 2])):
                if held >= 7:  # the ring holds 8 frames: keep the trace within it
                    break
                f = next_frame[sid]
                next_frame[sid] += 1
                enq = deadline - tick_ns // 2 + rng.choice([0, 0, 0, tick_ns])  # a quarter arrive after the deadline
                pcm = _pcm(sid, f)
                payload[(sid, f)] = pcm
                queues[sid].append(TickFrame(sid, f, enq))
                ing.submit(sid, f, enq, pcm)
                held += 1
        ref = snapshot_ready_rows(regs, paused, queues, deferred, deadline)
        rows, pcm, handles, frames = ing.dispatch_tick(deadline)
        assert rows == [(r.session_id, r.frame_id) for r in ref], tick
        got = pcm.cpu().numpy()
        for i, (sid, f) in enumerate(rows):
            np.testing.assert_array_equal(got[i], payload[(sid, f)])
        assert frames.cpu().tolist() == [f for _, f in rows]
        assert handles.cpu().tolist() == [int(sid[1:]) + 1 for sid, _ in rows]
    assert ing.status() == 0
    ing.close()


def test_ingress_row_cap_and_ring_overflow(pkg):
    from gemma4_omni_b200 import _lib
    from gemma4_omni_b200.ingress import GpuTickIngress

    ing = GpuTickIngress(max_sessions=8, ring_frames=2, max_rows=3)
    for i in range(5):
        ing.register_session(f"c{i}", handle=i)
        ing.submit(f"c{i}", 0, 0, _pcm(f"c{i}", 0))
    rows, *_ = ing.dispatch_tick(10)
    assert rows == [("c0", 0), ("c1", 0), ("c2", 0)]  # the first max_rows in registration order
    rows, *_ = ing.dispatch_tick(20)
    assert rows == [("c3", 0), ("c4", 0)]              # the rest waited one tick
    for f in (1, 2, 3):
        ing.submit("c0", f, 0, _pcm("c0", f))
    ing.dispatch_tick(-1)  # nothing ready: the frames stay queued
    assert ing.status() & _lib.DEV_INGRESS_OVERFLOW     # the third frame found the 2-frame ring full
    rows, *_ = ing.dispatch_tick(30)
    assert rows == [("c0", 1)]
    ing.close()


def test_ingress_feeds_the_listener_step(pkg):
    """Ingress rows -> pack -> PCM step equals the same step on host-supplied PCM."""
    from gemma4_omni_b200 import _lib, runtime, synthetic
    from gemma4_omni_b200.config import SMALL
    from gemma4_omni_b200.ingress import GpuTickIngress

    def engine():
        e = runtime.ListenerEngine(SMALL, max_sessions=8, weight_format=0)
        e.load_weights(synthetic.synthetic_tower_weights(SMALL, 5, nontrivial=True),
                       synthetic.synthetic_film_weights(SMALL, 6, nontrivial=True))
        return e

    a, b = engine(), engine()
    ing = GpuTickIngress(max_sessions=8, ring_frames=4)
    for i in range(4):
        ing.register_session(f"u{i}", handle=i)
    for t in range(3):
        host = []
        for i in (2, 0, 3, 1):  # arrival order differs from registration order
            pcm = synthetic.session_audio(2, i, 1, first_frame=t, total_frames=3)[0]
            ing.submit(f"u{i}", t, t, pcm)
        rows, pcm_dev, handles, frames = ing.dispatch_tick(t)
        assert [r[0] for r in rows] == ["u0", "u1", "u2", "u3"]
        expected = np.stack([synthetic.session_audio(2, i, 1, first_frame=t, total_frames=3)[0] for i in range(4)])
        # the gathered step input is the host PCM, bit for bit, in registration order
        assert torch.equal(pcm_dev.cpu(), torch.from_numpy(expected))
        assert handles.tolist() == [0, 1, 2, 3] and frames.tolist() == [t] * 4
        keys = torch.zeros(len(rows), dtype=torch.int64, device="cuda")
        a.pack(handles.contiguous(), keys, frames.contiguous(), frames.contiguous())
        out_a = a.step(pcm_dev.contiguous(), kind=_lib.LB_INPUT_PCM)
        a.commit()
        host = np.stack([synthetic.session_audio(2, i, 1, first_frame=t, total_frames=3)[0] for i in range(4)])
        hh = torch.arange(4, dtype=torch.int32, device="cuda")
        ff = torch.full((4,), t, dtype=torch.int64, device="cuda")
        b.pack(hh, keys, ff, ff.clone())
        out_b = b.step(torch.from_numpy(host).cuda(), kind=_lib.LB_INPUT_PCM)
        b.commit()
        # the same step on the same input; split-K GEMMs reduce more than two fp32
        # partial sums with atomics, so the two runs may differ in the last bits
        torch.testing.assert_close(out_a["soft"].float(), out_b["soft"].float(), rtol=1e-2, atol=1e-2)
    assert a.status() == 0 and ing.status() == 0
    ing.close()
    a.close()
    b.close()
