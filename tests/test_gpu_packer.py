"""GPU packer (slot policy, commit / abort / rollback / reset) vs the reference.

Bit-exact: slot ids, reasons and the committed cursor directory must equal the
reference's StreamingConformerAudioTower bookkeeping (golden trace) and the
oracle restatement (random traces).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import HandleBook
from oracle import packer_ref

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
REASONS = ("continue", "reset", "gap_or_cursor_mismatch", "identity_reset")


@pytest.fixture(scope="module")
def small_weights(pkg):
    from gemma4_omni_b200 import synthetic
    from gemma4_omni_b200.config import SMALL
    return synthetic.synthetic_tower_weights(SMALL, 3), synthetic.synthetic_film_weights(SMALL, 4)


def engine(small_weights, sessions, handles, rows=None):
    from gemma4_omni_b200 import runtime
    from gemma4_omni_b200.config import SMALL
    eng = runtime.ListenerEngine(SMALL, max_sessions=sessions, max_handles=handles, max_rows=rows)
    eng.load_weights(*small_weights)
    return eng


def step_rows(eng, book, rows):
    h, k, f, q = book.arrays(rows)
    eng.pack(h, k, f, q)
    eng.step(torch.zeros(len(rows), 8, 128, device="cuda"), kind=1, want_raw=False)
    return eng.read_rows(len(rows))


def committed(eng, book):
    slot, key, ef, es = eng.read_handles()
    inv_key = {v: k for k, v in book.keys.items()}
    out = []
    for sid, h in book.handles.items():
        if slot[h] >= 0 and ef[h] >= 0:
            gen, ep = inv_key[int(key[h])]
            out.append((sid, gen, ep, int(ef[h]), int(es[h])))
    return sorted(out)


def test_packer_replays_reference_slot_trace(small_weights):
    """Also checks lb_get_counters against the trace: calls, rows per reason,
    committed rows and the status history of the exhausted-bank steps."""
    g = np.load(GOLD / "packer.npz")
    S = int(g["max_sessions"])
    eng = engine(small_weights, S, 16, rows=S)
    book = HandleBook()
    want = {"packs": 0, "steps": 0, "commits": 0, "aborts": 0, "resets": 0, "rows_stepped": 0,
            "rows_committed": 0}
    reasons_seen = dict.fromkeys(REASONS, 0)
    for ev in json.loads(str(g["events"])):
        if ev["kind"] in ("reset", "reset_session"):
            want["resets"] += int(ev["kind"] == "reset_session" or ev["sid"] in book.handles)
        elif "error" in ev:
            want.update(packs=want["packs"] + 1, steps=want["steps"] + 1, aborts=want["aborts"] + 1,
                        rows_stepped=want["rows_stepped"] + len(ev["rows"]))
        else:
            n = len(ev["rows"])
            want.update(packs=want["packs"] + 1, steps=want["steps"] + 1, rows_stepped=want["rows_stepped"] + n)
            for r in ev["reasons"]:
                reasons_seen[r] += 1
            if ev["action"] == "commit":
                want.update(commits=want["commits"] + 1, rows_committed=want["rows_committed"] + n)
            else:
                want["aborts"] += 1
        if ev["kind"] == "reset":
            if ev["sid"] in book.handles:
                eng.reset_handle(book.handle(ev["sid"]))
        elif ev["kind"] == "reset_session":
            eng.reset_slot(ev["slot"])
        else:
            rows = [tuple(r) for r in ev["rows"]]
            if "error" in ev:
                eng.clear_status()
                step_rows(eng, book, rows)
                assert eng.status() & 2  # LB_DEV_SLOT_EXHAUSTED
                eng.abort()
                eng.clear_status()
                continue
            slots, reasons = step_rows(eng, book, rows)
            assert list(slots) == ev["slots"]
            assert [REASONS[r] for r in reasons] == ev["reasons"]
            eng.commit() if ev["action"] == "commit" else eng.abort()
        assert committed(eng, book) == sorted(tuple(x) for x in ev["committed"])
    assert eng.status() == 0
    ctr = eng.counters()
    for k, v in want.items():
        assert ctr[k] == v, (k, ctr[k], v)
    # rows of the exhausted-bank packs are counted by reason too (they resolved)
    assert ctr["rows_continue"] >= reasons_seen["continue"]
    assert ctr["rows_identity_reset"] >= reasons_seen["identity_reset"]
    assert ctr["rows_gap_or_cursor_mismatch"] >= reasons_seen["gap_or_cursor_mismatch"]
    assert sum(ctr[f"rows_{r}"] for r in REASONS) == want["rows_stepped"]
    assert ctr["stale_commits"] == 0 and ctr["status"] == 0
    assert ctr["status_history"] & 2  # the exhausted-bank steps' LB_DEV_SLOT_EXHAUSTED
    eng.close()


def test_packer_random_traces_match_oracle_policy(small_weights):
    rng = np.random.default_rng(11)
    S, H = 160, 400
    eng = engine(small_weights, S, H, rows=128)
    pol = packer_ref.SlotPolicy(S)
    book = HandleBook()
    gen = {}
    nxt = {}
    sids = [f"u{i}" for i in range(H)]
    for step in range(80):
        if rng.random() < 0.15:
            sid = sids[rng.integers(0, H)]
            pol.reset(sid)
            eng.reset_handle(book.handle(sid))
            continue
        n = int(rng.integers(1, 128))
        chosen = [sids[i] for i in rng.choice(H, size=n, replace=False)]
        rows = []
        for sid in chosen:
            u = rng.random()
            if u < 0.05:
                gen[sid] = gen.get(sid, 0) + 1
                nxt[sid] = 0
            elif u < 0.1:
                nxt[sid] = nxt.get(sid, 0) + 3
            rows.append((sid, gen.get(sid, 0), f"e{gen.get(sid, 0)}", nxt.get(sid, 0), nxt.get(sid, 0)))
        try:
            p = pol.prepare(rows)
        except RuntimeError:
            eng.clear_status()
            step_rows(eng, book, rows)
            assert eng.status() & 2
            eng.abort()
            eng.clear_status()
            # free capacity for the rest of the trace
            for sid in list({k[0] for k in pol.slots_by_key})[: S // 2]:
                pol.reset(sid)
                eng.reset_handle(book.handle(sid))
            continue
        slots, reasons = step_rows(eng, book, rows)
        assert list(slots) == p.slots
        assert [REASONS[r] for r in reasons] == p.reasons
        if rng.random() < 0.9:
            pol.commit()
            eng.commit()
            for sid, g_, e_, f_, q_ in rows:
                nxt[sid] = f_ + 1
        else:
            pol.abort()
            eng.abort()
        assert committed(eng, book) == sorted(pol.committed_positions)
    assert eng.status() == 0
    eng.close()


def test_duplicate_handle_and_stale_commit_fail_closed(small_weights):
    eng = engine(small_weights, 8, 8)
    book = HandleBook()
    step_rows(eng, book, [("a", 0, "e", 0), ("b", 0, "e", 0)])
    eng.commit()
    before = committed(eng, book)
    # duplicate session in one batch -> device status, nothing committed
    h, k, f, q = book.arrays([("a", 0, "e", 1), ("a", 0, "e", 1)])
    eng.pack(h, k, f, q)
    eng.step(torch.zeros(2, 8, 128, device="cuda"), kind=1)
    assert eng.status() & 4
    eng.commit()
    assert committed(eng, book) == before
    eng.clear_status()
    # stale cursor between pack and commit -> all-or-nothing refusal
    step_rows(eng, book, [("a", 0, "e", 1), ("b", 0, "e", 1)])
    eng.debug_set_expected(book.handle("b"), 99, 99)
    eng.commit()
    assert eng.status() & 16
    eng.debug_set_expected(book.handle("b"), 1, 1)
    assert committed(eng, book) == before
    eng.clear_status()
    # rollback restores the state before the last commit
    step_rows(eng, book, [("a", 0, "e", 1), ("b", 0, "e", 1), ("c", 0, "e", 0)])
    eng.commit()
    assert committed(eng, book) == [("a", 0, "e", 2, 2), ("b", 0, "e", 2, 2), ("c", 0, "e", 1, 1)]
    eng.rollback()
    assert committed(eng, book) == before
    slots, reasons = step_rows(eng, book, [("c", 0, "e", 0), ("a", 0, "e", 1)])
    assert [REASONS[r] for r in reasons] == ["identity_reset", "continue"]
    eng.abort()
    assert eng.status() == 0
    eng.close()


def test_state_machine_rejects_out_of_order_calls(small_weights):
    from gemma4_omni_b200 import _lib
    eng = engine(small_weights, 4, 4)
    with pytest.raises(_lib.ListenerLibError):
        eng.commit()  # nothing stepped
    book = HandleBook()
    h, k, f, q = book.arrays([("a", 0, "e", 0)])
    eng.pack(h, k, f, q)
    with pytest.raises(_lib.ListenerLibError):
        eng.pack(h, k, f, q)  # previous batch neither committed nor aborted
    with pytest.raises(_lib.ListenerLibError):
        eng.reset_handle(0)  # not while a batch is prepared
    eng.abort()
    eng.close()


def test_reset_handles_releases_many_at_once(small_weights):
    """lb_reset_handles_async == one lb_reset_handle_async per handle."""
    eng = engine(small_weights, 8, 16, rows=8)
    ref = engine(small_weights, 8, 16, rows=8)
    book = HandleBook()
    rows = [(f"s{i}", 0, "e", 0) for i in range(6)]
    for e in (eng, ref):
        step_rows(e, book, rows)
        e.commit()
    gone = [1, 4, 5]
    eng.reset_handles(torch.tensor([book.handle(f"s{i}") for i in gone], dtype=torch.int32, device="cuda"))
    for i in gone:
        ref.reset_handle(book.handle(f"s{i}"))
    assert all((a == b).all() for a, b in zip(eng.read_handles(), ref.read_handles()))
    nxt = [(f"s{i}", 0, "e", 1) for i in (0, 2, 3)] + [("t0", 0, "e", 0), ("t1", 0, "e", 0)]
    got = step_rows(eng, book, nxt)
    want = step_rows(ref, book, nxt)
    assert list(got[0]) == list(want[0]) and list(got[1]) == list(want[1])
    assert sorted(got[0][3:]) == [1, 4]  # the lowest freed slots
    bad = torch.tensor([99], dtype=torch.int32, device="cuda")
    eng.abort()
    eng.reset_handles(bad)
    assert eng.status() & 8  # LB_DEV_BAD_HANDLE
    eng.close()
    ref.close()
