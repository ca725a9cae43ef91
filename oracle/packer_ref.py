"""Pure-Python restatement of the listener packing/indexing rules (test oracle).

Three integer policies decide, every 80 ms tick, which sessions form the batch,
in which row order, and which persistent cache slot each row uses:

1. ``snapshot_ready_rows`` -- SharedListenerTickDispatcher._snapshot_ready_rows
   (duplex_kernel/shared_listener_scheduler.py:486-535): registration order,
   paused sessions skipped, one frame per session, a frame enqueued after the
   tick deadline is deferred to the next tick.
2. ``order_ready_heads`` -- ListenerMicrobatchCoordinator._candidate_heads_locked /
   _take_ready_locked (duplex_kernel/listener_microbatch.py:170-201): heads not in
   flight, sorted by (ready_at_ns, submission_order, session_id); a lone head
   waits for the coalesce window.
3. ``SlotPolicy`` -- StreamingConformerAudioTower.prepare_batch slot mapping and
   its commit/abort/rollback/reset bookkeeping
   (duplex_kernel/streaming_conformer.py:418-451, 571-615, 904-967).

TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class TickFrame:
    session_id: str
    frame_id: int
    enqueue_ns: int


def snapshot_ready_rows(registrations: list[str], paused: set[str], ingress: dict[str, list[TickFrame]],
                        deferred: dict[str, TickFrame], deadline_ns: int) -> list[TickFrame]:
    """Rows of one tick; mutates ``ingress`` (pops heads) and ``deferred``."""
    rows = []
    for sid in registrations:
        if sid in paused:
            continue
        frame = deferred.pop(sid, None)
        if frame is None:
            queue = ingress.get(sid, [])
            if not queue:
                continue
            frame = queue.pop(0)
        if frame.enqueue_ns > deadline_ns:
            deferred[sid] = frame
            continue
        rows.append(frame)
    return rows


def order_ready_heads(heads: list[tuple[int, int, str]], now_ns: int, coalesce_ns: int,
                      registered: int) -> tuple[list[tuple[int, int, str]], str | None]:
    """heads: (ready_at_ns, submission_order, session_id).  Returns (rows, reason)."""
    ready = sorted((h for h in heads if h[0] <= now_ns), key=lambda h: (h[0], h[1], h[2]))
    if not ready:
        return [], None
    if len(ready) == 1 and now_ns < ready[0][0] + coalesce_ns:
        return [], None
    if len(ready) == registered:
        reason = "batch_full"
    elif len(ready) >= 2:
        reason = "multiple_ready"
    else:
        reason = "coalesce_deadline"
    return ready, reason


Key = tuple  # (session_id, generation_id, state_epoch_id)


@dataclass
class Prepared:
    keys: list
    cursors: list  # (frame_id, sequence_position)
    slots: list[int]
    reasons: list[str]
    replacing: list
    expected_before: list


@dataclass
class SlotPolicy:
    max_sessions: int
    slots_by_key: dict = field(default_factory=dict)
    expected: dict = field(default_factory=dict)
    key_by_slot: dict = field(default_factory=dict)
    active: Prepared | None = None
    last_rollback: tuple | None = None

    def prepare(self, rows: list[tuple[str, int, str, int, int]]) -> Prepared:
        """rows: (session_id, generation_id, epoch_id, frame_id, sequence_position)."""
        if self.active is not None:
            raise RuntimeError("previous streaming audio batch has not committed or aborted")
        keys = [(r[0], r[1], r[2]) for r in rows]
        if len(set(keys)) != len(rows) or len({r[0] for r in rows}) != len(rows):
            raise ValueError("a streaming audio batch requires distinct session identities")
        unavailable = set(self.key_by_slot)
        slots, reasons, replacing, expected_before = [], [], [], []
        for r, key in zip(rows, keys):
            if key in self.slots_by_key:
                slot = self.slots_by_key[key]
                rep = None
                exp = self.expected.get(key)
                if exp is None:
                    reason = "reset"
                elif exp == (r[3], r[4]):
                    reason = "continue"
                else:
                    reason = "gap_or_cursor_mismatch"
            else:
                old = [k for k in self.slots_by_key if k[0] == r[0]]
                if old:
                    rep = old[0]
                    slot = self.slots_by_key[rep]
                else:
                    rep = None
                    free = next((c for c in range(self.max_sessions) if c not in unavailable), None)
                    if free is None:
                        raise RuntimeError(f"streaming audio session bank exhausted ({self.max_sessions} sessions)")
                    slot = free
                    unavailable.add(slot)
                exp = None
                reason = "identity_reset"
            slots.append(slot)
            reasons.append(reason)
            replacing.append(rep)
            expected_before.append(exp)
        if len(set(slots)) != len(rows):
            raise RuntimeError("streaming audio batch maps multiple rows to one persistent state slot")
        self.active = Prepared(keys, [(r[3], r[4]) for r in rows], slots, reasons, replacing, expected_before)
        return self.active

    def commit(self) -> None:
        batch = self.active
        if batch is None:
            raise RuntimeError("streaming audio transaction is no longer active")
        self.active = None
        for key, exp in zip(batch.keys, batch.expected_before):
            if self.expected.get(key) != exp:
                raise RuntimeError("cursor changed before streaming commit")
        old = [(self.slots_by_key.get(k), self.expected.get(k), self.key_by_slot.get(s), rep,
                self.slots_by_key.get(rep) if rep is not None else None,
                self.expected.get(rep) if rep is not None else None)
               for k, s, rep in zip(batch.keys, batch.slots, batch.replacing)]
        for key, slot, rep, cur in zip(batch.keys, batch.slots, batch.replacing, batch.cursors):
            if rep is not None:
                self.slots_by_key.pop(rep, None)
                self.expected.pop(rep, None)
            self.slots_by_key[key] = slot
            self.key_by_slot[slot] = key
            self.expected[key] = (cur[0] + 1, cur[1] + 1)
        self.last_rollback = (batch, old)

    def abort(self) -> None:
        if self.active is None:
            raise RuntimeError("streaming audio transaction is no longer active")
        self.active = None

    def rollback(self) -> None:
        batch, old = self.last_rollback
        for key, slot, o in zip(batch.keys, batch.slots, old):
            old_slot, old_pos, old_key_at_slot, rep, rep_slot, rep_pos = o
            self.slots_by_key.pop(key, None)
            self.expected.pop(key, None)
            if self.key_by_slot.get(slot) == key:
                self.key_by_slot.pop(slot, None)
            if old_slot is not None:
                self.slots_by_key[key] = old_slot
            if old_pos is not None:
                self.expected[key] = old_pos
            if old_key_at_slot is not None:
                self.key_by_slot[slot] = old_key_at_slot
            if rep is not None:
                if rep_slot is not None:
                    self.slots_by_key[rep] = rep_slot
                if rep_pos is not None:
                    self.expected[rep] = rep_pos
        self.last_rollback = None

    def reset(self, session_id: str, generation_id=None, epoch_id=None) -> list[int]:
        if self.active is not None:
            raise RuntimeError("cannot reset streaming audio state while a batch is prepared")
        selected = [k for k in self.slots_by_key if k[0] == session_id
                    and (generation_id is None or k[1] == generation_id)
                    and (epoch_id is None or k[2] == epoch_id)]
        freed = []
        for key in selected:
            slot = self.slots_by_key.pop(key)
            self.expected.pop(key, None)
            self.key_by_slot.pop(slot, None)
            freed.append(slot)
        return freed

    def reset_session(self, slot: int) -> None:
        if isinstance(slot, bool) or not isinstance(slot, int):
            raise TypeError("slot_idx must be an integer")
        if slot < 0 or slot >= self.max_sessions:
            raise IndexError(f"slot_idx {slot} is outside [0, {self.max_sessions})")
        if self.active is not None:
            raise RuntimeError("cannot reset a streaming audio slot while a batch is prepared")
        key = self.key_by_slot.pop(slot, None)
        if key is not None:
            self.slots_by_key.pop(key, None)
            self.expected.pop(key, None)

    @property
    def committed_positions(self):
        return tuple(sorted((k[0], k[1], k[2], e[0], e[1]) for k, e in self.expected.items()))
