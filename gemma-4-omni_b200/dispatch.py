"""Tick-level row selection on the GPU: the dispatcher snapshot and the
coordinator's head ordering that run in front of the packer.

``snapshot_ready_rows`` has the argument meaning and the side effects of
``SharedListenerTickDispatcher._snapshot_ready_rows``
(duplex_kernel/shared_listener_scheduler.py:486-535): sessions are walked in
registration order, paused sessions are skipped, a session's deferred frame is
taken before the head of its ingress queue (which is popped), a frame enqueued
after the tick deadline is kept as the session's deferred frame for the next
tick, and every other frame becomes a row, in registration order.

``order_ready_heads`` restates ``ListenerMicrobatchCoordinator.
_candidate_heads_locked`` / ``_take_ready_locked``
(duplex_kernel/listener_microbatch.py:170-201): heads with ``ready_at_ns <=
now`` sorted by ``(ready_at_ns, submission_order, session_id)``; a lone ready
head waits for the coalesce window; the reason is ``batch_full``,
``multiple_ready`` or ``coalesce_deadline``.

The decisions run in one CUDA kernel each (``lb_snapshot_ready_rows``,
``lb_order_ready_heads``); these wrappers only move the per-session fields to
the device and apply the returned pops and deferrals to the caller's queues.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

REASONS = {0: None, 1: "batch_full", 2: "multiple_ready", 3: "coalesce_deadline"}
MAX_SORT_HEADS = 8192


@dataclass
class TickFrame:
    """An ingress frame: the fields the snapshot reads."""
    session_id: str
    frame_id: int
    enqueue_ns: int


def _dev(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def snapshot_ready_rows(registrations: list[str], paused: set[str], ingress: dict[str, list],
                        deferred: dict[str, object], deadline_ns: int, *,
                        device: str | torch.device = "cuda", stream=None) -> list:
    """Rows of one tick (frames in registration order).

    ``ingress`` maps session id -> FIFO list of frames (``frame_id``,
    ``enqueue_ns``); consumed heads are popped.  ``deferred`` maps session id ->
    the frame held back from an earlier tick and is updated in place.
    """
    lib = _lib.load()
    device = torch.device(device)
    n = len(registrations)
    if len(set(registrations)) != n:
        raise ValueError("a session is registered twice")
    p = np.zeros(n, np.uint8)
    dv = np.zeros(n, np.uint8)
    df = np.zeros(n, np.int64)
    de = np.zeros(n, np.int64)
    hv = np.zeros(n, np.uint8)
    hf = np.zeros(n, np.int64)
    he = np.zeros(n, np.int64)
    for i, sid in enumerate(registrations):
        p[i] = sid in paused
        f = deferred.get(sid)
        if f is not None:
            dv[i], df[i], de[i] = 1, int(f.frame_id), int(f.enqueue_ns)
        q = ingress.get(sid)
        if q:
            hv[i], hf[i], he[i] = 1, int(q[0].frame_id), int(q[0].enqueue_ns)
    t = {k: _dev(v, device) for k, v in dict(p=p, dv=dv, df=df, de=de, hv=hv, hf=hf, he=he).items()}
    rows = torch.empty(max(n, 1), dtype=torch.int32, device=device)
    row_frame = torch.empty(max(n, 1), dtype=torch.int64, device=device)
    popped = torch.empty(max(n, 1), dtype=torch.uint8, device=device)
    n_rows = torch.zeros(1, dtype=torch.int32, device=device)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    rc = lib.lb_snapshot_ready_rows(n, t["p"].data_ptr(), t["dv"].data_ptr(), t["df"].data_ptr(),
                                    t["de"].data_ptr(), t["hv"].data_ptr(), t["hf"].data_ptr(),
                                    t["he"].data_ptr(), int(deadline_ns), rows.data_ptr(),
                                    row_frame.data_ptr(), popped.data_ptr(), n_rows.data_ptr(),
                                    s.cuda_stream)
    _lib.check("lb_snapshot_ready_rows", rc)
    s.synchronize()
    k = int(n_rows.item())
    rows_h = rows[:k].cpu().numpy()
    popped_h = popped[:n].cpu().numpy()
    dv_h, df_h = t["dv"].cpu().numpy(), t["df"].cpu().numpy()
    # frames the kernel selected, taken from the caller's own objects
    held = {sid: deferred.get(sid) for sid in registrations}
    heads = {sid: ingress[sid][0] for i, sid in enumerate(registrations) if popped_h[i]}
    for i, sid in enumerate(registrations):
        if popped_h[i]:
            ingress[sid].pop(0)
    out = []
    for i in rows_h:
        sid = registrations[int(i)]
        out.append(heads[sid] if sid in heads else held[sid])
    for i, sid in enumerate(registrations):
        if sid in paused:
            continue
        if dv_h[i]:
            frame = heads.get(sid, held.get(sid))
            if frame is None or int(frame.frame_id) != int(df_h[i]):
                raise RuntimeError(f"deferred frame mismatch for {sid}")
            deferred[sid] = frame
        else:
            deferred.pop(sid, None)
    return out


def order_ready_heads(heads: list[tuple[int, int, str]], now_ns: int, coalesce_ns: int,
                      registered: int, *, device: str | torch.device = "cuda",
                      stream=None) -> tuple[list[tuple[int, int, str]], str | None]:
    """heads: (ready_at_ns, submission_order, session_id) of every candidate
    head.  Returns (dispatched heads in order, reason), or ([], None)."""
    lib = _lib.load()
    device = torch.device(device)
    n = len(heads)
    if n > MAX_SORT_HEADS:
        raise RuntimeError(f"at most {MAX_SORT_HEADS} candidate heads per tick")
    rank_of = {sid: r for r, sid in enumerate(sorted({h[2] for h in heads}))}
    ra = _dev(np.array([h[0] for h in heads] or [0], np.int64), device)
    so = _dev(np.array([h[1] for h in heads] or [0], np.int64), device)
    rk = _dev(np.array([rank_of[h[2]] for h in heads] or [0], np.int32), device)
    perm = torch.empty(max(n, 1), dtype=torch.int32, device=device)
    cnt = torch.zeros(2, dtype=torch.int32, device=device)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    rc = lib.lb_order_ready_heads(n, ra.data_ptr(), so.data_ptr(), rk.data_ptr(), int(now_ns),
                                  int(coalesce_ns), int(registered), perm.data_ptr(),
                                  cnt[0:1].data_ptr(), cnt[1:2].data_ptr(), s.cuda_stream)
    _lib.check("lb_order_ready_heads", rc)
    s.synchronize()
    count, reason = (int(v) for v in cnt.cpu().tolist())
    order = perm[:count].cpu().tolist()
    return [heads[i] for i in order], REASONS[reason]
