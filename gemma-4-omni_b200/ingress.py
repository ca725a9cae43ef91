"""GPU-resident listener ingress: the fixed-grid dispatcher's queues on the device.

``GpuTickIngress`` keeps the session bookkeeping of the reference's
``SharedListenerTickDispatcher`` (duplex_kernel/shared_listener_scheduler.py:
``register_session``, ``pause_session``, ``unregister_session`` and the
per-tick ``_snapshot_ready_rows`` :486-535) but holds every session's queued
PCM frames in a device ring (``lb_ingress_*`` in include/listener_b200.h).
Per tick the host hands over only what changed -- the session events and the
frames that arrived, one host->device copy of each -- and the tick kernel
selects the rows (registration order, paused sessions skipped, frames enqueued
after the deadline held for the next tick), consumes them and gathers their
PCM into a ``[rows, 1280]`` device tensor that ``ListenerEngine.step`` takes
as its input; the rows' directory handles and frame ids come back as device
tensors for ``ListenerEngine.pack``.  The host does no per-session work per
tick: only the row count and the row list (for the caller's own bookkeeping)
are read back.

Differences from the reference, by design: each session's queue is a ring of
``ring_frames`` frames (a frame that finds it full is refused and flagged,
where the reference's queue is unbounded), and one tick emits at most
``max_rows`` rows (ready frames past that wait a tick, in registration order).
"""
from __future__ import annotations

import ctypes
from typing import Hashable

import numpy as np
import torch

from . import _lib

PCM_SAMPLES = 1280


class GpuTickIngress:
    """Device-resident ingress queues and tick snapshot for one GPU."""

    def __init__(self, *, max_sessions: int, ring_frames: int = 8, max_rows: int | None = None,
                 device: torch.device | str | None = None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("GpuTickIngress runs on a CUDA device (no CPU fallback)")
        self.max_sessions = int(max_sessions)
        self.max_rows = int(max_rows or max_sessions)
        self.ring_frames = int(ring_frames)
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check("lb_ingress_create", self.lib.lb_ingress_create(self.max_sessions, self.ring_frames,
                                                                       self.max_rows, ctypes.byref(h)))
        self._h = h
        self._index: dict[Hashable, int] = {}   # session id -> ring index
        self._ids: dict[int, Hashable] = {}
        self._free = list(range(self.max_sessions - 1, -1, -1))
        self._released: list[int] = []          # freed this tick: reusable after the next flush
        self._events: list[tuple[int, int, int]] = []
        self._arrivals: list[tuple[int, int, int, np.ndarray]] = []
        dev = self.device
        self.row_session = torch.empty(self.max_rows, dtype=torch.int32, device=dev)
        self.row_handle = torch.empty(self.max_rows, dtype=torch.int32, device=dev)
        self.row_frame = torch.empty(self.max_rows, dtype=torch.int64, device=dev)
        self.row_pcm = torch.empty((self.max_rows, PCM_SAMPLES), dtype=torch.float32, device=dev)
        self.n_rows = torch.zeros(1, dtype=torch.int32, device=dev)

    @property
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ------------------------------------------------------------ sessions
    def register_session(self, session_id: Hashable, handle: int) -> int:
        """Appends a session to the registration order; ``handle`` is its
        listener directory handle (ListenerEngine.pack)."""
        if session_id in self._index:
            raise ValueError(f"session already registered: {session_id}")
        if not self._free:
            raise RuntimeError("ingress session table exhausted")
        idx = self._free.pop()
        self._index[session_id] = idx
        self._ids[idx] = session_id
        self._events.append((_lib.INGRESS_JOIN, idx, int(handle)))
        return idx

    def unregister_session(self, session_id: Hashable) -> None:
        idx = self._index.pop(session_id)
        self._ids.pop(idx)
        self._events.append((_lib.INGRESS_LEAVE, idx, 0))
        self._arrivals = [a for a in self._arrivals if a[0] != idx]
        self._released.append(idx)

    def pause_session(self, session_id: Hashable) -> None:
        self._events.append((_lib.INGRESS_PAUSE, self._index[session_id], 0))

    def resume_session(self, session_id: Hashable) -> None:
        self._events.append((_lib.INGRESS_RESUME, self._index[session_id], 0))

    def submit(self, session_id: Hashable, frame_id: int, enqueue_ns: int, pcm: np.ndarray) -> None:
        """Queues one 80 ms frame (delivered to the device at the next tick)."""
        pcm = np.asarray(pcm, dtype=np.float32)
        if pcm.shape != (PCM_SAMPLES,):
            raise ValueError("listener frames carry 1280 PCM samples")
        self._arrivals.append((self._index[session_id], int(frame_id), int(enqueue_ns), pcm))

    # --------------------------------------------------------------- tick
    def _flush(self) -> None:
        dev, s = self.device, self._stream
        while self._events:
            batch, self._events = self._events[:1024], self._events[1024:]
            arr = torch.tensor(batch, dtype=torch.int32).t().contiguous().to(dev)
            _lib.check("lb_ingress_events_async", self.lib.lb_ingress_events_async(
                self._h, len(batch), arr[0].data_ptr(), arr[1].data_ptr(), arr[2].data_ptr(), s))
        # indices released before this flush may be reused from now on
        self._free.extend(reversed(self._released))
        self._released.clear()
        # at most one frame per session per push: the k-th queued frame of a
        # session goes into push k
        rounds: list[list] = []
        seen: dict[int, int] = {}
        for a in self._arrivals:
            k = seen.get(a[0], 0)
            seen[a[0]] = k + 1
            if k == len(rounds):
                rounds.append([])
            rounds[k].append(a)
        self._arrivals = []
        for r in rounds:
            n = len(r)
            sess = torch.tensor([a[0] for a in r], dtype=torch.int32)
            meta = torch.tensor([[a[1], a[2]] for a in r], dtype=torch.int64).t().contiguous()
            pcm = torch.from_numpy(np.stack([a[3] for a in r])).pin_memory()
            sess_d, meta_d = sess.to(dev), meta.to(dev)
            pcm_d = pcm.to(dev, non_blocking=True)
            _lib.check("lb_ingress_push_async", self.lib.lb_ingress_push_async(
                self._h, n, sess_d.data_ptr(), meta_d[0].data_ptr(), meta_d[1].data_ptr(), pcm_d.data_ptr(), s))
            # the staging tensors must outlive the asynchronous copies
            torch.cuda.current_stream(dev).synchronize()

    def dispatch_tick(self, deadline_ns: int) -> tuple[list[tuple[Hashable, int]], torch.Tensor, torch.Tensor,
                                                       torch.Tensor]:
        """Applies the pending events and arrivals, then runs one tick.

        Returns (rows as (session_id, frame_id) in registration order, row PCM
        [n,1280], row handles [n] int32, row frame ids [n] int64); the tensors
        are views of device buffers reused by the next tick."""
        self._flush()
        _lib.check("lb_ingress_tick_async", self.lib.lb_ingress_tick_async(
            self._h, int(deadline_ns), self.row_session.data_ptr(), self.row_handle.data_ptr(),
            self.row_frame.data_ptr(), self.row_pcm.data_ptr(), self.n_rows.data_ptr(), self._stream))
        n = int(self.n_rows.item())
        idx = self.row_session[:n].tolist()
        frames = self.row_frame[:n].tolist()
        rows = [(self._ids[i], f) for i, f in zip(idx, frames)]
        return rows, self.row_pcm[:n], self.row_handle[:n], self.row_frame[:n]

    def status(self) -> int:
        v = ctypes.c_int32(0)
        _lib.check("lb_ingress_get_status", self.lib.lb_ingress_get_status(self._h, ctypes.addressof(v),
                                                                           self._stream))
        return int(v.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.lb_ingress_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
