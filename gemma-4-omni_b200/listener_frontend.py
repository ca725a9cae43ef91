"""Drop-in ``ListenerMicrobatchAudioFrontend`` whose log-mel runs on the GPU.

Mirrors the reference frontend (duplex_kernel/listener_microbatch_frontend.py:
288-882): the constructor signature, ``encode_batch(batch, states, *,
listener_stream=None) -> PreparedListenerAudioBatch``, ``close_session``,
``close``, the single-owner-thread rule, one active manifest at a time, and
poisoning after a failed transaction.  ``PreparedListenerAudioBatch`` keeps
the reference fields the native listener consumes (``manifest_id``,
``audio_soft_tokens`` as a tuple of [2, text_hidden] tensors,
``audio_tower_raw_tokens``, ``audio_stream_cursors``,
``streaming_audio_input_shape``, ``input_shape``, ``valid_mel_counts``) and its
timing fields, plus ``commit`` / ``abort`` and
``cuda_phase_timings_after_completion``.

What changes is where the mel is made.  The reference extracts each row's
user mel with NumPy on the owner thread (``_stage_rows`` :748-835 ->
``listener.py:1807-1850``) and copies a [N, 240, 128] window to the GPU of
which the streaming tower reads the last 8 rows (:498-555).  Here the rows'
80 ms PCM frames ([N, 1280] float32, 5 KB per row) are copied once from a
pinned staging buffer and the tower's ``prepare_batch_pcm`` runs the log-mel
inside the step, with each session's 160-sample tail kept in its state slot
and advanced by the same commit as the rest of its state.  A new session or
identity starts from a zero tail; across a cursor gap the session keeps its
tail, as the reference keeps it in the session state.  The assistant
(reference) audio of every row is turned into mel as well, as the reference
does for its history (:792-809): all rows in one GPU pass (``lb_mel_async``)
with each session's assistant tail held on the device and advanced on commit;
``PreparedListenerAudioBatch.assistant_mels`` is that [N, 8, 128] tensor (a
row without reference audio uses silence, as in the reference).  No W240
window, per-row runner fallback or host mel history is kept: the streaming
tower is the only execution path.

The batch and state objects are the reference's contracts
(duplex_kernel/microbatch_contract.py), used by attribute: ``batch.manifest``
(``manifest_id``, ``batch_size``, ``rows`` with ``session_id``,
``session_generation``, ``state_epoch_id``, ``frame_id``,
``sequence_position``), ``batch.frames`` (``pcm``) and per-row states
(``session_id``).
"""
from __future__ import annotations

import threading
import time
from typing import Any, Sequence

import numpy as np
import torch

from .streaming_conformer import AudioStreamCursor, StreamingConformerAudioTower

MEL_ROWS_PER_FRAME = 8
MEL_BINS = 128
PCM_SAMPLES_PER_FRAME = 1280
CONTEXT_FRAMES = 64


def _elapsed(events: tuple[Any, Any] | None) -> float | None:
    if events is None:
        return None
    return float(events[0].elapsed_time(events[1]))


class PreparedListenerAudioBatch:
    """Encoded rows plus the all-row commit transaction (reference :113-286)."""

    def __init__(self, *, owner: "ListenerMicrobatchAudioFrontend", manifest_id: str, n: int,
                 streaming_batch, cursors: tuple, frontend_copy_ms: float, frontend_copy_events,
                 tower_events, graph_submit_ms: float, owner_thread_id: int,
                 assistant_mels: torch.Tensor, assistant_tails: torch.Tensor) -> None:
        self._owner = owner
        self.assistant_mels = assistant_mels
        self._assistant_tails = assistant_tails
        self.manifest_id = manifest_id
        self.input_shape = (n, MEL_ROWS_PER_FRAME, MEL_BINS)
        self.streaming_audio_input_shape = (n, MEL_ROWS_PER_FRAME, MEL_BINS)
        self.valid_mel_counts = tuple(MEL_ROWS_PER_FRAME for _ in range(n))
        soft = streaming_batch.soft_tokens
        raw = streaming_batch.raw_tokens
        self.audio_soft_tokens = tuple(soft[i].detach() for i in range(n))
        self.audio_tower_raw_tokens = tuple(raw[i].detach() for i in range(n))
        self.audio_stream_cursors = cursors
        self.mel_prepare_ms_by_row = tuple(0.0 for _ in range(n))  # mel runs inside the step
        self.frontend_copy_ms = frontend_copy_ms
        self.audio_tower_lock_wait_ms = 0.0
        self.audio_tower_lock_hold_ms = 0.0
        self.audio_tower_graph_submit_ms = graph_submit_ms
        self.audio_tower_execution_mode = f"streaming_conformer_{streaming_batch.execution_mode}_n{n}"
        self.audio_tower_workspace_lock_wait_ms = 0.0
        self.audio_tower_workspace_lock_hold_ms = 0.0
        self._copy_events = frontend_copy_events
        self._tower_events = tower_events
        self._streaming_audio_batch = streaming_batch
        self._owner_thread_id = owner_thread_id
        self._committed = False
        self._aborted = False

    def cuda_phase_timings_after_completion(self) -> tuple[float | None, float | None, float | None]:
        """(frontend copy ms, per-row copy ms, tower ms) from CUDA events; call
        only after the listener stream has completed (no synchronisation here)."""
        return _elapsed(self._copy_events), None, _elapsed(self._tower_events)

    def audio_tower_batch_cuda_span_ms_after_completion(self) -> float | None:
        return _elapsed(self._tower_events)

    @property
    def committed(self) -> bool:
        return self._committed

    def commit(self) -> None:
        """Installs every row's staged tower state and PCM tail, all or nothing."""
        if self._committed:
            raise RuntimeError("frontend transaction was already committed")
        if self._aborted:
            raise RuntimeError("frontend transaction was aborted")
        if threading.get_ident() != self._owner_thread_id:
            raise RuntimeError("frontend state must be committed by its single owner thread")
        try:
            self._streaming_audio_batch.commit()
        except BaseException:
            self._aborted = True
            self._owner._finish(self.manifest_id, failed=True)
            raise
        for i, cursor in enumerate(self.audio_stream_cursors):
            self._owner._assistant_tails[cursor.session_id] = self._assistant_tails[i]
        self._committed = True
        self._owner._finish(self.manifest_id, failed=False)

    def abort(self) -> None:
        """Releases the lease after downstream work failed; poisons the frontend."""
        if self._committed:
            raise RuntimeError("committed frontend transaction cannot be aborted")
        if self._aborted:
            raise RuntimeError("frontend transaction was already aborted")
        if threading.get_ident() != self._owner_thread_id:
            raise RuntimeError("frontend transaction must be aborted by its single owner thread")
        self._aborted = True
        try:
            self._streaming_audio_batch.abort()
        finally:
            self._owner._finish(self.manifest_id, failed=True)


class ListenerMicrobatchAudioFrontend:
    """Shared listener frontend: PCM rows in, streaming-tower soft tokens out."""

    def __init__(self, gemma_model: Any, extract_single_frame: Any = None, *, device: torch.device | str,
                 dtype: torch.dtype, context_frames: int = CONTEXT_FRAMES, mel_window_rows: int = 240,
                 audio_tower_lock: Any | None = None, audio_tower_row_runner: Any | None = None,
                 streaming_audio_tower: StreamingConformerAudioTower | None = None, max_sessions: int = 64) -> None:
        if isinstance(context_frames, bool) or not isinstance(context_frames, int) or context_frames != CONTEXT_FRAMES:
            raise ValueError(f"batched listener frontend is pinned to {CONTEXT_FRAMES} context frames")
        if not isinstance(dtype, torch.dtype):
            raise TypeError("dtype must be a torch.dtype")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the B200 listener frontend runs on CUDA only (no CPU fallback)")
        if streaming_audio_tower is None:
            streaming_audio_tower = StreamingConformerAudioTower.from_gemma_model(
                gemma_model, device=self.device, dtype=dtype, max_sessions=max_sessions)
        if not callable(getattr(streaming_audio_tower, "prepare_batch_pcm", None)):
            raise TypeError("streaming_audio_tower must be the B200 StreamingConformerAudioTower")
        self.dtype = dtype
        self.context_frames = context_frames
        self.mel_window_rows = mel_window_rows
        self.audio_tower_lock = audio_tower_lock
        self.streaming_audio_tower = streaming_audio_tower
        self._owner_thread_id: int | None = None
        self._call_lock = threading.Lock()
        self._active_manifest_id: str | None = None
        self._poisoned = False
        self._closed = False
        self._pinned: torch.Tensor | None = None
        self._copy_done: torch.cuda.Event | None = None
        self._assistant_tails: dict[str, torch.Tensor] = {}  # session -> device [160] float32
        self.encoder_call_count = 0

    # ------------------------------------------------------------ lifetime
    def _ensure_open(self) -> None:
        if self._closed:
            raise RuntimeError("listener audio frontend is closed")

    def close_session(self, session_id: str) -> None:
        """Release one session's tower state (and PCM tail) while the frontend is idle."""
        if not isinstance(session_id, str) or not session_id:
            raise ValueError("session_id must be a non-empty string")
        if not self._call_lock.acquire(blocking=False):
            raise RuntimeError("cannot close streaming audio state while the frontend is active")
        try:
            self._ensure_open()
            if self._active_manifest_id is not None:
                raise RuntimeError("cannot close streaming audio state while a batch is prepared")
            self.streaming_audio_tower.reset(session_id)
            self._assistant_tails.pop(session_id, None)
        finally:
            self._call_lock.release()

    def close(self) -> None:
        if not self._call_lock.acquire(blocking=False):
            raise RuntimeError("cannot close listener audio frontend while it is active")
        try:
            if self._active_manifest_id is not None:
                raise RuntimeError("cannot close listener audio frontend with a prepared batch")
            if self._closed:
                return
            self.streaming_audio_tower.close()
            self._pinned = None
            self._owner_thread_id = None
            self._closed = True
        finally:
            self._call_lock.release()

    def _finish(self, manifest_id: str, *, failed: bool) -> None:
        if self._active_manifest_id == manifest_id:
            self._active_manifest_id = None
        if failed:
            self._poisoned = True

    def _staging(self, n: int) -> torch.Tensor:
        # the previous tick's H2D must have left the buffer before it is rewritten
        # (long done in steady state: the caller waited for that tick's outputs)
        if self._copy_done is not None:
            self._copy_done.synchronize()
            self._copy_done = None
        if self._pinned is None or self._pinned.shape[0] < n:
            cap = max(n, 2 * (self._pinned.shape[0] // 2 if self._pinned is not None else 0), 16)
            # rows [0, cap): user PCM; rows [cap, 2 cap): assistant (reference) PCM
            self._pinned = torch.empty((2 * cap, PCM_SAMPLES_PER_FRAME), dtype=torch.float32, pin_memory=True)
        cap = self._pinned.shape[0] // 2
        return self._pinned[:n], self._pinned[cap:cap + n]

    # ----------------------------------------------------------- the tick
    def encode_batch(self, batch: Any, states: Sequence[Any], *,
                     listener_stream: Any | None = None) -> PreparedListenerAudioBatch:
        rows = tuple(states)
        with self._call_lock:
            self._ensure_open()
            current = threading.get_ident()
            if self._owner_thread_id is None:
                self._owner_thread_id = current
            elif self._owner_thread_id != current:
                raise RuntimeError("listener audio frontend has a single owner thread")
            if self._poisoned:
                raise RuntimeError("listener audio frontend is poisoned after a failed transaction")
            if self._active_manifest_id is not None:
                raise RuntimeError("previous frontend batch has not committed")
            manifest = batch.manifest
            n = int(manifest.batch_size)
            if len(rows) != n or len(batch.frames) != n or len(manifest.rows) != n:
                raise ValueError("batch, manifest, and state row counts must match")
            if len({id(s) for s in rows}) != n:
                raise ValueError("a frontend batch cannot alias a session state object")
            if len({s.session_id for s in rows}) != n:
                raise ValueError("a frontend batch requires distinct session states")
            for row, state in zip(manifest.rows, rows):
                if state.session_id != row.session_id:
                    raise RuntimeError("frontend row does not match its current session snapshot")
            stream = listener_stream if listener_stream is not None else torch.cuda.current_stream(self.device)
            copy_started = time.perf_counter_ns()
            host, host_ref = self._staging(n)
            for i, frame in enumerate(batch.frames):
                pcm = np.asarray(frame.pcm, dtype=np.float32)
                if pcm.shape != (PCM_SAMPLES_PER_FRAME,):
                    raise ValueError("listener frames must carry 1280 PCM samples")
                host[i].numpy()[:] = pcm
                ref = getattr(frame, "reference_pcm", None)
                if ref is None:
                    host_ref[i].numpy()[:] = 0.0  # no assistant audio: silence, as the reference
                else:
                    ref = np.asarray(ref, dtype=np.float32)
                    if ref.shape != (PCM_SAMPLES_PER_FRAME,):
                        raise ValueError("reference frames must carry 1280 PCM samples")
                    host_ref[i].numpy()[:] = ref
            cursors = tuple(AudioStreamCursor(session_id=row.session_id, generation_id=int(row.session_generation),
                                              state_epoch_id=row.state_epoch_id, frame_id=int(row.frame_id),
                                              sequence_position=int(row.sequence_position))
                            for row in manifest.rows)
            self._active_manifest_id = manifest.manifest_id
            try:
                with torch.cuda.stream(stream):
                    copy_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    tower_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    copy_ev[0].record(stream)
                    pcm_dev = host.to(self.device, non_blocking=True)
                    ref_dev = host_ref.to(self.device, non_blocking=True)
                    copy_ev[1].record(stream)
                    zero = torch.zeros(160, dtype=torch.float32, device=self.device)
                    tail_in = torch.stack([self._assistant_tails.get(s.session_id, zero) for s in rows])
                    tail_out = torch.empty((n, 160), dtype=torch.float32, device=self.device)
                    assistant_mels = torch.empty((n, MEL_ROWS_PER_FRAME, MEL_BINS), dtype=torch.float32,
                                                 device=self.device)
                    self.streaming_audio_tower._engine.mel(ref_dev, tail_in, tail_out, assistant_mels)
                    frontend_copy_ms = (time.perf_counter_ns() - copy_started) / 1e6
                    self.encoder_call_count += 1
                    submit = time.perf_counter_ns()
                    streaming = self.streaming_audio_tower.prepare_batch_pcm(pcm_dev, cursors,
                                                                             graph_event_pair=tower_ev)
                    graph_submit_ms = (time.perf_counter_ns() - submit) / 1e6
                    # the staging buffer is reused by the next tick: its copy must have left
                    done = torch.cuda.Event()
                    done.record(stream)
                self._copy_done = done
            except BaseException:
                self._active_manifest_id = None
                self._poisoned = True
                raise
            return PreparedListenerAudioBatch(owner=self, manifest_id=manifest.manifest_id, n=n,
                                              streaming_batch=streaming, cursors=cursors,
                                              frontend_copy_ms=round(frontend_copy_ms, 3),
                                              frontend_copy_events=copy_ev, tower_events=tower_ev,
                                              graph_submit_ms=round(graph_submit_ms, 3),
                                              owner_thread_id=current, assistant_mels=assistant_mels,
                                              assistant_tails=tail_out)
