"""Drop-in ``StreamingConformerAudioTower`` backed by the B200 listener step.

Mirrors the public interface of the reference class
(duplex_kernel/streaming_conformer.py:27-1052): ``AudioStreamCursor``,
``StreamingConformerAudioTower(audio_tower, embed_audio, *, device, dtype,
max_sessions, ...)``, ``from_gemma_model(_optimized_cuda)``,
``prepare_batch(mel_tick, cursors, *, input_mask=None, ...)`` returning a
``PreparedStreamingAudioBatch`` with ``raw_tokens``, ``soft_tokens``,
``subsampled``, ``layer_tokens``, ``slot_ids``, ``reset_reasons``,
``execution_mode`` and the ``commit / abort / rollback_committed``
transaction, plus ``reset``, ``reset_session``, ``capture_graph``,
``committed_positions`` and ``close``.  Error types and messages follow the
reference (ValueError / TypeError for contract violations, RuntimeError for
state and capacity).

What differs, by design:
- the slot policy, cache staging and commit run on the GPU (one packer kernel,
  ring-head commits); slot ids and reasons are read back lazily, and
  ``prepare_batch`` does not wait for the step (the host-side checks that
  precede it are the reference's own capacity and identity rules); the one
  host wait is in ``commit``, which reads the device's all-or-nothing cursor
  check -- by then the caller has already waited for the step's outputs;
- ``prepare_batch_pcm`` takes the 80 ms PCM frames themselves ([N,1280]
  float32) and runs the log-mel frontend on the GPU with each session's
  160-sample tail kept in its slot (committed with the rest of its state);
- one CUDA graph per power-of-two row bucket with a device-side row count
  replaces one graph per N; ``capture_graph`` is accepted and is a no-op;
- per-layer outputs (``layer_tokens``) and ``subsampled`` cost an eager
  diagnostic run, so they are produced only with ``return_layer_tokens=True``.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np
import torch

from . import _lib
from .config import WEIGHT_BF16, WEIGHT_INT8, ListenerConfig
from .runtime import ListenerEngine

MEL_TICK_ROWS = 8
MEL_BINS = 128
Q2_TOKENS = 2
PCM_SAMPLES = 1280
REASONS = _lib.REASONS


@dataclass(frozen=True, slots=True)
class AudioStreamCursor:
    """Stable session identity and the cursor before this Mel tick (streaming_conformer.py:27-49)."""

    session_id: str
    generation_id: int
    state_epoch_id: str
    frame_id: int
    sequence_position: int

    def __post_init__(self) -> None:
        if not isinstance(self.session_id, str) or not self.session_id:
            raise ValueError("audio stream session_id must be non-empty")
        if not isinstance(self.state_epoch_id, str) or not self.state_epoch_id:
            raise ValueError("audio stream state_epoch_id must be non-empty")
        for name in ("generation_id", "frame_id", "sequence_position"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, int) or value < 0:
                raise ValueError(f"audio stream {name} must be a non-negative integer")

    @property
    def key(self) -> tuple[str, int, str]:
        return (self.session_id, self.generation_id, self.state_epoch_id)


class PreparedStreamingAudioBatch:
    """A staged tower result whose state advances only on ``commit``."""

    def __init__(self, owner: "StreamingConformerAudioTower", *, cursors, raw_tokens, soft_tokens,
                 subsampled, layer_tokens, execution_mode: str) -> None:
        self._owner = owner
        self.cursors = cursors
        self.raw_tokens = raw_tokens
        self.soft_tokens = soft_tokens
        self.subsampled = subsampled
        self.layer_tokens = layer_tokens
        self.execution_mode = execution_mode
        self._slots: tuple[int, ...] | None = None
        self._reasons: tuple[str, ...] | None = None
        self._committed = False
        self._aborted = False
        self._rollback_ok = False

    def _read_rows(self) -> None:
        if self._slots is None:
            slots, reasons = self._owner._engine.read_rows(len(self.cursors))
            self._slots = tuple(int(s) for s in slots)
            self._reasons = tuple(REASONS[int(r)] for r in reasons)

    @property
    def slot_ids(self) -> tuple[int, ...]:
        self._read_rows()
        return self._slots

    @property
    def reset_reasons(self) -> tuple[str, ...]:
        self._read_rows()
        return self._reasons

    @property
    def committed(self) -> bool:
        return self._committed

    def commit(self) -> None:
        if self._committed:
            raise RuntimeError("streaming audio batch was already committed")
        if self._aborted:
            raise RuntimeError("streaming audio batch was aborted")
        self._read_rows()
        self._owner._commit(self)
        self._committed = True

    def rollback_committed(self) -> None:
        """Restore the prior state if its enclosing listener transaction fails."""
        if not self._committed or not self._rollback_ok:
            raise RuntimeError("streaming audio batch has no committed state to roll back")
        self._owner._rollback(self)
        self._committed = False
        self._rollback_ok = False

    def abort(self) -> None:
        if self._committed:
            raise RuntimeError("committed streaming audio batch cannot be aborted")
        if self._aborted:
            raise RuntimeError("streaming audio batch was already aborted")
        self._owner._abort(self)
        self._aborted = True


def config_from_modules(audio_tower: Any, embed_audio: Any) -> ListenerConfig:
    c = audio_tower.config
    text_hidden = int(getattr(embed_audio, "text_hidden_size", c.output_proj_dims))
    return ListenerConfig(hidden=int(c.hidden_size), layers=int(c.num_hidden_layers),
                          heads=int(c.num_attention_heads), ffn=4 * int(c.hidden_size),
                          sub_ch0=int(c.subsampling_conv_channels[0]), sub_ch1=int(c.subsampling_conv_channels[1]),
                          output_dims=int(c.output_proj_dims), text_hidden=text_hidden,
                          conv_kernel=int(c.conv_kernel_size), rms_eps=float(c.rms_norm_eps),
                          softcap=float(c.attention_logit_cap), invalid_logit=float(c.attention_invalid_logits_value),
                          gradient_clipping=float(c.gradient_clipping), residual_weight=float(c.residual_weight),
                          film_enabled=False)


def state_dict_numpy(audio_tower: Any, embed_audio: Any) -> dict[str, np.ndarray]:
    out = {k: v.detach().float().cpu().numpy() for k, v in audio_tower.state_dict().items()
           if not k.endswith("inv_timescales")}
    out.update({f"embed.{k}": v.detach().float().cpu().numpy() for k, v in embed_audio.state_dict().items()})
    # clip bounds stay scalars; +/-inf bounds are the unclipped default
    return {k: v for k, v in out.items()
            if not (k.endswith(("input_min", "input_max", "output_min", "output_max")) and not np.isfinite(v).all())}


class StreamingConformerAudioTower:
    """Per-session incremental execution of Gemma4AudioModel on the B200 listener step."""

    def __init__(self, audio_tower: Any, embed_audio: Any, *, device: torch.device | str, dtype: torch.dtype,
                 max_sessions: int = 64, capture_cuda_graphs: bool = False, optimize_cuda: bool = False,
                 weight_format: int | None = None, max_rows: int | None = None,
                 return_layer_tokens: bool = False) -> None:
        if not callable(getattr(audio_tower, "subsample_conv_projection", None)):
            raise TypeError("audio_tower must be an installed Gemma4AudioModel")
        if not callable(embed_audio):
            raise TypeError("embed_audio must be Gemma4MultimodalEmbedder")
        if not isinstance(dtype, torch.dtype):
            raise TypeError("dtype must be a torch.dtype")
        if isinstance(max_sessions, bool) or not isinstance(max_sessions, int) or max_sessions < 2:
            raise ValueError("max_sessions must be an integer >= 2")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the B200 listener tower runs on CUDA only (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.audio_tower = audio_tower
        self.embed_audio = embed_audio
        self.dtype = dtype
        self.max_sessions = max_sessions
        self.optimize_cuda = bool(optimize_cuda)
        self._validate_model()
        cfg = config_from_modules(audio_tower, embed_audio)
        self.hidden_size, self.num_layers = cfg.hidden, cfg.layers
        self.num_heads, self.head_dim = cfg.heads, cfg.head_dim
        self.output_size, self.text_hidden_size = cfg.output_dims, cfg.text_hidden
        fmt = weight_format if weight_format is not None else WEIGHT_BF16
        if fmt not in (WEIGHT_BF16, WEIGHT_INT8):
            raise ValueError("weight_format must be WEIGHT_BF16 or WEIGHT_INT8")
        self._engine = ListenerEngine(cfg, max_sessions=max_sessions, max_rows=max_rows or max_sessions,
                                      max_handles=max(max_sessions * 4, 64), weight_format=fmt, device=self.device)
        self._engine.load_weights(state_dict_numpy(audio_tower, embed_audio), None, keep_effective=False)
        self._return_layers = bool(return_layer_tokens)
        self._lock = threading.RLock()
        self._closed = False
        self._active: PreparedStreamingAudioBatch | None = None
        # session id -> handle of the device-side session directory; a handle is
        # returned to the pool when its session's state is released (reset,
        # reset_session) or when the batch that introduced it is aborted, so
        # the pool never runs dry under session churn
        self._handles: dict[str, int] = {}
        self._free_handles: list[int] = list(range(self._engine.max_handles - 1, -1, -1))
        self._key_ids: dict[tuple[int, str], int] = {}  # (generation, epoch) -> int64 key
        self._identity: dict[str, tuple[int, str]] = {}  # committed identity per bound session
        self._bound: set[str] = set()
        self._last_commit: tuple | None = None

    # ------------------------------------------------------------ factories
    @classmethod
    def from_gemma_model(cls, gemma_model: Any, *, device, dtype, max_sessions: int = 64,
                         capture_cuda_graphs: bool = False, optimize_cuda: bool = False, **kw):
        audio_tower = getattr(gemma_model, "audio_tower", None)
        embed_audio = getattr(gemma_model, "embed_audio", None)
        if audio_tower is None or embed_audio is None:
            raise TypeError("Gemma4Model must expose audio_tower and embed_audio")
        return cls(audio_tower, embed_audio, device=device, dtype=dtype, max_sessions=max_sessions,
                   capture_cuda_graphs=capture_cuda_graphs, optimize_cuda=optimize_cuda, **kw)

    @classmethod
    def from_gemma_model_optimized_cuda(cls, gemma_model: Any, *, device, dtype, max_sessions: int = 128,
                                        max_graph_batch_size: int = 4, **kw):
        if isinstance(max_sessions, bool) or not isinstance(max_sessions, int) or max_sessions < 2:
            raise ValueError("max_sessions must be an integer >= 2")
        if (isinstance(max_graph_batch_size, bool) or not isinstance(max_graph_batch_size, int)
                or max_graph_batch_size < 1 or max_graph_batch_size > max_sessions):
            raise ValueError("max_graph_batch_size must be within persistent session capacity")
        if torch.device(device).type != "cuda" or dtype is not torch.bfloat16:
            raise ValueError("optimized CUDA startup requires CUDA BF16")
        return cls.from_gemma_model(gemma_model, device=device, dtype=dtype, max_sessions=max_sessions,
                                    capture_cuda_graphs=True, optimize_cuda=True, **kw)

    def _validate_model(self) -> None:
        """The reference's checks (streaming_conformer.py:375-407): exact chunking,
        eval mode, modules already on the requested device and dtype, and the
        subsampler geometry the streaming state layout assumes."""
        config = self.audio_tower.config
        exact = {"attention_chunk_size": 12, "attention_context_left": 13, "attention_context_right": 0,
                 "conv_kernel_size": 5}
        for name, expected in exact.items():
            actual = int(getattr(config, name, -1))
            if actual != expected:
                raise ValueError(f"Gemma audio {name} must be {expected}, found {actual}")
        if int(config.hidden_size) % int(config.num_attention_heads):
            raise ValueError("Gemma audio hidden_size must divide evenly across attention heads")
        if len(self.audio_tower.layers) != int(config.num_hidden_layers):
            raise ValueError("Gemma audio layer count differs from its configuration")
        if self.audio_tower.training or self.embed_audio.training:
            raise ValueError("incremental Gemma audio tower requires eval mode")
        parameter = next(self.audio_tower.parameters())
        embed_parameter = next(self.embed_audio.parameters())
        if parameter.device != self.device or embed_parameter.device != self.device:
            raise ValueError("audio tower and embed_audio must already be on the requested device")
        if parameter.dtype != self.dtype or embed_parameter.dtype != self.dtype:
            raise ValueError("audio tower and embed_audio must already use the requested dtype")
        layers = self.audio_tower.subsample_conv_projection
        for name in ("layer0", "layer1"):
            layer = getattr(layers, name, None)
            if layer is None or tuple(layer.conv.kernel_size) != (3, 3):
                raise ValueError("Gemma audio subsampler must use its 3x3 convolution layers")
            if tuple(layer.conv.stride) != (2, 2) or tuple(layer.conv.padding) != (1, 1):
                raise ValueError("Gemma audio subsampler must use stride 2 and symmetric padding 1")
            if layer.conv.bias is not None:
                raise ValueError("Gemma audio subsampler convolutions must remain biasless")

    # --------------------------------------------------------------- state
    @property
    def committed_positions(self) -> tuple[tuple[str, int, str, int, int], ...]:
        slot, key, ef, es = self._engine.read_handles()
        inv = {v: k for k, v in self._key_ids.items()}
        out = []
        for sid, h in self._handles.items():
            if slot[h] >= 0 and ef[h] >= 0 and int(key[h]) in inv:
                gen, ep = inv[int(key[h])]
                out.append((sid, gen, ep, int(ef[h]), int(es[h])))
        return tuple(sorted(out))

    def _ensure_open(self) -> None:
        if self._closed:
            raise RuntimeError("StreamingConformerAudioTower is closed")

    def reset(self, session_id: str, generation_id: int | None = None, state_epoch_id: str | None = None) -> None:
        """Clear one identity, or every generation/epoch for a session."""
        with self._lock:
            self._ensure_open()
            if self._active is not None:
                raise RuntimeError("cannot reset streaming audio state while a batch is prepared")
            ident = self._identity.get(session_id)
            if session_id not in self._bound or ident is None:
                return
            if (generation_id is not None and ident[0] != generation_id) or \
                    (state_epoch_id is not None and ident[1] != state_epoch_id):
                return
            self._engine.reset_handle(self._handles[session_id])
            self._bound.discard(session_id)
            self._identity.pop(session_id, None)
            self._release_handle(session_id)
            self._last_commit = None

    def reset_session(self, slot_idx: int) -> None:
        """Release exactly one persistent slot after its owner session is idle."""
        if isinstance(slot_idx, bool) or not isinstance(slot_idx, int):
            raise TypeError("slot_idx must be an integer")
        if slot_idx < 0 or slot_idx >= self.max_sessions:
            raise IndexError(f"slot_idx {slot_idx} is outside [0, {self.max_sessions})")
        with self._lock:
            self._ensure_open()
            if self._active is not None:
                raise RuntimeError("cannot reset a streaming audio slot while a batch is prepared")
            slot, _, _, _ = self._engine.read_handles()
            owners = [sid for sid, h in self._handles.items() if slot[h] == slot_idx]
            self._engine.reset_slot(slot_idx)
            for sid in owners:
                self._bound.discard(sid)
                self._identity.pop(sid, None)
                self._release_handle(sid)
            self._last_commit = None

    def capture_graph(self, batch_size: int) -> None:
        """Accepted for API compatibility: graphs are captured per row bucket on first use."""
        if isinstance(batch_size, bool) or not isinstance(batch_size, int) or not 1 <= batch_size <= self.max_sessions:
            raise ValueError(f"streaming Conformer graph batch size must be within [1, {self.max_sessions}]")

    # ----------------------------------------------------------- the step
    def _handle(self, sid: str) -> int:
        h = self._handles.get(sid)
        if h is None:
            if not self._free_handles:
                raise RuntimeError("streaming audio session handle table exhausted")
            h = self._free_handles.pop()
            self._handles[sid] = h
        return h

    def _release_handle(self, sid: str) -> None:
        """Returns a session's handle to the pool; its directory entry is clear
        (never committed, or cleared by the reset kernel)."""
        h = self._handles.pop(sid, None)
        if h is not None:
            self._free_handles.append(h)

    def prepare_batch(self, mel_tick: torch.Tensor, cursors: Sequence[AudioStreamCursor], *,
                      input_mask: torch.Tensor | None = None, use_cuda_graph: bool = False,
                      graph_event_pair: tuple[Any, Any] | None = None) -> PreparedStreamingAudioBatch:
        rows = tuple(cursors)
        if not isinstance(mel_tick, torch.Tensor) or mel_tick.ndim != 3:
            raise ValueError("streaming Q2 Mel input must be [N,8,128]")
        n = len(rows)
        if n <= 0 or tuple(mel_tick.shape) != (n, MEL_TICK_ROWS, MEL_BINS):
            raise ValueError("streaming Q2 Mel input must match [N,8,128] cursors")
        if mel_tick.device != self.device:
            raise ValueError("streaming Q2 Mel input device/dtype differs from the audio tower")
        return self._prepare(mel_tick.to(torch.float32).contiguous(), _lib.LB_INPUT_MEL, rows, input_mask,
                             graph_event_pair)

    def prepare_batch_pcm(self, pcm_frames: torch.Tensor, cursors: Sequence[AudioStreamCursor], *,
                          input_mask: torch.Tensor | None = None,
                          graph_event_pair: tuple[Any, Any] | None = None) -> PreparedStreamingAudioBatch:
        """``prepare_batch`` from the raw 80 ms PCM frames ([N,1280] float32, 16 kHz).

        The incremental log-mel of each row (duplex_kernel/listener.py:1807-1850:
        [160-sample tail | 1280 samples], 8 Hann-windowed 320-sample frames, hop
        160, |rfft 512|, HTK mel 128, log(x + 1e-3)) runs on the GPU inside the
        step; the tail lives in the session's slot, advances on ``commit`` and
        starts from zeros on every reset reason, exactly when the tower state does.
        """
        rows = tuple(cursors)
        if not isinstance(pcm_frames, torch.Tensor) or pcm_frames.ndim != 2:
            raise ValueError("streaming PCM input must be [N,1280]")
        n = len(rows)
        if n <= 0 or tuple(pcm_frames.shape) != (n, PCM_SAMPLES):
            raise ValueError("streaming PCM input must match [N,1280] cursors")
        if pcm_frames.device != self.device or pcm_frames.dtype != torch.float32:
            raise ValueError("streaming PCM input must be float32 on the audio device")
        return self._prepare(pcm_frames.contiguous(), _lib.LB_INPUT_PCM, rows, input_mask, graph_event_pair)

    def _prepare(self, inputs: torch.Tensor, kind: int, rows: tuple, input_mask, graph_event_pair):
        n = len(rows)
        if len({row.key for row in rows}) != n or len({row.session_id for row in rows}) != n:
            raise ValueError("a streaming audio batch requires distinct session identities")
        if input_mask is not None and (not isinstance(input_mask, torch.Tensor)
                                       or tuple(input_mask.shape) != (n, MEL_TICK_ROWS)
                                       or input_mask.device != self.device):
            raise ValueError("streaming input mask must have shape [N,8] on the audio device")
        with self._lock:
            self._ensure_open()
            if self._active is not None:
                raise RuntimeError("previous streaming audio batch has not committed or aborted")
            # a new step overwrites the ring entries a rollback would need
            self._last_commit = None
            new = sum(1 for r in rows if r.session_id not in self._bound)
            if len(self._bound) + new > self.max_sessions:
                raise RuntimeError(f"streaming audio session bank exhausted ({self.max_sessions} sessions)")
            handles = torch.tensor([self._handle(r.session_id) for r in rows], dtype=torch.int32)
            keys = torch.tensor([self._key_ids.setdefault((r.generation_id, r.state_epoch_id), len(self._key_ids))
                                 for r in rows], dtype=torch.int64)
            frames = torch.tensor([r.frame_id for r in rows], dtype=torch.int64)
            seqs = torch.tensor([r.sequence_position for r in rows], dtype=torch.int64)
            masks = None
            if input_mask is not None:
                bits = (input_mask.to(torch.uint8) << torch.arange(8, device=self.device, dtype=torch.uint8)).sum(1)
                masks = bits.to(torch.uint8).contiguous()
            dev = self.device
            try:
                self._engine.pack(handles.to(dev, non_blocking=True), keys.to(dev, non_blocking=True),
                                  frames.to(dev, non_blocking=True), seqs.to(dev, non_blocking=True), masks)
                if graph_event_pair is not None:
                    graph_event_pair[0].record()
                try:
                    out = self._engine.step(inputs, kind=kind, debug=self._return_layers)
                except BaseException:
                    self._engine.abort()
                    raise
            except BaseException:
                self._release_new_handles(rows)
                raise
            if graph_event_pair is not None:
                graph_event_pair[1].record()
            layers = tuple(out["layers"][i].to(self.dtype) for i in range(self.num_layers)) if self._return_layers else ()
            sub = out["subsampled"].to(self.dtype) if self._return_layers else None
            prepared = PreparedStreamingAudioBatch(
                self, cursors=rows, raw_tokens=out["raw"].to(self.dtype), soft_tokens=out["soft"].to(self.dtype),
                subsampled=sub, layer_tokens=layers,
                execution_mode="eager" if self._return_layers else "cuda_graph")
            self._active = prepared
            return prepared

    def _release_new_handles(self, rows) -> None:
        """Handles of sessions this (aborted) batch introduced go back to the pool."""
        for r in rows:
            if r.session_id not in self._bound:
                self._release_handle(r.session_id)

    def _commit(self, batch: PreparedStreamingAudioBatch) -> None:
        with self._lock:
            if self._active is not batch:
                raise RuntimeError("streaming audio transaction is no longer active")
            self._active = None
            self._engine.commit()
            # the one host wait of a tick: the device's all-or-nothing cursor
            # check (and the packer's capacity / identity checks) of this batch
            st = self._engine.status()
            if st & _lib.DEV_STALE_COMMIT:
                self._engine.clear_status()
                batch._aborted = True
                self._release_new_handles(batch.cursors)
                raise RuntimeError("cursor changed before streaming commit")
            if st & (_lib.DEV_SLOT_EXHAUSTED | _lib.DEV_DUPLICATE_ROW | _lib.DEV_BAD_HANDLE):
                self._engine.clear_status()
                batch._aborted = True
                self._release_new_handles(batch.cursors)
                raise RuntimeError(f"streaming audio session bank exhausted ({self.max_sessions} sessions)")
            if st:
                raise RuntimeError(f"listener device status {st:#x}")
            prev = (set(self._bound), dict(self._identity))
            for r in batch.cursors:
                self._bound.add(r.session_id)
                self._identity[r.session_id] = (r.generation_id, r.state_epoch_id)
            self._last_commit = (batch, prev)
            batch._rollback_ok = True

    def _rollback(self, batch: PreparedStreamingAudioBatch) -> None:
        with self._lock:
            if self._last_commit is None or self._last_commit[0] is not batch:
                raise RuntimeError("streaming audio rollback record is missing")
            self._engine.rollback()
            self._bound, self._identity = self._last_commit[1]
            self._last_commit = None
            # sessions the rolled-back batch had introduced are unbound again
            self._release_new_handles(batch.cursors)

    def _abort(self, batch: PreparedStreamingAudioBatch) -> None:
        with self._lock:
            if self._active is not batch:
                raise RuntimeError("streaming audio transaction is no longer active")
            self._active = None
            self._engine.abort()
            self._release_new_handles(batch.cursors)

    def close(self) -> None:
        """Release session state when idle."""
        with self._lock:
            if self._active is not None:
                raise RuntimeError("cannot close StreamingConformerAudioTower with an active batch")
            if self._closed:
                return
            self._engine.close()
            self._handles.clear()
            self._bound.clear()
            self._identity.clear()
            self._closed = True
