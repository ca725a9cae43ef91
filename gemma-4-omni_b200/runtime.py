"""Python wrapper of one listener context (one GPU, one owner thread).

``ListenerEngine`` owns a C-ABI context (include/listener_b200.h) and exposes
the step transaction with torch tensors: ``pack`` -> ``step`` -> ``commit`` (or
``abort`` / ``rollback``).  Device memory for weights, per-slot session state
and activations lives in the C library; torch is used only for the caller's
input/output tensors and the CUDA stream.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .config import WEIGHT_BF16, ListenerConfig
from .weights import prepare


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class ListenerEngine:
    """One streaming-listener context bound to the current CUDA device."""

    def __init__(self, cfg: ListenerConfig, *, max_sessions: int, max_rows: int | None = None,
                 max_handles: int | None = None, weight_format: int = WEIGHT_BF16,
                 device: torch.device | str | None = None):
        cfg.validate()
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("ListenerEngine runs on a CUDA device (no CPU fallback)")
        self.max_sessions = int(max_sessions)
        self.max_rows = int(max_rows or max_sessions)
        self.max_handles = int(max_handles or max_sessions)
        self.weight_format = int(weight_format)
        self.lib = _lib.load()
        c = _lib.LbConfig()
        c.struct_size = ctypes.sizeof(_lib.LbConfig)
        c.api_version = 1
        c.max_sessions = self.max_sessions
        c.max_handles = self.max_handles
        c.max_rows = self.max_rows
        c.hidden, c.layers, c.heads, c.ffn = cfg.hidden, cfg.layers, cfg.heads, cfg.ffn
        c.sub_ch0, c.sub_ch1 = cfg.sub_ch0, cfg.sub_ch1
        c.output_dims, c.text_hidden = cfg.output_dims, cfg.text_hidden
        c.conv_kernel = cfg.conv_kernel
        c.weight_format = self.weight_format
        c.film_enabled = int(cfg.film_enabled)
        c.film_query_dim, c.film_bottleneck = cfg.film_query_dim, cfg.film_bottleneck
        c.rms_eps, c.softcap, c.invalid_logit = cfg.rms_eps, cfg.softcap, cfg.invalid_logit
        c.gradient_clipping, c.residual_weight = cfg.gradient_clipping, cfg.residual_weight
        c.film_max_scale = cfg.film_max_scale
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check("lb_create", self.lib.lb_create(ctypes.byref(c), ctypes.byref(handle)))
        self._ctx = handle
        self.effective_weights: dict[str, np.ndarray] | None = None
        self.last_rows = 0

    # ------------------------------------------------------------ lifetime
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self.lib.lb_destroy(self._ctx)
            self._ctx = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    @property
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def tensor_names(self) -> list[str]:
        n = self.lib.lb_tensor_count(self._ctx)
        return [self.lib.lb_tensor_name(self._ctx, i).decode() for i in range(n)]

    def load_weights(self, tower: dict[str, np.ndarray], film: dict[str, np.ndarray] | None = None,
                     keep_effective: bool = True) -> None:
        uploads, eff = prepare(self.cfg, tower, film if self.cfg.film_enabled else None, self.weight_format)
        with torch.cuda.device(self.device):
            for name, arr, dtype in uploads:
                a = np.ascontiguousarray(arr)
                rc = self.lib.lb_set_tensor(self._ctx, name.encode(), a.ctypes.data, dtype, a.size)
                _lib.check(f"lb_set_tensor({name})", rc)
            _lib.check("lb_finalize_weights", self.lib.lb_finalize_weights(self._ctx))
        self.effective_weights = eff if keep_effective else None

    # ----------------------------------------------------------- per step
    def pack(self, handles: torch.Tensor, keys: torch.Tensor, frames: torch.Tensor, seqs: torch.Tensor,
             masks: torch.Tensor | None = None) -> None:
        n = int(handles.numel())
        for t, dt in ((handles, torch.int32), (keys, torch.int64), (frames, torch.int64), (seqs, torch.int64)):
            if t.dtype != dt or t.numel() != n or not t.is_contiguous():
                raise ValueError("pack arrays must be contiguous int32 handles and int64 keys/frames/seqs")
        if masks is not None and (masks.dtype != torch.uint8 or masks.numel() != n):
            raise ValueError("masks must be uint8 [n]")
        rc = self.lib.lb_pack_async(self._ctx, n, handles.data_ptr(), keys.data_ptr(), frames.data_ptr(),
                                    seqs.data_ptr(), _ptr(masks), self._stream)
        _lib.check("lb_pack_async", rc)
        self.last_rows = n

    def step(self, inputs: torch.Tensor, *, kind: int = _lib.LB_INPUT_PCM, query: torch.Tensor | None = None,
             want_raw: bool = True, want_soft: bool = True, debug: bool = False):
        """Runs the packed step.  Returns dict of bf16 [n,2,*] tensors (+ debug fp32)."""
        n = self.last_rows
        cfg = self.cfg
        if inputs.dtype != torch.float32 or not inputs.is_contiguous():
            raise ValueError("inputs must be contiguous float32")
        expect = (n, 1280) if kind == _lib.LB_INPUT_PCM else (n, 8, 128)
        if tuple(inputs.shape) != expect:
            raise ValueError(f"inputs must have shape {expect}")
        out = {}
        dev = self.device
        raw = torch.empty((n, 2, cfg.output_dims), dtype=torch.bfloat16, device=dev) if want_raw else None
        soft = torch.empty((n, 2, cfg.text_hidden), dtype=torch.bfloat16, device=dev) if want_soft else None
        film = None
        if query is not None:
            if query.dtype != torch.bfloat16 or tuple(query.shape) != (n, 2, cfg.film_query_dim):
                raise ValueError("query must be bf16 [n,2,film_query_dim]")
            film = torch.empty((n, 2, cfg.film_query_dim), dtype=torch.bfloat16, device=dev)
        dbg_sub = dbg_layers = None
        if debug:
            dbg_sub = torch.empty((n, 2, cfg.hidden), dtype=torch.float32, device=dev)
            dbg_layers = torch.empty((cfg.layers, n, 2, cfg.hidden), dtype=torch.float32, device=dev)
            self.lib.lb_set_debug_outputs(self._ctx, dbg_sub.data_ptr(), dbg_layers.data_ptr())
        try:
            rc = self.lib.lb_step_async(self._ctx, kind, inputs.data_ptr(), _ptr(query), _ptr(raw), _ptr(soft),
                                        _ptr(film), self._stream)
        finally:
            if debug:
                self.lib.lb_set_debug_outputs(self._ctx, None, None)
        _lib.check("lb_step_async", rc)
        out["raw"], out["soft"], out["film"] = raw, soft, film
        if debug:
            out["subsampled"], out["layers"] = dbg_sub, dbg_layers
        return out

    def commit(self) -> None:
        _lib.check("lb_commit_async", self.lib.lb_commit_async(self._ctx, self._stream))

    def abort(self) -> None:
        _lib.check("lb_abort", self.lib.lb_abort(self._ctx))

    def rollback(self) -> None:
        _lib.check("lb_rollback_async", self.lib.lb_rollback_async(self._ctx, self._stream))

    def reset_handle(self, handle: int) -> None:
        _lib.check("lb_reset_handle_async", self.lib.lb_reset_handle_async(self._ctx, int(handle), self._stream))

    def reset_handles(self, handles: torch.Tensor) -> None:
        """Releases every handle of an int32 device tensor in one launch."""
        if handles.dtype != torch.int32 or not handles.is_contiguous() or handles.device != self.device:
            raise ValueError("handles must be a contiguous int32 tensor on the engine's device")
        n = int(handles.numel())
        if n:
            _lib.check("lb_reset_handles_async",
                       self.lib.lb_reset_handles_async(self._ctx, n, handles.data_ptr(), self._stream))

    def reset_slot(self, slot: int) -> None:
        _lib.check("lb_reset_slot_async", self.lib.lb_reset_slot_async(self._ctx, int(slot), self._stream))

    # ------------------------------------------------------------- reads
    def status(self) -> int:
        v = ctypes.c_int32(0)
        _lib.check("lb_get_status", self.lib.lb_get_status(self._ctx, ctypes.addressof(v), self._stream))
        return int(v.value)

    def mel(self, pcm: torch.Tensor, tail_in: torch.Tensor | None, tail_out: torch.Tensor,
            mel_out: torch.Tensor) -> None:
        """lb_mel_async: log-mel of [n,1280] float32 frames with caller-held
        [n,160] tails (None: fresh streams) into [n,8,128]; asynchronous."""
        n = int(pcm.shape[0])
        for t, shape in ((pcm, (n, 1280)), (tail_out, (n, 160)), (mel_out, (n, 8, 128))):
            if t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"mel tensors must be contiguous float32 {shape} on the engine's device")
        if tail_in is not None and (tail_in.dtype != torch.float32 or tuple(tail_in.shape) != (n, 160)
                                    or not tail_in.is_contiguous() or tail_in.device != self.device):
            raise ValueError("tail_in must be a contiguous float32 [n,160] tensor on the engine's device")
        _lib.check("lb_mel_async", self.lib.lb_mel_async(self._ctx, n, pcm.data_ptr(), _ptr(tail_in),
                                                         tail_out.data_ptr(), mel_out.data_ptr(), self._stream))

    def counters(self) -> dict[str, int]:
        """lb_get_counters as a dict (synchronises the current stream)."""
        c = _lib.LbCounters()
        c.struct_size = ctypes.sizeof(_lib.LbCounters)
        c.api_version = 1
        _lib.check("lb_get_counters", self.lib.lb_get_counters(self._ctx, ctypes.byref(c), self._stream))
        return {name: int(getattr(c, name)) for name, _ in _lib.LbCounters._fields_
                if name not in ("struct_size", "api_version", "reserved")}

    def clear_status(self) -> None:
        _lib.check("lb_clear_status", self.lib.lb_clear_status(self._ctx, self._stream))

    def read_rows(self, n: int | None = None) -> tuple[np.ndarray, np.ndarray]:
        n = self.last_rows if n is None else n
        slots = np.zeros(n, np.int32)
        reasons = np.zeros(n, np.int32)
        _lib.check("lb_read_rows", self.lib.lb_read_rows(self._ctx, slots.ctypes.data, reasons.ctypes.data, n,
                                                         self._stream))
        return slots, reasons

    def read_handles(self) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        H = self.max_handles
        slot = np.zeros(H, np.int32)
        key = np.zeros(H, np.int64)
        ef = np.zeros(H, np.int64)
        es = np.zeros(H, np.int64)
        _lib.check("lb_read_handles", self.lib.lb_read_handles(self._ctx, slot.ctypes.data, key.ctypes.data,
                                                               ef.ctypes.data, es.ctypes.data, self._stream))
        return slot, key, ef, es

    def debug_set_expected(self, handle: int, frame: int, seq: int) -> None:
        _lib.check("lb_debug_set_expected",
                   self.lib.lb_debug_set_expected(self._ctx, int(handle), int(frame), int(seq), self._stream))

    # ---------------------------------------------------------- host form
    def step_host(self, handles: np.ndarray, keys: np.ndarray, frames: np.ndarray, seqs: np.ndarray,
                  pcm: np.ndarray, query: np.ndarray | None = None, masks: np.ndarray | None = None,
                  commit: bool = True, out_raw: np.ndarray | None = None, out_soft: np.ndarray | None = None,
                  out_film: np.ndarray | None = None, kind: int = _lib.LB_INPUT_PCM) -> None:
        """End-to-end tick through the C ABI with host buffers (synchronous).

        Output arrays hold bf16 bit patterns (uint16)."""
        n = int(handles.size)
        rc = self.lib.lb_step_host(
            self._ctx, n, handles.ctypes.data, keys.ctypes.data, frames.ctypes.data, seqs.ctypes.data,
            None if masks is None else masks.ctypes.data, kind, pcm.ctypes.data,
            None if query is None else query.ctypes.data,
            None if out_raw is None else out_raw.ctypes.data,
            None if out_soft is None else out_soft.ctypes.data,
            None if out_film is None else out_film.ctypes.data, int(commit), self._stream)
        _lib.check("lb_step_host", rc)
        self.last_rows = n
