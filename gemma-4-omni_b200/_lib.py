"""ctypes binding of liblistener_b200.so (the C ABI declared in include/listener_b200.h).

The library is built in-tree (``build.py``).  There is no fallback: if the
shared object is missing or fails to load, importing the engine raises.
"""
from __future__ import annotations

import ctypes
import functools
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblistener_b200.so"

LB_OK = 0
ERRORS = {
    -1: "invalid argument",
    -2: "CUDA error",
    -3: "invalid state",
    -4: "capacity exceeded",
    -5: "API version mismatch",
    -6: "device status error",
}
LB_F32, LB_BF16, LB_I8, LB_F16 = 0, 1, 2, 3
LB_INPUT_PCM, LB_INPUT_MEL = 0, 1
REASONS = ("continue", "reset", "gap_or_cursor_mismatch", "identity_reset")

DEV_WAIT_TIMEOUT = 1 << 0
DEV_SLOT_EXHAUSTED = 1 << 1
DEV_DUPLICATE_ROW = 1 << 2
DEV_BAD_HANDLE = 1 << 3
DEV_STALE_COMMIT = 1 << 4
DEV_BAD_ROW_COUNT = 1 << 5
DEV_INGRESS_OVERFLOW = 1 << 6
INGRESS_JOIN, INGRESS_LEAVE, INGRESS_PAUSE, INGRESS_RESUME = 0, 1, 2, 3


class LbConfig(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("api_version", ctypes.c_uint32),
        ("max_sessions", ctypes.c_int32),
        ("max_handles", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("layers", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("ffn", ctypes.c_int32),
        ("sub_ch0", ctypes.c_int32),
        ("sub_ch1", ctypes.c_int32),
        ("output_dims", ctypes.c_int32),
        ("text_hidden", ctypes.c_int32),
        ("conv_kernel", ctypes.c_int32),
        ("weight_format", ctypes.c_int32),
        ("film_enabled", ctypes.c_int32),
        ("film_query_dim", ctypes.c_int32),
        ("film_bottleneck", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("softcap", ctypes.c_float),
        ("invalid_logit", ctypes.c_float),
        ("gradient_clipping", ctypes.c_float),
        ("residual_weight", ctypes.c_float),
        ("film_max_scale", ctypes.c_float),
    ]


class LbCounters(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("api_version", ctypes.c_uint32)] + [
        (n, ctypes.c_uint64) for n in (
            "packs", "steps", "commits", "aborts", "rollbacks", "resets", "rows_stepped", "rows_continue",
            "rows_reset", "rows_gap_or_cursor_mismatch", "rows_identity_reset", "rows_committed",
            "stale_commits")] + [
        (n, ctypes.c_int32) for n in ("status", "status_history", "graphs_captured", "reserved")]


P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64

# name -> (restype, argtypes); every symbol include/listener_b200.h declares
SIGNATURES: dict[str, tuple] = {
    "lb_create": (I, [ctypes.POINTER(LbConfig), ctypes.POINTER(P)]),
    "lb_destroy": (I, [P]),
    "lb_set_tensor": (I, [P, ctypes.c_char_p, P, I, I64]),
    "lb_finalize_weights": (I, [P]),
    "lb_tensor_count": (I, [P]),
    "lb_tensor_name": (ctypes.c_char_p, [P, I]),
    "lb_pack_async": (I, [P, I, P, P, P, P, P, P]),
    "lb_step_async": (I, [P, I, P, P, P, P, P, P]),
    "lb_step_host": (I, [P, I, P, P, P, P, P, I, P, P, P, P, P, I, P]),
    "lb_set_debug_outputs": (I, [P, P, P]),
    "lb_commit_async": (I, [P, P]),
    "lb_abort": (I, [P]),
    "lb_rollback_async": (I, [P, P]),
    "lb_reset_handle_async": (I, [P, I, P]),
    "lb_reset_slot_async": (I, [P, I, P]),
    "lb_get_status": (I, [P, P, P]),
    "lb_clear_status": (I, [P, P]),
    "lb_read_rows": (I, [P, P, P, I, P]),
    "lb_read_handles": (I, [P, P, P, P, P, P]),
    "lb_debug_set_expected": (I, [P, I, I64, I64, P]),
    "lb_debug_set_stop": (I, [P, I, I]),
    "lb_step_kernel_count": (I, [P]),
    "lb_debug_read_buffer": (I, [P, ctypes.c_char_p, P, ctypes.c_size_t, P]),
    "lb_get_counters": (I, [P, ctypes.POINTER(LbCounters), P]),
    "lb_mel_async": (I, [P, I, P, P, P, P, P]),
    "lb_op_control6_head": (I, [I, P, I, P, P, P, P, P, I, ctypes.c_float, P, P, P]),
    "lb_ingress_create": (I, [I, I, I, ctypes.POINTER(P)]),
    "lb_ingress_destroy": (I, [P]),
    "lb_ingress_events_async": (I, [P, I, P, P, P, P]),
    "lb_ingress_push_async": (I, [P, I, P, P, P, P, P]),
    "lb_ingress_tick_async": (I, [P, I64, P, P, P, P, P, P]),
    "lb_ingress_get_status": (I, [P, P, P]),
    "lb_film_talker_async": (I, [P, I, P, I, P, P, P, P, P]),
    "lb_reset_handles_async": (I, [P, I, P, P]),
    "lb_op_gemm": (I, [P, I, I, P, I, P, P, I, I, P, I, I, I, I, P, P]),
    "lb_op_gemm_clipped": (I, [P, I, I, I, P, I, P, P, I, I, P, I, I, I, I, I, P, P, P, P, P]),
    "lb_op_gemm_splitk_scratch": (I, [P, I, I, P, I, P, P, I, I, P, I, I, I, P, P]),
    "lb_snapshot_ready_rows": (I, [I, P, P, P, P, P, P, P, I64, P, P, P, P, P]),
    "lb_order_ready_heads": (I, [I, P, P, P, I64, I64, I, P, P, P, P]),
}


class ListenerLibError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {ERRORS.get(code, code)} ({code})")
        self.code = code


@functools.lru_cache(maxsize=1)
def load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built; run `python gemma-4-omni_b200/build.py` "
            "(the listener step has no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def check(fn: str, code: int) -> None:
    if code != LB_OK:
        raise ListenerLibError(fn, code)
