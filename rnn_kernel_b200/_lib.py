"""ctypes binding of ``librnn_kernel_b200.so`` (the C ABI in ``include/rnn_kernel_b200.h``).

The library is built in-tree by :mod:`rnn_kernel_b200.build`.  Loading it does
not need a GPU; calling any compute entry point does.  There is no fallback:
if the library is missing the call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

# status codes of include/rnn_kernel_b200.h
GRU_OK = 0
GRU_ERR_INVALID = 1
GRU_ERR_CUDA = 2
GRU_ERR_UNSUPPORTED = 3

_lock = threading.Lock()
_lib = None

_c_float_p = ctypes.c_void_p
_size_t = ctypes.c_size_t
_int = ctypes.c_int

# name -> (restype, argtypes); mirrors include/rnn_kernel_b200.h
SIGNATURES = {
    "gru_last_error": (ctypes.c_char_p, []),
    "gru_device_supported": (_int, [_int]),
    "gru_stash_bytes": (_size_t, [_int, _int, _int]),
    "gru_forward_workspace_bytes": (_size_t, [_int, _int, _int, _int]),
    "gru_backward_workspace_bytes": (_size_t, [_int, _int, _int, _int]),
    "gru_forward": (_int, [_c_float_p] * 9 + [ctypes.c_void_p, _size_t] + [_int] * 4 + [ctypes.c_void_p]),
    "gru_backward": (_int, [_c_float_p] * 12 + [ctypes.c_void_p, _size_t] + [_int] * 4 + [ctypes.c_void_p]),
    "gru_forward_inference_noalloc": (_int, [_c_float_p] * 8 + [_int] * 4 + [ctypes.c_void_p]),
    "gru_device_status": (_int, [_int]),
    "gru_selftest_wait_timeout": (_int, [_int, ctypes.c_void_p, ctypes.c_void_p]),
    "gru_launch_count": (ctypes.c_ulonglong, []),
    "gru_set_time_chunks": (_int, [_int]),
    "gru_set_small_loops": (_int, [_int]),
    "gru_mse_workspace_bytes": (_size_t, [ctypes.c_long]),
    "gru_mse_loss": (_int, [_c_float_p, _c_float_p, ctypes.c_long, _c_float_p, ctypes.c_void_p, _size_t,
                            ctypes.c_void_p]),
    "gru_mse_loss_backward": (_int, [_c_float_p, _c_float_p, _c_float_p, _c_float_p, ctypes.c_long, ctypes.c_void_p]),
    "gru_timing_enable": (_int, [_int]),
    "gru_timing_collect": (_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int), _int]),
}

KERNEL_KINDS = ("input_gemm", "fwd_recurrent", "bwd_recurrent", "grad_gemm", "colsum", "layout", "loss")


def timing_enable(on: bool) -> None:
    load().gru_timing_enable(1 if on else 0)


def timing_collect() -> dict:
    """Per kernel kind: (total device ms, timed launches) since the last collect."""
    n = len(KERNEL_KINDS)
    tot = (ctypes.c_double * n)()
    cnt = (ctypes.c_int * n)()
    check(load().gru_timing_collect(tot, cnt, n), "gru_timing_collect")
    return {k: (tot[i], cnt[i]) for i, k in enumerate(KERNEL_KINDS)}


def device_status(reset: bool = False) -> int:
    """The device status word (0 = every bounded wait completed); synchronises."""
    st = load().gru_device_status(1 if reset else 0)
    if st < 0:
        raise RuntimeError(f"gru_device_status failed: {last_error()}")
    return st


def set_time_chunks(n: int) -> int:
    """Time chunks of the forward/backward (0 automatic, 1 off, 2..4 forced
    where the shape allows); returns the previous setting."""
    prev = load().gru_set_time_chunks(int(n))
    if prev < 0:
        raise ValueError(f"time chunks must be 0..4, got {n}")
    return prev


def set_small_loops(mode: int) -> int:
    """Time-loop kernels for H <= 96: 0 single-CTA (default), 1 cluster;
    returns the previous mode."""
    prev = load().gru_set_small_loops(int(mode))
    if prev < 0:
        raise ValueError(f"small-loops mode must be 0 or 1, got {mode}")
    return prev


def launch_count() -> int:
    return int(load().gru_launch_count())


TIMELINE_POINTS = {
    "fwd": ("step_start", "wait_done", "product_done", "barrier_done", "partials_summed", "gates_done",
            "sent", "stored", "step_end", "prefetch_issued"),
    "bwd": ("step_start", "copies_waited", "wait_done", "barrier1_done", "dh_summed", "pointwise_done",
            "dG_stored", "db_added", "barrier2_done", "product_done", "sent", "step_end"),
}


def timeline_read():
    """Step timeline of an instrumented build (RNN_KERNEL_B200_VARIANT=timeline):
    int64 clock64 values [direction (fwd, bwd)][CTA 0 thread 0, CTA 0 last
    thread, CTA 1 thread 0, CTA 1 last thread][step][point] of the last
    launch of each time loop (points: TIMELINE_POINTS; 0 = not recorded)."""
    import numpy as np

    lib = load()
    fn = getattr(lib, "gru_timeline_read", None)
    if fn is None:
        raise RuntimeError("this library was built without the step timeline "
                           "(set RNN_KERNEL_B200_VARIANT=timeline)")
    fn.restype = _int
    fn.argtypes = [ctypes.c_void_p]
    buf = np.zeros((2, 4, 8, 12), dtype=np.int64)
    check(fn(buf.ctypes.data), "gru_timeline_read")
    return buf


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed and possible) the CUDA library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if build_if_missing and _build.needs_build():
            _build.build()
        if not path.exists():
            raise RuntimeError(f"rnn_kernel_b200 CUDA library not found at {path}; run "
                               "`python -m rnn_kernel_b200.build`")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().gru_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what} failed (status {status}): {last_error()}")
