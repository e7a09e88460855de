"""ctypes binding of the C ABI in ``include/ravel_b200.h``.

The shared library ``libravel_b200.so`` sits next to this file (built by
``ravel_lm_b200.build``).  Loading it needs no GPU; calling a compute entry
point does.  There is no fallback: if the library is missing, every operator
raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Callable, Optional

_LIB_PATH = Path(__file__).resolve().parent / "libravel_b200.so"

RAVEL_OK = 0
RAVEL_ERR_INVALID_ARG = 1
RAVEL_ERR_WORKSPACE = 2
RAVEL_ERR_CUDA = 3
RAVEL_ERR_UNSUPPORTED = 4
RAVEL_ERR_DEVICE = 5

RAVEL_F32, RAVEL_BF16, RAVEL_F16, RAVEL_F64 = 0, 1, 2, 3
RAVEL_I32, RAVEL_I64 = 0, 1
RAVEL_TAPE_GENERAL_READS = 1
RAVEL_TAPE_WRITE_MASK = 2
RAVEL_NOALLOC_SCRATCH_BYTES = 32 << 20
RAVEL_DEVERR_SPIN = 1

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_sz = ctypes.c_size_t

# name -> (restype, argtypes); the order follows include/ravel_b200.h
SIGNATURES = {
    "ravel_tape_bytes": (_c_sz, [_c_i64, _c_i64, _c_i64, _c_i64, _c_int]),
    "ravel_scratch_bytes": (_c_sz, [_c_i64] * 6 + [_c_int, _c_int]),
    "ravel_tape_build": (_c_int, [_c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int,
                                  _c_vp, _c_sz, _c_vp, _c_sz, _c_vp]),
    "ravel_latestk_fwd_tape": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 6 +
                               [_c_vp, _c_vp, _c_vp]),
    "ravel_latestk_fwd": (_c_int, [_c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_int] + [_c_i64] * 6 +
                          [_c_vp, _c_vp, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp]),
    "ravel_latestk_bwd": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 6 +
                          [_c_vp, _c_vp, _c_sz, _c_vp]),
    "ravel_latestk_bwd_accumulate": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 6 +
                                     [_c_vp, _c_vp, _c_sz, _c_vp]),
    "ravel_segsum_fwd_tape": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 5 +
                              [_c_vp, _c_vp, _c_vp, _c_sz, _c_vp]),
    "ravel_segsum_fwd": (_c_int, [_c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_int] + [_c_i64] * 5 +
                         [_c_vp, _c_vp, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp]),
    "ravel_segsum_bwd": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 5 +
                         [_c_vp, _c_vp, _c_sz, _c_vp]),
    "ravel_segsum_fwd_noalloc": (_c_int, [_c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_int] + [_c_i64] * 5 +
                                 [_c_vp, _c_vp, _c_vp]),
    "ravel_cache_read": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_int] + [_c_i64] * 4 + [_c_vp, _c_vp, _c_vp]),
    "ravel_cache_write": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 4 + [_c_vp]),
    "ravel_cache_step": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 4 +
                         [_c_vp, _c_vp, _c_vp]),
    "ravel_cache_prefill_scratch_bytes": (ctypes.c_size_t, [_c_i64] * 4),
    "ravel_cache_prefill": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 5 +
                            [_c_vp, ctypes.c_size_t, _c_vp]),
    "ravel_literal_addresses": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_i64, _c_i64, _c_vp, _c_vp]),
    "ravel_tape_build_tokens": (_c_int, [_c_vp, _c_int, _c_i64, _c_vp, _c_vp, _c_int, _c_vp] + [_c_i64] * 4 +
                                [_c_int, _c_vp, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp]),
    "ravel_latestk_sources": (_c_int, [_c_vp, _c_int, _c_vp, _c_int] + [_c_i64] * 5 + [_c_vp, _c_vp]),
    "ravel_gather_gemm": (_c_int, [_c_vp, _c_vp, _c_vp] + [_c_i64] * 5 + [_c_vp, _c_i64] + [_c_vp] * 5),
    "ravel_gather_rows": (_c_int, [_c_vp, _c_vp, _c_vp] + [_c_i64] * 5 + [_c_vp, _c_vp]),
    "ravel_gate_residual_fwd": (_c_int, [_c_vp] * 4 + [_c_i64, _c_int, _c_vp]),
    "ravel_gate_residual_bwd": (_c_int, [_c_vp] * 5 + [_c_i64, _c_int, _c_vp]),
    "ravel_rms_norm_fwd": (_c_int, [_c_vp, _c_vp, ctypes.c_float, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_vp]),
    "ravel_rms_norm_scratch_bytes": (_c_sz, [_c_i64, _c_i64]),
    "ravel_rms_norm_bwd": (_c_int, [_c_vp] * 6 + [_c_i64, _c_i64, _c_int, _c_vp, _c_sz, _c_vp]),
    "ravel_set_wait_limit": (_c_int, [ctypes.c_uint32]),
    "ravel_wait_selftest": (_c_int, [_c_vp, _c_vp]),
    "ravel_device_error": (_c_int, [ctypes.POINTER(_c_int), _c_vp]),
    "ravel_clear_device_error": (_c_int, [_c_vp]),
    "ravel_kernel_launches": (ctypes.c_uint64, []),
    "ravel_timing_start": (_c_int, [_c_i64]),
    "ravel_timing_stop": (_c_int, []),
    "ravel_timing_count": (_c_i64, []),
    "ravel_timing_read": (_c_int, [_c_i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_float)]),
    "ravel_status_string": (ctypes.c_char_p, [_c_int]),
    "ravel_version": (ctypes.c_char_p, []),
}

_lib: Optional[ctypes.CDLL] = None

# Optional observer of every compute call: fn(name, call) -> result (used by
# tests to see which entry points a Python call reaches).  While one is set the
# per-step paths go through it instead of their direct calls.
_call_hook: Optional[Callable] = None

# The C++ host extension (``_ravel_host``): the per-step calls of the Python
# API -- argument checks, output allocation, the C-ABI call -- without ctypes.
_host = None


class RavelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, status: int):
        self.status = status
        msg = load().ravel_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"{name} failed: {msg} (status {status})")


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load ``libravel_b200.so``; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise RuntimeError(
            f"ravel_lm_b200: CUDA library {_LIB_PATH.name} is not built; run "
            "`python -m ravel_lm_b200.build` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(name: str, status: int) -> None:
    if status == RAVEL_OK:
        return
    if status in (RAVEL_ERR_INVALID_ARG, RAVEL_ERR_UNSUPPORTED):
        err = RavelError(name, status)
        raise ValueError(str(err))
    raise RavelError(name, status)


_fns: dict = {}


def call(name: str, *args) -> None:
    """Call a status-returning entry point, raising on failure."""
    fn = _fns.get(name)
    if fn is None:
        fn = _fns[name] = getattr(load(), name)
    if _call_hook is not None:
        status = _call_hook(name, lambda: fn(*args))
    else:
        status = fn(*args)
    if status:
        check(name, status)


def host():
    """The C++ host extension, next to the library (built with it); raise if it has not been built."""
    global _host
    if _host is not None:
        return _host
    load()  # the extension links against the library: load it from its own path first
    try:
        from . import _ravel_host
    except ImportError as e:
        raise RuntimeError("ravel_lm_b200: host extension _ravel_host is not built; run "
                           "`python -m ravel_lm_b200.build`") from e
    _host = _ravel_host
    return _host


def run(name: str, fn: Callable, *args):
    """Call a host-extension function that returns (status, *outputs); raise on failure."""
    if _call_hook is not None:
        res = _call_hook(name, lambda: fn(*args))
    else:
        res = fn(*args)
    if res[0]:
        check(name, res[0])
    return res


def set_call_hook(hook: Optional[Callable]) -> None:
    global _call_hook
    _call_hook = hook


def device_error(stream: int) -> int:
    """Device error bits (RAVEL_DEVERR_*) after the work queued on ``stream``."""
    out = _c_int(0)
    check("ravel_device_error", load().ravel_device_error(ctypes.byref(out), stream))
    return int(out.value)


def kernel_launches() -> int:
    """Kernels launched by the library in this process so far."""
    return int(load().ravel_kernel_launches())


def clear_device_error(stream: int) -> None:
    check("ravel_clear_device_error", load().ravel_clear_device_error(stream))


def timing_start(max_records: int) -> None:
    """Record the GPU time of every compute entry point (up to ``max_records`` calls), natively."""
    check("ravel_timing_start", load().ravel_timing_start(int(max_records)))


def timing_stop() -> list:
    """Stop recording; return [(entry point name, milliseconds)] in call order (waits for the GPU)."""
    lib = load()
    check("ravel_timing_stop", lib.ravel_timing_stop())
    out = []
    name, ms = ctypes.c_char_p(), ctypes.c_float()
    for i in range(int(lib.ravel_timing_count())):
        rc = lib.ravel_timing_read(i, ctypes.byref(name), ctypes.byref(ms))
        if rc == RAVEL_OK:
            out.append((name.value.decode(), float(ms.value)))
        elif rc != RAVEL_ERR_INVALID_ARG:  # a record whose end was never enqueued is skipped
            check("ravel_timing_read", rc)
    return out
