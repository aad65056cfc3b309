"""Loads libkd_b200.so (built in-tree by ``build.py``) and declares the C ABI of ``include/kd_b200.h`` for ctypes.

There is no fallback: a missing or unloadable library raises at import of the ops that need it, so no CPU or
library path ever answers in its place.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libkd_b200.so"

KD_OK = 0
KD_DEVICE_TIMEOUT = 1
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_GEGLU = 0, 1, 2, 3
NORM_NONE, NORM_WEIGHT, NORM_ONE_PLUS = 0, 1, 2

P = c_void_p
#: Every exported entry point: name -> argument types (all return int).
SIGNATURES: dict[str, list] = {
    "kd_version": [],
    "kd_last_error": [ctypes.c_char_p, c_size_t],
    "kd_wait_selftest": [P, c_int64, P, P],
    "kd_gemm_bf16": [P, c_int64, P, c_int64, P, c_int64, P, c_int64, c_int, c_int, c_int, c_int, P, P],
    "kd_gemm_fp8": [P, c_int64, P, P, c_int64, P, P, c_int64, P, c_int64, c_int, c_int, c_int, c_int, P, P],
    "kd_qkv_projection": [P, c_int64, P, c_int64, c_int, c_int, c_int, P, c_int, c_int, c_int, c_int, P, P, c_int,
                          c_int, c_float, P, c_int, P, P, P, P, P, P],
    "kd_qkv_projection_fp8": [P, c_int64, P, P, c_int64, P, c_int, c_int, c_int, P, c_int, c_int, c_int, c_int, P, P,
                              c_int, c_int, c_float, P, c_int, P, P, P, P, P, P],
    "kd_rope_gather": [P, c_int64, P, P, c_int64, c_int, P, P],
    "kd_qkv_projection_noalloc": [P, c_int64, P, c_int64, c_int, c_int, c_int, P, c_int, c_int, c_int, c_int, P, P,
                                  c_int, c_int, c_float, P, P, c_int64, c_int, P, P, P, P, P, P],
    "kd_embed": [P, c_int64, P, c_int64, c_int, c_float, P, P],
    "kd_rmsnorm": [P, c_int64, P, c_int, c_float, P, c_int64, c_int64, c_int, P],
    "kd_add_rmsnorm": [P, P, P, c_int, c_float, P, c_int64, c_int, P],
    "kd_norm_add": [P, P, P, c_int, c_float, P, P, c_int64, c_int, P],
    "kd_rmsnorm_e4m3": [P, c_int64, P, c_int, c_float, P, P, c_int64, c_int, P],
    "kd_quantize_rows_e4m3": [P, c_int64, c_int, P, P, P],
    "kd_rope_table": [P, c_int, c_int64, P, P, P],
    "kd_rope_table_axes": [P, c_int, P, c_int64, c_int64, P, c_int, P, P, P],
    "kd_qkv_norm_rope": [P, c_int64, c_int64, P, c_int, c_int, c_int, c_int, P, P, c_int, c_int, c_float, P, P,
                         c_int, P, P, P, P, P],
    "kd_attention_varlen": [P, c_int64, P, c_int64, P, c_int64, P, c_int64, P, c_int64, P, P, c_int, c_int, c_int64,
                            c_int64, c_int, c_int, c_int, c_float, c_int, c_int, P, P, P],
    "kd_gather_rows": [P, c_int64, P, c_int64, c_int, P, c_int64, P],
    "kd_scatter_rows": [P, c_int64, P, c_int64, c_int, P, c_int64, P],
    "kd_conv_silu": [P, c_int64, c_int64, c_int, P, c_int, P, P, c_int64, P],
    "kd_gated_delta_rule": [P, c_int64, P, c_int64, P, P, P, c_int, c_int64, c_int, c_int, c_int, c_int, P, c_int64,
                            P, P],
    "kd_gated_norm": [P, c_int64, P, c_int64, P, c_int64, c_int, c_int, c_float, P, c_int64, P],
    "kd_marker_norm": [P, c_int, P, c_int64, P, c_int, c_float, P, P],
    "kd_readout": [P, c_int64, c_int, P, c_int, c_float, P, P],
}

_lib: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A libkd_b200 entry point rejected its arguments or failed to launch."""


def load() -> ctypes.CDLL:
    """The loaded library with every entry point's argument types declared."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise KernelError(f"{LIBRARY} is missing: build it with python -m karpo_decision_b200.build")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is not None:  # a missing export fails the call that needs it (and the ABI test)
                fn.argtypes = args
                fn.restype = c_int
        _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().kd_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


_profiler = None


def set_profiler(profiler) -> None:
    """Installs (or removes, with None) the per-launch event recorder of ``profile.kernels``."""
    global _profiler
    _profiler = profiler


def call(name: str, *args) -> None:
    """Calls entry point ``name``; raises KernelError with the library's message on a non-zero status."""
    fn = getattr(load(), name)
    prof = _profiler
    if prof is None:
        rc = fn(*args)
    else:
        token = prof.before(name, args)
        rc = fn(*args)
        prof.after(name, args, token)
    if rc != KD_OK:
        raise KernelError(f"{name} failed ({rc}): {last_error()}")
