"""ctypes binding of ``libkda_b200.so`` (declarations: ``include/kda_b200.h``).

The library is loaded from the package directory.  There is no fallback: if
the library is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p, c_char_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkda_b200.so"

KDA_OK = 0
KDA_ERR_INVALID = 1
KDA_ERR_UNSUPPORTED = 2
KDA_ERR_CUDA = 3

# every symbol the header declares, with its ctypes signature
SIGNATURES = {
    "kda_b200_version": ([], c_char_p),
    "kda_b200_last_error": ([], c_char_p),
    "kda_b200_saved_bytes": ([c_int64, c_int, c_int, c_int], c_size_t),
    "kda_b200_fwd_workspace_bytes": ([c_int64, c_int, c_int, c_int, c_int], c_size_t),
    "kda_b200_bwd_workspace_bytes": ([c_int64, c_int, c_int, c_int], c_size_t),
    "kda_b200_fwd": ([c_void_p] * 12 + [c_int] * 5 + [c_float, c_float]
                     + [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p], c_int),
    "kda_b200_bwd": ([c_void_p] * 12 + [c_int] * 5 + [c_float, c_float]
                     + [c_void_p, c_size_t] + [c_void_p] * 13 + [c_void_p, c_size_t, c_void_p], c_int),
    "kda_b200_f32_saved_bytes": ([c_int64, c_int, c_int], c_size_t),
    "kda_b200_f32_fwd_workspace_bytes": ([c_int64, c_int, c_int, c_int], c_size_t),
    "kda_b200_f32_bwd_workspace_bytes": ([c_int64, c_int, c_int], c_size_t),
    "kda_b200_fwd_f32": ([c_void_p] * 12 + [c_int] * 5 + [c_float, c_float]
                         + [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p], c_int),
    "kda_b200_bwd_f32": ([c_void_p] * 12 + [c_int] * 5 + [c_float, c_float]
                         + [c_void_p, c_size_t] + [c_void_p] * 13 + [c_void_p, c_size_t, c_void_p], c_int),
    "kda_b200_recurrent": ([c_void_p] * 9 + [c_int] * 6 + [c_float, c_float] + [c_void_p] * 3, c_int),
    "kda_b200_decode": ([c_void_p] * 13 + [c_int] * 6 + [c_float, c_float] + [c_void_p] * 3, c_int),
    "kda_b200_doc_cu_seqlens": ([c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p], c_int),
    "kda_b200_chunk_table": ([c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p, c_void_p], c_int),
    "kda_b200_device_error": ([c_int], c_int),
    "kda_b200_debug_set_input_wait_polls": ([ctypes.c_uint], c_int),
    "kda_b200_debug_set_state_wait": ([ctypes.c_uint, c_int], c_int),
    "kda_b200_fwd_noalloc": ([c_void_p] * 12 + [c_int] * 5 + [c_float, c_float] + [c_void_p, c_void_p, c_void_p],
                             c_int),
    "kda_b200_timing_enable": ([c_int], c_int),
    "kda_b200_timing_reset": ([], c_int),
    "kda_b200_timing_read": ([c_int, c_void_p, c_void_p, c_void_p], c_int),
    "kda_b200_gated_norm_workspace_bytes": ([c_int64, c_int], c_size_t),
    "kda_b200_gated_norm_fwd": ([c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int, c_void_p, c_void_p],
                                c_int),
    "kda_b200_gated_norm_bwd": ([c_void_p] * 4 + [c_int64, c_int, c_float, c_int] + [c_void_p] * 4
                                + [c_size_t, c_void_p], c_int),
}

_lib = None


class KdaError(RuntimeError):
    """A non-OK status from the CUDA library."""


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"KDA CUDA library not built ({LIB_PATH}); run `python -m sophia_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc == KDA_OK:
        return
    msg = load().kda_b200_last_error().decode()
    if rc in (KDA_ERR_INVALID,):
        raise ValueError(msg)
    if rc == KDA_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise KdaError(msg)


def timing_enable(on: bool) -> None:
    load().kda_b200_timing_enable(int(on))


def timing_reset() -> None:
    load().kda_b200_timing_reset()


def timing_read() -> dict[str, tuple[int, float]]:
    """{kernel name: (launches, total ms)} since the last reset."""
    n = 32
    names = (ctypes.c_char_p * n)()
    launches = (ctypes.c_int * n)()
    ms = (ctypes.c_float * n)()
    rc = load().kda_b200_timing_read(n, ctypes.cast(names, c_void_p), ctypes.cast(launches, c_void_p),
                                     ctypes.cast(ms, c_void_p))
    if rc <= 0:
        raise KdaError(load().kda_b200_last_error().decode())
    return {names[i].decode(): (launches[i], ms[i]) for i in range(rc)}


def device_error(reset: bool = True) -> int:
    """Nonzero when a tensor-core kernel hit a bounded-wait timeout (synchronises)."""
    return int(load().kda_b200_device_error(int(reset)))
