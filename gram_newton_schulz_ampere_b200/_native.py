"""ctypes binding of the C ABI in ``include/gns_b200.h`` (``lib/libgns_b200.so``).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises. Calls pass raw device pointers and the current torch CUDA
stream; torch owns every allocation (outputs and workspaces).
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_double, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgns_b200.so"

F16, BF16, F32 = 0, 1, 2
DTYPE_CODES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

ERROR_NAMES = {
    -1: "argument",
    -2: "layout",
    -3: "workspace",
    -4: "cuda",
    -5: "device",
    -6: "unsupported",
}

_P = c_void_p
_I64 = c_int64
_PP = ctypes.POINTER(c_void_p)
_PI64 = ctypes.POINTER(c_int64)
_PF = ctypes.POINTER(c_float)

# name -> (restype, argtypes); mirrors include/gns_b200.h exactly.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "gns_version": (c_int, []),
    "gns_last_error": (ctypes.c_char_p, []),
    "gns_device_status": (c_int, [ctypes.POINTER(c_int), c_int]),
    "gns_profile_enable": (c_int, [c_int]),
    "gns_profile_collect": (
        c_int,
        [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_float), ctypes.POINTER(c_double), ctypes.POINTER(c_int)],
    ),
    "gns_gemm": (
        c_int,
        [c_int, _I64, _I64, _I64, _I64,
         _P, _I64, _I64, _I64,
         _P, _I64, _I64, _I64,
         _P, c_int, _I64, _I64,
         _P, c_int, _I64, _I64,
         c_float, c_float, c_int, _P],
    ),
    "gns_normalize_workspace_size": (c_size_t, [_I64, _I64, _I64]),
    "gns_frobenius_normalize": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, _I64, c_float, _P, c_size_t, _P],
    ),
    "gns_frobenius_normalize_noalloc": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, _I64, c_float, _P],
    ),
    "gns_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_ulonglong)]),
    "gns_selftest_normalize_timeout": (c_int, [_I64, _I64, _I64, _P, _P, _P, c_size_t, _P]),
    "gns_newton_schulz_workspace_size": (c_size_t, [_I64, _I64, _I64]),
    "gns_gram_newton_schulz": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, c_int, _I64, _I64,
         ctypes.POINTER(c_double), c_int, c_uint32, c_float, _P, c_size_t, _P],
    ),
    "gns_standard_newton_schulz": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, c_int, _I64, _I64,
         ctypes.POINTER(c_double), c_int, c_float, _P, c_size_t, _P],
    ),
    "gns_set_small_chain": (c_int, [c_int]),
    "gns_set_gemm_sm_limit": (c_int, [c_int]),
    "gns_frobenius_sumsq": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, c_size_t, _P],
    ),
    "gns_frobenius_scale": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _I64, _I64, _P, c_float, _P, _I64, _P],
    ),
    "gns_gram_iterations_workspace_size": (c_size_t, [_I64, _I64]),
    "gns_gram_iterations": (
        c_int,
        [_I64, _I64, _P, c_int, _I64, _I64, ctypes.POINTER(c_double), c_int, c_int, c_int,
         _P, _I64, _I64, _P, c_size_t, _P],
    ),
    "gns_muon_momentum": (
        c_int,
        [c_int, _PP, _PP, _PP, _PI64, c_int, c_int, c_int, c_float, c_int, _P],
    ),
    "gns_muon_apply": (
        c_int,
        [c_int, _PP, _PP, _PI64, c_int, c_int, c_float, c_int, _PF, _P],
    ),
    "gns_dion3_select_workspace_size": (c_size_t, [_I64, _I64]),
    "gns_dion3_select_rows": (
        c_int,
        [c_int, _I64, _I64, _I64, _P, _P, _P, _I64, c_float, c_float, _P, _P, _P, c_size_t, _P],
    ),
    "gns_dion3_select_rows_multi": (
        c_int,
        [c_int, c_int, _I64, _I64, _PP, _PP, _PP, _I64, c_float, c_float, _P, _P, _P, c_size_t, _P],
    ),
    "gns_dion3_normalize_workspace_size": (c_size_t, [_I64, _I64]),
    "gns_dion3_normalize_apply_multi": (
        c_int,
        [c_int, c_int, c_int, _I64, _I64, _I64, _PP, _P, _I64, _I64, _PP, _P,
         c_float, c_float, c_float, c_float, c_float, _P, c_size_t, _P],
    ),
    "gns_dion3_normalize_apply": (
        c_int,
        [c_int, c_int, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _P, _P,
         c_float, c_float, c_float, c_float, c_float, _P, c_size_t, _P],
    ),
    "gns_adamw_step": (
        c_int,
        [c_int, _PP, _PP, _PP, _PP, _PI64, c_int, c_int, c_int, _PF, _PF, c_float, c_float, c_float, c_float,
         c_float, c_float, c_int, _P],
    ),
    "gns_lion_step": (
        c_int,
        [c_int, _PP, _PP, _PP, _PI64, c_int, c_int, c_int, c_float, c_float, c_float, c_float, c_float, c_float,
         c_int, _P],
    ),
    "gns_dion3_normalize_rows": (
        c_int,
        [c_int, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, c_float, c_float, _P, _P, _P, c_size_t, _P],
    ),
    "gns_dion3_apply_rows": (
        c_int,
        [c_int, _I64, _I64, _I64, _I64, _P, _P, _P, _P, c_float, c_float, c_float, c_float, _P],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def library_path() -> Path:
    override = os.environ.get("GNS_B200_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Loads the shared library (once). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"gram_newton_schulz_ampere_b200 native library not found at {path}; "
                "build it with `python -m gram_newton_schulz_ampere_b200.build`"
            )
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().gns_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        kind = ERROR_NAMES.get(rc, str(rc))
        raise NativeError(f"{what} failed ({kind}): {last_error()}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {dtype}; expected float16, bfloat16 or float32") from exc


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(clear: bool = True) -> int:
    status = c_int(0)
    check(load().gns_device_status(ctypes.byref(status), 1 if clear else 0), "gns_device_status")
    return int(status.value)


def set_wait_limit_ns(limit_ns: int) -> int:
    """Sets the normalisation's bounded-wait limit; returns the previous one."""
    previous = ctypes.c_ulonglong(0)
    check(load().gns_set_wait_limit_ns(int(limit_ns), ctypes.byref(previous)), "gns_set_wait_limit_ns")
    return int(previous.value)


def profile_enable(capacity: int) -> None:
    check(load().gns_profile_enable(int(capacity)), "gns_profile_enable")


def profile_collect(capacity: int) -> list[tuple[float, float, int]]:
    """(milliseconds, algorithmic flops, symmetric) for each recorded GEMM launch."""
    n = c_int(0)
    ms = (c_float * max(capacity, 1))()
    fl = (c_double * max(capacity, 1))()
    sym = (c_int * max(capacity, 1))()
    check(load().gns_profile_collect(int(capacity), ctypes.byref(n), ms, fl, sym), "gns_profile_collect")
    return [(float(ms[i]), float(fl[i]), int(sym[i])) for i in range(n.value)]


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
