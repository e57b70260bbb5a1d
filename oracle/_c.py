"""TEST INFRASTRUCTURE ONLY: ctypes loader of the oracle's C helpers (oracle/c/oracle_c.c), built by oracle/Makefile."""

import ctypes
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SO = _HERE / "_build" / "liboracle_c.so"
_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        if not _SO.exists():
            subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
        L = ctypes.CDLL(str(_SO))
        L.oracle_fold_group.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 2
        L.oracle_fmaf.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64]
        _LIB = L
    return _LIB


def fold_group(part: np.ndarray, s: np.ndarray, acc: np.ndarray):
    """acc = fmaf(float(part), s[:, None], acc) in place (int32 [M, N], fp32 [M], fp32 [M, N])."""
    assert part.dtype == np.int32 and s.dtype == np.float32 and acc.dtype == np.float32
    part, s = np.ascontiguousarray(part), np.ascontiguousarray(s)
    assert acc.flags.c_contiguous
    M, N = part.shape
    lib().oracle_fold_group(part.ctypes.data, s.ctypes.data, acc.ctypes.data, M, N)


def fmaf(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    a, b, c = (np.ascontiguousarray(np.broadcast_to(v, np.broadcast(a, b, c).shape), dtype=np.float32)
               for v in (a, b, c))
    out = np.empty_like(a)
    lib().oracle_fmaf(a.ctypes.data, b.ctypes.data, c.ctypes.data, out.ctypes.data, a.size)
    return out
