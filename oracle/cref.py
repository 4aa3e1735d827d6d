"""ctypes binding of the C oracle (scans_ref.c) -- TEST INFRASTRUCTURE ONLY.

Builds ``oracle/_build/liboracle_scans.so`` on first use with the Makefile
beside it.  Used as the timed CPU baseline and as a second oracle in tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle_scans.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        fp = ctypes.POINTER(ctypes.c_float)
        L.oracle_wkv7_scan.argtypes = [fp] * 9 + [ctypes.c_int] * 5
        L.oracle_wkv7_scan.restype = None
        L.oracle_rosa_scan.argtypes = [fp] * 8 + [ctypes.c_int] * 5
        L.oracle_rosa_scan.restype = None
        _lib = L
    return _lib


def _p(x):
    if x is None:
        return None
    assert x.dtype == np.float32 and x.flags.c_contiguous
    return x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def threads_default() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def wkv7_scan(r, w, k, v, a, b, s0=None, n_threads=None):
    arrs = [np.ascontiguousarray(x, np.float32) for x in (r, w, k, v, a, b)]
    B, T, H, N = arrs[0].shape
    s0c = None if s0 is None else np.ascontiguousarray(s0, np.float32)
    y = np.empty((B, T, H, N), np.float32)
    sT = np.empty((B, H, N, N), np.float32)
    lib().oracle_wkv7_scan(*[_p(x) for x in arrs], _p(s0c), _p(y), _p(sT), B, T, H, N,
                           n_threads or threads_default())
    return y, sT


def rosa_scan(cand, write, read_gate, decay, direction, m0, gated=True, n_threads=None):
    c, wr, g = (np.ascontiguousarray(x, np.float32) for x in (cand, write, read_gate))
    dec = np.ascontiguousarray(decay, np.float32).reshape(-1)
    d = np.ascontiguousarray(direction, np.float32).reshape(-1)
    m0c = np.ascontiguousarray(m0, np.float32)
    B, T, R = c.shape
    read = np.empty((B, T, R), np.float32)
    mT = np.empty((B, R), np.float32)
    lib().oracle_rosa_scan(_p(c), _p(wr), _p(g), _p(dec), _p(d), _p(m0c), _p(read), _p(mT),
                           B, T, R, 1 if gated else 0, n_threads or threads_default())
    return read, mT
