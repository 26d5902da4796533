"""ctypes wrapper of oracle/q4_cpu.c -- TEST INFRASTRUCTURE / CPU BASELINE.

Used only by tests/ and bench.py's CPU-baseline / reference arm.  Builds the
library with oracle/Makefile when it is missing."""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libq4cpu.so")
_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "q4_cpu.c")):
            subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
        L = ctypes.CDLL(LIB)
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.q4cpu_gemv.argtypes = [vp, i, i, i, vp, vp, i]
        L.q4cpu_ffn.argtypes = [vp, vp, vp, i, i, i, vp, vp, vp, i]
        L.q4cpu_ffn_block.argtypes = [vp, vp, vp, i, i, vp, i]
        for f in (L.q4cpu_gemv, L.q4cpu_ffn, L.q4cpu_ffn_block, L.q4cpu_max_threads):
            f.restype = i
        _lib = L
    return _lib


def max_threads() -> int:
    return load().q4cpu_max_threads()


def _p(a):
    return a.ctypes.data


def gemv(combined: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    combined = np.ascontiguousarray(combined, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    N, K = combined.shape[0], combined.shape[1] // 20 * 32
    ntok = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((ntok, N), np.float32)
    rc = load().q4cpu_gemv(_p(combined), N, K, ntok, _p(x), _p(y), nthreads)
    assert rc == 0, rc
    return y[0] if x.ndim == 1 else y


def ffn(gate_c, up_c, down_c, x, activation="gelu", nthreads: int = 0):
    g, u, d = (np.ascontiguousarray(a, np.uint8) for a in (gate_c, up_c, down_c))
    I, H = g.shape[0], g.shape[1] // 20 * 32
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(H, np.float32)
    act = np.empty(I, np.float32)
    rc = load().q4cpu_ffn(_p(g), _p(u), _p(d), H, I, 0 if activation == "gelu" else 1, _p(x), _p(y), _p(act),
                          nthreads)
    assert rc == 0, rc
    return y, act


def ffn_block(gate_c, up_c, down_c, x_bf, nthreads: int = 0) -> np.ndarray:
    g, u, d = (np.ascontiguousarray(a, np.uint8) for a in (gate_c, up_c, down_c))
    I, H = g.shape[0], g.shape[1] // 20 * 32
    x = np.array(x_bf, np.float32, copy=True)
    rc = load().q4cpu_ffn_block(_p(g), _p(u), _p(d), H, I, _p(x), nthreads)
    assert rc == 0, rc
    return x
