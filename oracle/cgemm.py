"""Build and bind the C restatement of the GEMM (oracle/c/oracle_gemm.c) — test and
CPU-baseline infrastructure only.  Built with gcc -O3 -march=native -fopenmp into
oracle/_build/ (not committed)."""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "c" / "oracle_gemm.c"
OUT = HERE / "_build" / "liboracle_gemm.so"


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(parents=True, exist_ok=True)
    if force or not OUT.exists() or OUT.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O3", "-march=native", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC",
               str(SRC), "-o", str(OUT)]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
    return OUT


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(build()))
        p = ctypes.c_void_p
        L.oracle_qgemm_bf16.argtypes = [ctypes.c_int] * 4 + [p] * 5
        L.oracle_qgemm_bf16.restype = ctypes.c_int
        L.oracle_qgemm_tile_bf16.argtypes = [ctypes.c_int] * 4 + [p] * 5
        L.oracle_gemm_dense_bf16.argtypes = [ctypes.c_int] * 3 + [p] * 3
        L.oracle_threads.restype = ctypes.c_int
        L.oracle_set_reverse.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def qgemm(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    n = packed.shape[0]
    out = np.empty((m, n), np.float32)
    rc = lib().oracle_qgemm_bf16(m, n, k, bits, x.ctypes.data, np.ascontiguousarray(packed).ctypes.data,
                                 np.ascontiguousarray(scales).ctypes.data, np.ascontiguousarray(biases).ctypes.data,
                                 out.ctypes.data)
    if rc != 0:
        raise MemoryError("oracle_qgemm_bf16: group sums")
    return out


def qgemm_tile(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int) -> np.ndarray:
    """x . W'^T with every weight dequantized to bf16 first (oracle_qgemm_tile_bf16)."""
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    n = packed.shape[0]
    out = np.empty((m, n), np.float32)
    lib().oracle_qgemm_tile_bf16(m, n, k, bits, x.ctypes.data, np.ascontiguousarray(packed).ctypes.data,
                                 np.ascontiguousarray(scales).ctypes.data, np.ascontiguousarray(biases).ctypes.data,
                                 out.ctypes.data)
    return out


def gemm_dense(x: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    n = w_bits.shape[0]
    out = np.empty((m, n), np.float32)
    lib().oracle_gemm_dense_bf16(m, n, k, x.ctypes.data, np.ascontiguousarray(w_bits).ctypes.data, out.ctypes.data)
    return out


def threads() -> int:
    return int(lib().oracle_threads())


def set_reverse(reverse: bool) -> None:
    """Sum along K in descending order (True) or ascending (False, the default)."""
    lib().oracle_set_reverse(int(bool(reverse)))
