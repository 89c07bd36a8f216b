"""ctypes wrapper of the C Philox restatement (oracle/philox_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the product's Philox kernel. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline leg may use it.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "philox_oracle.c"
LIB = HERE / "_build" / "libphilox_oracle.so"


def build(force: bool = False) -> Path:
    """Compile the C restatement with gcc into oracle/_build/ (idempotent)."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-o", str(LIB), str(SRC), "-lm"], check=True)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        _lib.oracle_philox_raw.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64,
                                           ctypes.c_uint64]
        _lib.oracle_randn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64,
                                      ctypes.c_int]
        _lib.oracle_philox4x32_10.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib.oracle_philox_grid.restype = ctypes.c_int64
        _lib.oracle_philox_grid.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        _lib.oracle_philox_offset_increment.restype = ctypes.c_int64
        _lib.oracle_philox_offset_increment.argtypes = [ctypes.c_int64, ctypes.c_int]
    return _lib


def philox_block(ctr: tuple[int, int, int, int], key: tuple[int, int]) -> np.ndarray:
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(c.ctypes.data, k.ctypes.data, out.ctypes.data)
    return out


def philox_raw(threads: int, rounds: int, seed: int, offset: int) -> np.ndarray:
    out = np.zeros(threads * rounds * 4, dtype=np.uint32)
    lib().oracle_philox_raw(out.ctypes.data, threads, rounds, seed, offset)
    return out


def randn(n: int, seed: int, offset: int, grid: int) -> np.ndarray:
    """float64 normals in the torch grid-stride layout (see philox_oracle.c)."""
    out = np.zeros(n, dtype=np.float64)
    lib().oracle_randn(out.ctypes.data, n, seed, offset, grid)
    return out


def grid_for(n: int, sms: int, max_threads_per_sm: int) -> int:
    return int(lib().oracle_philox_grid(n, sms, max_threads_per_sm))


def offset_increment(n: int, grid: int) -> int:
    return int(lib().oracle_philox_offset_increment(n, grid))


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float64 -> float32 -> bfloat16 (nearest-even) and return the uint16 bits."""
    f = x.astype(np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)
