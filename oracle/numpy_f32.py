"""ctypes access to oracle/numpy_f32.c (numpy's float32 exp and row sum restated) — TEST
INFRASTRUCTURE ONLY.

``build()`` compiles the C file with gcc into ``oracle/_lib/`` (ignored by git; it travels to
the GPU box like the native library); ``lib()`` builds it on first use when it is missing.
"""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "numpy_f32.c"
LIBRARY = HERE / "_lib" / "liboracle_numpy_f32.so"


def build(force: bool = False) -> Path:
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    compiler = shutil.which("gcc") or shutil.which("cc")
    if compiler is None:
        raise RuntimeError("no C compiler for the oracle's numpy restatement")
    LIBRARY.parent.mkdir(exist_ok=True)
    tmp = LIBRARY.with_suffix(".tmp.so")
    # -ffp-contract=off: every multiply and add rounds on its own unless written as fmaf.
    subprocess.run([compiler, "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", str(SOURCE),
                    "-o", str(tmp), "-lm"], check=True, capture_output=True)
    tmp.replace(LIBRARY)
    return LIBRARY


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    handle = ctypes.CDLL(str(build()))
    handle.oracle_numpy_expf_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    handle.oracle_numpy_row_sums.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    return handle


def expf(values: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_numpy_expf_array(x.ctypes.data, out.ctypes.data, x.size)
    return out


def row_sums(matrix: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(matrix, dtype=np.float32)
    rows, width = a.shape
    out = np.empty(rows, dtype=np.float32)
    lib().oracle_numpy_row_sums(a.ctypes.data, rows, width, out.ctypes.data)
    return out
