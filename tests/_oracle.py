"""ctypes access to the CPU oracle (oracle/liboracle.so) for the tests.

Test infrastructure only: the checker the CUDA path is compared against.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_DIR = ROOT / "oracle"
ORACLE_SO = ORACLE_DIR / "liboracle.so"

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
        L = C.CDLL(str(ORACLE_SO))
        fp, dp, sz = C.c_void_p, C.c_void_p, C.c_size_t
        L.zgo_splitmix64_at.restype = C.c_uint64
        L.zgo_splitmix64_at.argtypes = [C.c_uint64, C.c_uint64]
        L.zgo_fill_uniform.argtypes = [fp, sz, C.c_uint64]
        L.zgo_fill_uniform_range.argtypes = [fp, sz, C.c_uint64, C.c_float, C.c_float]
        L.zgo_fill_normal.argtypes = [fp, sz, C.c_uint64]
        L.zgo_add_f32.argtypes = [fp, fp, fp, sz]
        L.zgo_relu_f32.argtypes = [fp, fp, sz]
        L.zgo_add_f32_mt.argtypes = [fp, fp, fp, sz, C.c_int]
        L.zgo_relu_f32_mt.argtypes = [fp, fp, sz, C.c_int]
        L.zgo_saxpy_f32.argtypes = [C.c_float, fp, fp, sz]
        L.zgo_sscal_f32.argtypes = [C.c_float, fp, sz]
        L.zgo_sgemm_ref.argtypes = [C.c_int] * 3 + [C.c_float, fp, fp, fp] + [C.c_int] * 3
        L.zgo_sgemm_fast.argtypes = [C.c_int] * 3 + [C.c_float, fp, fp, fp, C.c_int]
        L.zgo_sgemm_bias_relu.argtypes = [C.c_int] * 3 + [C.c_float, fp, fp, fp, fp, C.c_int]
        L.zgo_dgemm_tile.argtypes = [C.c_int] * 3 + [C.c_double, fp, fp] + [C.c_int] * 4 + [dp]
        L.zgo_rel_fro_f32.restype = C.c_double
        L.zgo_rel_fro_f32.argtypes = [fp, fp, sz]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def uniform(n: int, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    if lo == -1.0 and hi == 1.0:
        lib().zgo_fill_uniform(_p(out), n, seed)
    else:
        lib().zgo_fill_uniform_range(_p(out), n, seed, lo, hi)
    return out


def normal(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().zgo_fill_normal(_p(out), n, seed)
    return out


def add(a, b, threads: int = 1) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    if threads > 1:
        lib().zgo_add_f32_mt(_p(a), _p(b), _p(out), a.size, threads)
    else:
        lib().zgo_add_f32(_p(a), _p(b), _p(out), a.size)
    return out


def relu(a, threads: int = 1) -> np.ndarray:
    a = _f32(a)
    out = np.empty_like(a)
    if threads > 1:
        lib().zgo_relu_f32_mt(_p(a), _p(out), a.size, threads)
    else:
        lib().zgo_relu_f32(_p(a), _p(out), a.size)
    return out


def saxpy(alpha: float, x, y) -> np.ndarray:
    x, y = _f32(x), _f32(y).copy()
    lib().zgo_saxpy_f32(alpha, _p(x), _p(y), x.size)
    return y


def sscal(alpha: float, x) -> np.ndarray:
    x = _f32(x).copy()
    lib().zgo_sscal_f32(alpha, _p(x), x.size)
    return x


def sgemm_ref(a, b, alpha: float = 1.0, rows: tuple[int, int] | None = None,
              threads: int = 1) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32)
    r0, r1 = rows if rows else (0, m)
    lib().zgo_sgemm_ref(m, n, k, alpha, _p(a), _p(b), _p(c), r0, r1, threads)
    return c


def sgemm(a, b, alpha: float = 1.0, threads: int = 8) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().zgo_sgemm_fast(m, n, k, alpha, _p(a), _p(b), _p(c), threads)
    return c


def sgemm_bias_relu(a, b, bias, alpha: float = 1.0, threads: int = 8) -> np.ndarray:
    a, b, bias = _f32(a), _f32(b), _f32(bias)
    m, k = a.shape
    n = b.shape[1]
    y = np.empty((m, n), np.float32)
    lib().zgo_sgemm_bias_relu(m, n, k, alpha, _p(a), _p(b), _p(bias), _p(y), threads)
    return y


def dgemm_tile(a, b, r0: int, c0: int, h: int, w: int, alpha: float = 1.0) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((h, w), np.float64)
    lib().zgo_dgemm_tile(m, n, k, alpha, _p(a), _p(b), r0, c0, h, w, _p(out))
    return out


def rel_fro(x, ref) -> float:
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)
