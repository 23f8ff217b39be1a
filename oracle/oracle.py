"""ctypes/numpy face of the CPU oracle (bw_oracle.c). TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs as
the checker. The library never imports it.

Each function names the reference code it restates (paths within
waynehacking8/blackwell-tensorcore-kernels):
  ref_fill_rand     include/util.cuh:17             glibc rand() inputs, uniform[-0.5, 0.5]
  f32_to_f16        src/gemm_wmma.cu:106-108         __float2half (RNE)
  quant_fp8         src/gemm_mma_fp8.cu:37-45        __nv_fp8_e4m3 satfinite, B -> Bt
  e2m1_code         src/gemm_mma_fp8.cu:47-58        f32_to_e2m1
  quant_fp4         src/gemm_mma_fp8.cu:61-68        q_fp4 / q_fp4_t (code << 2)
  quant_mxfp4       src/gemm_mma_fp8.cu:70-80        q_mxfp4 / q_mxfp4_t (packed)
  gemm_f64          src/gemm_mma.cu:23-141           C = A x B (accumulated in FP64 here)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build() -> str:
    """Compile liboracle.so (gcc) if missing or stale."""
    src = os.path.join(_HERE, "bw_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.or_srand.argtypes = [ctypes.c_uint]
        L.or_ref_fill_rand.argtypes = [P, ctypes.c_long]
        L.or_f32_to_f16_array.argtypes = [P, P, ctypes.c_long]
        L.or_f16_to_f32_array.argtypes = [P, P, ctypes.c_long]
        L.or_e2m1_code.argtypes = [ctypes.c_float]
        L.or_e2m1_code.restype = ctypes.c_uint8
        L.or_f32_to_e4m3_sat.argtypes = [ctypes.c_float]
        L.or_f32_to_e4m3_sat.restype = ctypes.c_uint8
        L.or_quant_fp8.argtypes = [P, P, P, I, I, I, I]
        L.or_quant_fp4.argtypes = [P, P, P, I, I, I, I, I]
        L.or_quant_mxfp4.argtypes = [P, P, P, I, I, I, I]
        L.or_dequant_mxfp4.argtypes = [P, P, P, I, I]
        L.or_dequant_fp8.argtypes = [P, P, ctypes.c_long]
        L.or_sf_bytes.argtypes = [I, I]
        L.or_sf_bytes.restype = ctypes.c_long
        L.or_sf_offset.argtypes = [I, I, I]
        L.or_sf_offset.restype = ctypes.c_long
        L.or_gemm_f64.argtypes = [P, P, P, I, I, I, I, I]
        L.or_gemm_f64.restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ inputs
def ref_fill_rand(M: int, N: int, K: int, seed: int = 1):
    """hA then hB from glibc rand() after srand(seed) (default seed = 1), as src/main.cu:49."""
    L = lib()
    L.or_srand(seed)
    A = np.empty((M, K), np.float32)
    B = np.empty((K, N), np.float32)
    L.or_ref_fill_rand(_p(A), A.size)
    L.or_ref_fill_rand(_p(B), B.size)
    return A, B


def seeded_uniform(shape, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    return np.random.default_rng(seed).uniform(lo, hi, size=shape).astype(np.float32)


def seeded_normal(shape, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(size=shape).astype(np.float32)


# ------------------------------------------------------------------ element conversions
def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_f16_array(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().or_f16_to_f32_array(_p(h), _p(out), h.size)
    return out


def e2m1_code(v: float) -> int:
    return int(lib().or_e2m1_code(float(v)))


def e4m3_code(v: float) -> int:
    return int(lib().or_f32_to_e4m3_sat(float(v)))


E2M1_LEVELS = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float32)


# ------------------------------------------------------------------ quantisers
SCALE_NONE, SCALE_FIXED8, SCALE_AMAX = 0, 1, 2
FP4_PACKED, FP4_BYTE_SHL2 = 0, 1
MX_UNIT_FIXED8, MX_BLOCK32 = 0, 1


def quant_fp8(src: np.ndarray, transpose: bool, mode: int):
    src = np.ascontiguousarray(src, np.float32)
    rows, cols = src.shape
    out = np.empty((cols, rows) if transpose else (rows, cols), np.uint8)
    s = np.zeros(1, np.float32)
    lib().or_quant_fp8(_p(src), _p(out), _p(s), rows, cols, int(transpose), mode)
    return out, float(s[0])


def quant_fp4(src: np.ndarray, transpose: bool, mode: int, container: int):
    src = np.ascontiguousarray(src, np.float32)
    rows, cols = src.shape
    orows, ocols = (cols, rows) if transpose else (rows, cols)
    out = np.empty((orows, ocols if container == FP4_BYTE_SHL2 else ocols // 2), np.uint8)
    s = np.zeros(1, np.float32)
    lib().or_quant_fp4(_p(src), _p(out), _p(s), rows, cols, int(transpose), mode, container)
    return out, float(s[0])


def sf_bytes(outer: int, K: int) -> int:
    return int(lib().or_sf_bytes(outer, K))


def sf_offset(row: int, kblock: int, K: int) -> int:
    return int(lib().or_sf_offset(row, kblock, K))


def quant_mxfp4(src: np.ndarray, transpose: bool, mode: int):
    src = np.ascontiguousarray(src, np.float32)
    rows, cols = src.shape
    K, outer = (rows, cols) if transpose else (cols, rows)
    q = np.empty((outer, K // 2), np.uint8)
    sf = np.empty(sf_bytes(outer, K), np.uint8)
    lib().or_quant_mxfp4(_p(src), _p(q), _p(sf), rows, cols, int(transpose), mode)
    return q, sf


def dequant_mxfp4(q: np.ndarray, sf: np.ndarray | None, K: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.uint8)
    rows = q.shape[0]
    out = np.empty((rows, K), np.float32)
    lib().or_dequant_mxfp4(_p(q), None if sf is None else _p(np.ascontiguousarray(sf)), _p(out), rows, K)
    return out


def dequant_fp4_byte(q: np.ndarray) -> np.ndarray:
    return E2M1_LEVELS[(np.asarray(q) >> 2) & 15]


def dequant_fp8(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, np.uint8)
    out = np.empty(q.shape, np.float32)
    lib().or_dequant_fp8(_p(q), _p(out), q.size)
    return out


# ------------------------------------------------------------------ GEMM
def gemm_f64(A: np.ndarray, B: np.ndarray, b_trans: bool = False, threads: int | None = None) -> np.ndarray:
    """C = A x B (B given K x N, or N x K when b_trans) accumulated in double."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[0] if b_trans else B.shape[1]
    C = np.empty((M, N), np.float64)
    if threads is None:
        threads = os.cpu_count() or 1
    rc = lib().or_gemm_f64(_p(A), _p(B), _p(C), M, N, K, int(b_trans), int(threads))
    if rc != 0:
        raise MemoryError("oracle GEMM allocation failed")
    return C


def f16_tolerance(K: int, amax_a: float, amax_b: float) -> float:
    """FP16 bound of the north star: 2^-10 * sqrt(K) * max|a| * max|b|."""
    return 2.0 ** -10 * np.sqrt(K) * amax_a * amax_b


def lowp_tolerance(K: int, amax_a: float, amax_b: float, cref_absmax: float = 0.0, bf16_out: bool = False) -> float:
    """FP8/FP4/MXFP4 bound: 1e-5 * K * max|a_deq| * max|b_deq| (+ half a bf16 ulp of |C|)."""
    tol = 1e-5 * K * amax_a * amax_b
    if bf16_out:
        tol += cref_absmax * 2.0 ** -8
    return tol
