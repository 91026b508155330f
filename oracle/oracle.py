"""CPU oracle for the INT8 group-64 linear path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped: only tests/,
``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` / reference legs
import it.  It wraps ``liboracle.so`` (built from ``mli_oracle.c`` by
``oracle/Makefile``), whose functions restate the reference routines:

    quantize_weights        scripts/quantize_int8_group.py:55-71
    quantize_activation     src/model_cuda_v2_shared.cu:429-455
    gemv_w8a32              src/model_cuda_v2_shared.cu:36-62
    gemv_w8a8               src/model_cuda_v2_shared.cu:465-501
    matmul_f32              src/model_cuda_v2_shared.cu:10-19 (fp32 classifier)
    rmsnorm_chain           src/model_cuda_v2_shared.cu:74-89, in the chained prologue's order
    group_dots              the int32 group partials of :483-494

Parity pins: ``tests/golden/`` holds the reference quantiser script's own
output on a synthetic weight file and the reference CUDA kernels' outputs
(rebuilt for sm_100a, run on a B200); the CPU tests check this oracle against
both bit for bit.

It also exposes the reference's own CUDA kernels (``oracle/_ref/libmli_ref.so``,
compiled unmodified from the reference tree) for GPU parity tests and for the
reference arm of bench.py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_REF_PATH = os.path.join(_HERE, "_ref", "libmli_ref.so")
_lib = None
_ref = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_L = ctypes.c_long
_I = ctypes.c_int


def build() -> None:
    """Compile liboracle.so (and _ref/libmli_ref.so when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        l = ctypes.CDLL(_LIB_PATH)
        sig = {
            "oracle_quantize_weights": (_I, [_i8p, _f32p, _f32p, _L, _L, _I]),
            "oracle_quantize_activation": (None, [_i8p, _f32p, _f32p, _L]),
            "oracle_quantize_activation_rows": (None, [_i8p, _f32p, _f32p, _L, _L]),
            "oracle_gemv_w8a32": (None, [_f32p, _f32p, _i8p, _f32p, _L, _L, _I]),
            "oracle_group_dots": (None, [_i32p, _i8p, _i8p, _L, _L, _I]),
            "oracle_gemv_w8a8": (None, [_f32p, _i8p, _f32p, _i8p, _f32p, _L, _L, _I]),
            "oracle_gemm_w8a8": (None, [_f32p, _i8p, _f32p, _i8p, _f32p, _L, _L, _L, _I]),
            "oracle_gemv_w8a32_f64": (None, [_f64p, _f32p, _i8p, _f32p, _L, _L, _I]),
            "oracle_gemv_w8a8_f64": (None, [_f64p, _i8p, _f32p, _i8p, _f32p, _L, _L, _I]),
            "oracle_matmul_f32": (None, [_f32p, _f32p, _f32p, _L, _L]),
            "oracle_rmsnorm_chain": (None, [_f32p, _f32p, _f32p, _L]),
            "oracle_matmul_f64": (None, [_f64p, _f32p, _f32p, _L, _L]),
            "oracle_gemm_w8a8_f64": (None, [_f64p, _i8p, _f32p, _i8p, _f32p, _L, _L, _L, _I]),
            "oracle_group_dot_sums": (None, [_i64p, _i8p, _i8p, _i32p, _L, _L, _L, _I]),
            "oracle_dequant_matvec": (None, [_f32p, _f32p, _i8p, _f32p, _L, _L, _I]),
            "oracle_num_threads": (_I, []),
            "oracle_set_num_threads": (None, [_I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def quantize_weights(w: np.ndarray, group_size: int = 64):
    """(int8 [rows][cols], fp32 [rows][cols/gs]) exactly as the reference script."""
    w = _c(w, np.float32)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty((rows, cols // group_size), np.float32)
    rc = lib().oracle_quantize_weights(q, s, w, rows, cols, group_size)
    if rc != 0:
        raise ValueError("cols must be a multiple of group_size")
    return q, s


def quantize_activation(x: np.ndarray):
    x = _c(x, np.float32)
    if x.ndim == 1:
        xq = np.empty(x.shape, np.int8)
        xs = np.empty(1, np.float32)
        lib().oracle_quantize_activation(xq, xs, x, x.shape[0])
        return xq, xs
    m, n = x.shape
    xq = np.empty((m, n), np.int8)
    xs = np.empty(m, np.float32)
    lib().oracle_quantize_activation_rows(xq, xs, x, m, n)
    return xq, xs


def gemv_w8a32(x, w_q, w_s, group_size: int = 64):
    d, n = w_q.shape
    y = np.empty(d, np.float32)
    lib().oracle_gemv_w8a32(y, _c(x, np.float32), _c(w_q, np.int8), _c(w_s, np.float32), n, d, group_size)
    return y


def gemv_w8a8(xq, xs, w_q, w_s, group_size: int = 64):
    d, n = w_q.shape
    y = np.empty(d, np.float32)
    lib().oracle_gemv_w8a8(y, _c(xq, np.int8), _c(xs, np.float32).reshape(-1), _c(w_q, np.int8),
                           _c(w_s, np.float32), n, d, group_size)
    return y


def gemm_w8a8(xq, xs, w_q, w_s, group_size: int = 64):
    d, n = w_q.shape
    m = xq.shape[0]
    y = np.empty((m, d), np.float32)
    lib().oracle_gemm_w8a8(y, _c(xq, np.int8), _c(xs, np.float32), _c(w_q, np.int8),
                           _c(w_s, np.float32), m, n, d, group_size)
    return y


def group_dots(xq, w_q, group_size: int = 64):
    d, n = w_q.shape
    out = np.empty((d, n // group_size), np.int32)
    lib().oracle_group_dots(out, _c(xq, np.int8), _c(w_q, np.int8), n, d, group_size)
    return out


def gemv_w8a32_f64(x, w_q, w_s, group_size: int = 64):
    d, n = w_q.shape
    y = np.empty(d, np.float64)
    lib().oracle_gemv_w8a32_f64(y, _c(x, np.float32), _c(w_q, np.int8), _c(w_s, np.float32), n, d,
                                group_size)
    return y


def gemv_w8a8_f64(xq, xs, w_q, w_s, group_size: int = 64):
    d, n = w_q.shape
    y = np.empty(d, np.float64)
    lib().oracle_gemv_w8a8_f64(y, _c(xq, np.int8), _c(xs, np.float32).reshape(-1), _c(w_q, np.int8),
                               _c(w_s, np.float32), n, d, group_size)
    return y


def rmsnorm_chain(x, w):
    """RMSNorm (src/model_cuda_v2_shared.cu:74-89) summed in the chained GEMV
    prologue's fixed order: bit-identical to what the chain computes."""
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().oracle_rmsnorm_chain(out, x, _c(w, np.float32), x.shape[0])
    return out


def matmul_f32(x, w):
    """The reference's fp32 matmul, in its order (one sequential FMA chain per row)."""
    d, n = w.shape
    y = np.empty(d, np.float32)
    lib().oracle_matmul_f32(y, _c(x, np.float32), _c(w, np.float32), n, d)
    return y


def matmul_f64(x, w):
    d, n = w.shape
    y = np.empty(d, np.float64)
    lib().oracle_matmul_f64(y, _c(x, np.float32), _c(w, np.float32), n, d)
    return y


def gemm_w8a8_f64(xq, xs, w_q, w_s, group_size: int = 64):
    """fp64 recompute of m tokens at once (y [m][d]); token t equals
    gemv_w8a8_f64(xq[t], xs[t:t+1], ...)."""
    d, n = w_q.shape
    xq = _c(xq, np.int8).reshape(-1, n)
    m = xq.shape[0]
    y = np.empty((m, d), np.float64)
    lib().oracle_gemm_w8a8_f64(y, xq, _c(xs, np.float32).reshape(-1), _c(w_q, np.int8), _c(w_s, np.float32),
                               m, n, d, group_size)
    return y


def group_dot_sums(xq, w_q, k, group_size: int = 64):
    """Exact int64 y[t][r] = sum_g I_t[r][g] * k[r][g] (k integer, [d][n/gs])."""
    d, n = w_q.shape
    xq = _c(xq, np.int8).reshape(-1, n)
    m = xq.shape[0]
    y = np.empty((m, d), np.int64)
    lib().oracle_group_dot_sums(y, xq, _c(w_q, np.int8), _c(k, np.int32), m, n, d, group_size)
    return y


def dequant_matvec(x, w_q, w_s, group_size: int = 64, out=None):
    """CPU baseline: float32 dequant-then-matvec, OpenMP over rows."""
    d, n = w_q.shape
    y = np.empty(d, np.float32) if out is None else out
    lib().oracle_dequant_matvec(y, x, w_q, w_s, n, d, group_size)
    return y


_CPU_BASELINE = os.path.join(_HERE, "cpu_baseline.c")


def cpu_baseline_lib(out_dir: str):
    """Compiles cpu_baseline.c with -O3 -march=native for the host that calls
    this (into out_dir) and returns its ctypes handle."""
    so = os.path.join(out_dir, "libcpu_baseline.so")
    cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
    subprocess.run([cc, "-O3", "-march=native", "-fopenmp", "-fPIC", "-shared", "-std=c11",
                    _CPU_BASELINE, "-o", so], check=True)
    l = ctypes.CDLL(so)
    l.cpu_dequant_matvec.argtypes = [_f32p, _f32p, _i8p, _f32p, _L, _L, _I]
    l.cpu_dequant_matvec.restype = None
    l.cpu_num_threads.restype = _I
    return l


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(t: int) -> None:
    lib().oracle_set_num_threads(int(t))


def max_abs_rel(y, y_ref) -> float:
    """max_i |y - y_ref| / max_i |y_ref| (the tolerance metric of the parity tests)."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    den = float(np.max(np.abs(y_ref)))
    if den == 0.0:
        return float(np.max(np.abs(y)))
    return float(np.max(np.abs(y - y_ref)) / den)


# ---------------------------------------------------------------------------
# The reference's own CUDA kernels (GPU; device pointers as integers)
# ---------------------------------------------------------------------------
def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


def ref():
    """ctypes handle of oracle/_ref/libmli_ref.so (the reference's kernels)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(
                f"{_REF_PATH} missing: build it with `make -C oracle ref` where the reference tree exists")
        l = ctypes.CDLL(_REF_PATH)
        P = ctypes.c_void_p
        l.ref_matmul_int8.argtypes = [P, P, P, P, _I, _I, _I]
        l.ref_matmul_int8.restype = None
        l.ref_matmul_dp4a.argtypes = [P, P, P, P, P, _I, _I, _I]
        l.ref_matmul_dp4a.restype = None
        l.ref_quantize_activation.argtypes = [P, P, P, _I]
        l.ref_quantize_activation.restype = None
        l.ref_last_error.restype = _I
        l.ref_device_synchronize.restype = _I
        _ref = l
    return _ref
