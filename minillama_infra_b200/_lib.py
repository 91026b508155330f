"""ctypes binding of libmli_gemv.so (the C ABI declared in include/mli_gemv.h).

The shared library is built in-tree by ``minillama_infra_b200/Makefile`` (see
``minillama_infra_b200.build``).  There is no fallback: if the library is
missing or fails to load, importing the ops raises, so a GPU run can never
silently take another path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libmli_gemv.so")
DROPIN_PATH = os.path.join(LIB_DIR, "libmli_dropin.so")

MLI_OK = 0
MLI_ERR_INVALID_ARG = 1
MLI_ERR_UNSUPPORTED = 2
MLI_ERR_CUDA = 3
MLI_ERR_DEVICE = 4
MLI_LAUNCH_PDL = 1
MLI_LAUNCH_NO_CLUSTER = 4
MLI_LAUNCH_NO_PERSISTENT = 8

# Every symbol include/mli_gemv.h declares with C linkage, with its ctypes
# signature (device pointers and streams travel as void*).
_P = ctypes.c_void_p
_I = ctypes.c_int
_U = ctypes.c_uint


class GemvOp(ctypes.Structure):
    """struct mli_gemv_op (include/mli_gemv.h): one GEMV of a chain."""
    _fields_ = [("form", _I), ("n", _I), ("d", _I), ("group_size", _I), ("wait", _I),
                ("epilogue", _I), ("y", _P), ("x", _P), ("xq", _P), ("xs", _P), ("w_q", _P),
                ("w_s", _P), ("norm_w", _P)]


_OPS = ctypes.POINTER(GemvOp)


class GemmOp(ctypes.Structure):
    """struct mli_gemm_op (include/mli_gemv.h): one GEMM of a group launch."""
    _fields_ = [("y", _P), ("xq", _P), ("xs", _P), ("w_q", _P), ("w_s", _P), ("n", _I), ("d", _I)]
SIGNATURES = {
    "mli_status_string": (ctypes.c_char_p, [_I]),
    "mli_last_status": (_I, []),
    "mli_last_cuda_error": (_I, []),
    "mli_version": (_I, []),
    "mli_get_launch_flags": (_U, []),
    "mli_set_launch_flags": (None, [_U]),
    "mli_device_error": (_I, [ctypes.POINTER(_U)]),
    "mli_gemv_w8a32": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "mli_quantize_activation": (_I, [_P, _P, _P, _I, _P]),
    "mli_gemv_w8a8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "mli_gemv_w8a8_fused": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "mli_quantize_activation_rows": (_I, [_P, _P, _P, _I, _I, _P]),
    "mli_gemm_w8a8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, ctypes.c_size_t, _P]),
    "mli_gemm_w8a8_workspace_bytes": (ctypes.c_size_t, [_I, _I, _I]),
    "mli_gemm_w8a8_cuda_core": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "mli_gemm_w8a8_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "mli_quantize_weights": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "mli_debug_group_dots": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "mli_debug_plan_gemv": (_I, [_I, _I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "mli_peer_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(_P), ctypes.c_char_p]),
    "mli_peer_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "mli_peer_close": (_I, [_P]),
    "mli_peer_free": (_I, [_P]),
    "mli_gemv_rowshard": (_I, [_I, ctypes.POINTER(_P), _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "mli_rowshard_wait_argmax": (_I, [_I, _I, _P, _P, ctypes.POINTER(_I), _I, _I, _P, _I, _P]),
    "mli_gemv_rowshard_argmax": (_I, [_I, ctypes.POINTER(_P), _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                      ctypes.POINTER(_I), _P, _I, _P]),
    "mli_rowshard_block_bytes": (ctypes.c_size_t, [_I]),
    "mli_argmax": (_I, [_P, _I, _P, _P]),
    "mli_gemv_f32": (_I, [_P, _P, _P, _I, _I, _P]),
    "mli_chain_create": (_I, [_OPS, _I, ctypes.POINTER(_P)]),
    "mli_chain_create_sharded": (_I, [_OPS, ctypes.POINTER(_I), ctypes.POINTER(_I), _I, _I, ctypes.POINTER(_P)]),
    "mli_chain_export": (_I, [_P, ctypes.c_char_p]),
    "mli_chain_set_peers": (_I, [_P, ctypes.POINTER(_P), _I]),
    "mli_chain_rows": (_I, [_P, _I, _P, ctypes.POINTER(_I)]),
    "mli_chain_run": (_I, [_P, _P]),
    "mli_chain_destroy": (_I, [_P]),
    "mli_debug_plan_chain": (_I, [_OPS, _I, _I, _I, ctypes.POINTER(_I)]),
    "mli_debug_plan_gemm": (_I, [_I, _I, _I, ctypes.c_size_t, ctypes.POINTER(_I)]),
    "mli_debug_plan_gemm_group": (_I, [ctypes.POINTER(GemmOp), _I, _I, ctypes.POINTER(_I)]),
    "mli_debug_int8_mma_peak": (_I, [_I, _I, _I, _P]),
    "mli_gemm_w8a8_group": (_I, [ctypes.POINTER(GemmOp), _I, _I, _I, _P]),
}

# The drop-in shim's C++ symbols (include/mli_gemv.h, reference include/model.h:62-64).
DROPIN_SYMBOLS = {
    "matmul_int8": "_Z11matmul_int8PfS_PaS_iii",
    "matmul_dp4a": "_Z11matmul_dp4aPfPKaPKfS1_S3_iii",
    "quantize_activation": "_Z19quantize_activationPaPfPKfi",
    "matmul": "_Z6matmulPfS_S_ii",
}

_lib = None
_dropin = None


class MliError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = lib().mli_status_string(status).decode()
        if status == MLI_ERR_CUDA:
            msg += f" (cudaError {lib().mli_last_cuda_error()})"
        super().__init__(f"{what}: {msg} [status {status}]")


def lib():
    """Load libmli_gemv.so once; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is not built; run `make -C {_HERE}` or __graft_entry__.build()")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def dropin():
    """Load libmli_dropin.so (the reference-signature shim)."""
    global _dropin
    if _dropin is None:
        if not os.path.exists(DROPIN_PATH):
            raise ImportError(f"{DROPIN_PATH} is not built")
        lib()
        l = ctypes.CDLL(DROPIN_PATH)
        P = ctypes.c_void_p
        f = getattr(l, DROPIN_SYMBOLS["matmul_int8"])
        f.argtypes, f.restype = [P, P, P, P, _I, _I, _I], None
        f = getattr(l, DROPIN_SYMBOLS["matmul_dp4a"])
        f.argtypes, f.restype = [P, P, P, P, P, _I, _I, _I], None
        f = getattr(l, DROPIN_SYMBOLS["quantize_activation"])
        f.argtypes, f.restype = [P, P, P, _I], None
        f = getattr(l, DROPIN_SYMBOLS["matmul"])
        f.argtypes, f.restype = [P, P, P, _I, _I], None
        _dropin = l
    return _dropin


def check(status: int, what: str) -> None:
    if status != MLI_OK:
        raise MliError(status, what)
