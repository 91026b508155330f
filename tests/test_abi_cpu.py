"""CPU checks of the C ABI boundary: the libraries load, export every symbol
include/mli_gemv.h declares, and reject bad arguments before touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

from minillama_infra_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mli_gemv.h")


def header_c_functions():
    text = open(HEADER).read()
    # drop comments, then collect every mli_* function declaration
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mli_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = header_c_functions()
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    l = _lib.lib()
    for name in header_c_functions():
        assert hasattr(l, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (mli_\w+)", out))
    assert set(header_c_functions()) <= exported


def test_dropin_exports_reference_signatures():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.DROPIN_PATH], capture_output=True,
                         text=True, check=True).stdout
    for mangled in _lib.DROPIN_SYMBOLS.values():
        assert f" T {mangled}" in out, mangled
    # the mangled names equal the reference build's own (when it was built here)
    ref = os.path.join(ROOT, "oracle", "_ref", "libmli_ref.so")
    if os.path.exists(ref):
        rout = subprocess.run(["nm", "-D", "--defined-only", ref], capture_output=True, text=True,
                              check=True).stdout
        for mangled in _lib.DROPIN_SYMBOLS.values():
            assert f" T {mangled}" in rout, mangled
    _lib.dropin()


def test_status_strings_and_version():
    l = _lib.lib()
    assert l.mli_status_string(0) == b"ok"
    assert l.mli_status_string(1) == b"invalid argument"
    assert l.mli_status_string(99) == b"unknown status"
    assert l.mli_version() >= 100


def test_launch_flags_roundtrip():
    l = _lib.lib()
    old = l.mli_get_launch_flags()
    l.mli_set_launch_flags(0)
    assert l.mli_get_launch_flags() == 0
    l.mli_set_launch_flags(old)
    assert l.mli_get_launch_flags() == old


@pytest.mark.parametrize("call", [
    lambda l: l.mli_gemv_w8a32(None, None, None, None, 64, 8, 64, None),
    lambda l: l.mli_gemv_w8a32(8, 8, 8, 8, 0, 8, 64, None),
    lambda l: l.mli_gemv_w8a32(8, 8, 8, 8, 64, -1, 64, None),
    lambda l: l.mli_gemv_w8a32(8, 8, 8, 8, 64, 8, 0, None),
    lambda l: l.mli_gemv_w8a8(8, None, 8, 8, 8, 64, 8, 64, None),
    lambda l: l.mli_gemv_w8a8_fused(8, 8, None, 8, 8, 8, 64, 8, 64, None),
    lambda l: l.mli_quantize_activation(None, 8, 8, 64, None),
    lambda l: l.mli_quantize_activation(8, 8, 8, 0, None),
    lambda l: l.mli_quantize_activation_rows(8, 8, 8, 0, 64, None),
    lambda l: l.mli_gemm_w8a8(8, 8, 8, 8, 8, 0, 64, 8, 64, None, 0, None),
    lambda l: l.mli_gemm_w8a8_cuda_core(8, 8, 8, 8, 8, 4, 100, 8, 64, None),
    lambda l: l.mli_rowshard_wait_argmax(0, 2048, 8, 8, None, 1, 64, 8, 100, None),
    lambda l: l.mli_gemv_rowshard_argmax(0, None, 8, 8, 8, 8, 2048, 64, 0, 64, 0, 1, 64, None, 8, 100, None),
    lambda l: l.mli_gemv_rowshard(0, None, 8, 8, 8, 8, 2048, 64, 0, 64, 0, 1, 64, None),
    lambda l: l.mli_argmax(None, 8, 8, None),
    lambda l: l.mli_gemv_f32(None, 8, 8, 64, 8, None),
    lambda l: l.mli_gemv_f32(8, 8, 8, 0, 8, None),
    lambda l: l.mli_quantize_weights(8, 8, 8, 4, 100, 64, None),
    lambda l: l.mli_debug_group_dots(None, 8, 8, 64, 8, 64, None),
    lambda l: l.mli_chain_create_sharded(None, None, None, 1, 2, None),
    lambda l: l.mli_chain_export(None, None),
    lambda l: l.mli_chain_set_peers(None, None, 0),
    lambda l: l.mli_chain_rows(None, 0, None, None),
])
def test_invalid_arguments_rejected_without_gpu(call):
    l = _lib.lib()
    assert call(l) == _lib.MLI_ERR_INVALID_ARG
    assert l.mli_last_status() == _lib.MLI_ERR_INVALID_ARG


def test_gemm_group_arguments_checked_without_gpu():
    """mli_gemm_w8a8_group: an empty or null op list and null operands are
    invalid, more than MLI_GEMM_GROUP_MAX ops or shapes off the tensor-core
    path unsupported -- all decided before any CUDA call."""
    l = _lib.lib()
    ops = (_lib.GemmOp * 9)()
    assert l.mli_gemm_w8a8_group(None, 1, 16, 64, None) == _lib.MLI_ERR_INVALID_ARG
    assert l.mli_gemm_w8a8_group(ops, 0, 16, 64, None) == _lib.MLI_ERR_INVALID_ARG
    assert l.mli_gemm_w8a8_group(ops, 1, 16, 64, None) == _lib.MLI_ERR_INVALID_ARG  # null pointers
    assert l.mli_gemm_w8a8_group(ops, 9, 16, 64, None) == _lib.MLI_ERR_UNSUPPORTED
    for i in range(2):
        ops[i] = _lib.GemmOp(256, 256, 256, 256, 256, 1024, 128)  # 256-byte aligned stand-ins
    assert l.mli_gemm_w8a8_group(ops, 2, 8, 64, None) == _lib.MLI_ERR_UNSUPPORTED    # m < 16
    assert l.mli_gemm_w8a8_group(ops, 2, 16, 32, None) == _lib.MLI_ERR_UNSUPPORTED   # group 32
    ops[1] = _lib.GemmOp(256, 256, 256, 256, 256, 1000, 128)
    assert l.mli_gemm_w8a8_group(ops, 2, 16, 64, None) == _lib.MLI_ERR_UNSUPPORTED   # n % 128
    ops[1] = _lib.GemmOp(256, 257, 256, 256, 256, 1024, 128)
    assert l.mli_gemm_w8a8_group(ops, 2, 16, 64, None) == _lib.MLI_ERR_UNSUPPORTED   # xq misaligned


def test_oracle_library_is_not_linked_by_product():
    """The product library must not depend on the oracle."""
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out and "mli_ref" not in out
