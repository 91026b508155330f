"""Row-sharded classifier pieces on one GPU: device argmax semantics, the
fused GEMV -> peer-logits -> wait/argmax step with this rank as its own only
peer, and the bounded wait giving up (status, not a hang) when rows never
arrive."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200._lib import check, lib
from minillama_infra_b200.shard import read_tagged_logits

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
HEADER = 256


def dev():
    return torch.device("cuda:0")


def argmax_dev(x):
    out = torch.full((), -7, dtype=torch.int64, device=dev())
    check(lib().mli_argmax(x.data_ptr(), x.numel(), out.data_ptr(), None), "mli_argmax")
    torch.cuda.synchronize()
    return int(out.item())


def first_max(a):
    """The reference's host argmax (src/model_cuda_v2_shared.cu:571-575)."""
    best, bi = a[0], 0
    for i in range(1, len(a)):
        if a[i] > best:
            best, bi = a[i], i
    return bi


@pytest.mark.parametrize("n", [1, 5, 1000, 128256, 128257])
def test_argmax_matches_reference_scan(n):
    x = synth.activation_np(n, n)
    assert argmax_dev(torch.from_numpy(x).to(dev())) == int(np.argmax(x))


def test_argmax_ties_zeros_nan_misaligned():
    a = np.array([1.0, 3.0, -2.0, 3.0, 3.0], np.float32)
    assert argmax_dev(torch.from_numpy(a).to(dev())) == first_max(a) == 1
    z = np.array([-0.0, 0.0, -0.0, -1.0], np.float32)
    assert argmax_dev(torch.from_numpy(z).to(dev())) == first_max(z) == 0
    nan = np.array([1.0, np.nan, 2.0, np.nan, 5.0, 1.0], np.float32)
    assert argmax_dev(torch.from_numpy(nan).to(dev())) == first_max(nan) == 4
    nan0 = np.array([np.nan, 2.0, 5.0, 1.0], np.float32)  # the reference's scan starts from x[0]
    assert argmax_dev(torch.from_numpy(nan0).to(dev())) == first_max(nan0) == 0
    ninf = np.full(9, -np.inf, np.float32)
    assert argmax_dev(torch.from_numpy(ninf).to(dev())) == first_max(ninf) == 0
    big = synth.activation_np(4099, 3)
    t = torch.zeros(4100, dtype=torch.float32, device=dev())
    t[1:] = torch.from_numpy(big).to(dev())
    out = torch.zeros((), dtype=torch.int64, device=dev())
    check(lib().mli_argmax(t.data_ptr() + 4, 4099, out.data_ptr(), None), "mli_argmax")
    torch.cuda.synchronize()
    assert int(out.item()) == int(np.argmax(big))


class Block:
    def __init__(self, d):
        self.ptr = ctypes.c_void_p()
        self.h = ctypes.create_string_buffer(64)
        check(lib().mli_peer_alloc(lib().mli_rowshard_block_bytes(d), ctypes.byref(self.ptr), self.h), "alloc")
        self.base = self.ptr.value
        self.d = d

    def logits(self, half=0):
        """Device address of the logits words (8 bytes per row) of one half."""
        return self.base + HEADER + half * self.d * 8

    def read_logits(self, step):
        """fp32 logits of step `step`, every word checked for the step's tag."""
        return read_tagged_logits(self.logits(0), self.d, step & 1, step)

    def free(self):
        lib().mli_peer_free(self.base)


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_rowshard_single_rank_loopback(form):
    d, n = 5003, 2048
    w_q, w_s = synth.weights_gpu(d, n, seed=3, device=dev())
    x = synth.activation_gpu(n, 4, dev(), outliers=(form == "w8a8"))
    ref = torch.empty(d, dtype=torch.float32, device=dev())
    if form == "w8a32":
        ops.matmul_int8(ref, x, w_q, w_s, n, d, 64)
    else:
        ops.matmul_dp4a_fused(ref, x, w_q, w_s, n, d, 64)
    b = Block(d)
    P = ctypes.c_void_p
    logits_arr = (P * 1)(b.logits(0))
    shard_rows = (ctypes.c_int * 1)(d)
    out = torch.zeros((), dtype=torch.int64, device=dev())
    code = 0 if form == "w8a32" else 2
    try:
        for step in range(3):  # both halves, then the first again
            check(lib().mli_gemv_rowshard(code, logits_arr, b.base + 128, x.data_ptr(),
                                          w_q.data_ptr(), w_s.data_ptr(), n, d, 0, d, 0, 1, 64, None),
                  "rowshard")
            check(lib().mli_rowshard_wait_argmax(code, n, b.logits(0), b.base + 128, shard_rows, 1, d,
                                                 out.data_ptr(), 1_000_000, None), "wait")
            torch.cuda.synchronize()
            got = b.read_logits(step)
            assert np.array_equal(got.view(np.uint32), ref.cpu().numpy().view(np.uint32))
            assert int(out.item()) == int(torch.argmax(ref).item())
        assert ops.device_error() == 0
    finally:
        b.free()


def test_rowshard_argmax_first_max_across_ctas():
    """Equal maxima in rows handled by different CTAs: the smallest index wins,
    as in the reference's scan; all-negative logits never pick a stale zero."""
    d, n = 9000, 256
    w = np.zeros((d, n), np.float32)
    w[:, 0] = -1.0                 # every row: -x0 ...
    w[[100, 5000, 8999], 0] = 2.0  # ... except three equal maxima in far-apart rows
    w_q, w_s = orc.quantize_weights(w)
    x = np.zeros(n, np.float32)
    x[0] = 1.0
    tw, ts, tx = (torch.from_numpy(a).to(dev()) for a in (w_q, w_s, x))
    b = Block(d)
    P = ctypes.c_void_p
    out = torch.zeros((), dtype=torch.int64, device=dev())
    try:
        for step in range(2):
            check(lib().mli_gemv_rowshard(0, (P * 1)(b.logits(0)), b.base + 128, tx.data_ptr(),
                                          tw.data_ptr(), ts.data_ptr(), n, d, 0, d, 0, 1, 64, None), "rowshard")
            check(lib().mli_rowshard_wait_argmax(0, n, b.logits(0), b.base + 128, (ctypes.c_int * 1)(d), 1,
                                                 d, out.data_ptr(), 1_000_000, None), "wait")
            torch.cuda.synchronize()
            assert int(out.item()) == 100
    finally:
        b.free()


def test_rowshard_wait_gives_up_when_rows_never_arrive():
    d = 1024
    b = Block(d)
    out = torch.zeros((), dtype=torch.int64, device=dev())
    shard_rows = (ctypes.c_int * 2)(512, 512)
    try:
        check(lib().mli_rowshard_wait_argmax(0, 2048, b.logits(0), b.base + 128, shard_rows, 2, d,
                                             out.data_ptr(), 100_000, None), "wait")
        torch.cuda.synchronize()
        assert int(out.item()) == -1
        assert ops.device_error() == 3
        assert ops.device_error() == 0  # read-and-clear
        # the context is still usable
        assert argmax_dev(torch.arange(10, dtype=torch.float32, device=dev())) == 9
    finally:
        b.free()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_rowshard_fused_argmax_single_rank(form):
    """mli_gemv_rowshard_argmax (one launch per step): the same logits and
    argmax as the two-launch step, over both halves and back."""
    d, n = 5003, 2048
    w_q, w_s = synth.weights_gpu(d, n, seed=5, device=dev())
    x = synth.activation_gpu(n, 6, dev(), outliers=(form == "w8a8"))
    ref = torch.empty(d, dtype=torch.float32, device=dev())
    if form == "w8a32":
        ops.matmul_int8(ref, x, w_q, w_s, n, d, 64)
    else:
        ops.matmul_dp4a_fused(ref, x, w_q, w_s, n, d, 64)
    b = Block(d)
    P = ctypes.c_void_p
    out = torch.full((), -7, dtype=torch.int64, device=dev())
    code = 0 if form == "w8a32" else 2
    try:
        for step in range(3):
            check(lib().mli_gemv_rowshard_argmax(code, (P * 1)(b.logits(0)), b.base, x.data_ptr(),
                                                 w_q.data_ptr(), w_s.data_ptr(), n, d, 0, d, 0, 1, 64,
                                                 (ctypes.c_int * 1)(d), out.data_ptr(), 1_000_000, None), "fused")
            torch.cuda.synchronize()
            got = b.read_logits(step)
            assert np.array_equal(got.view(np.uint32), ref.cpu().numpy().view(np.uint32))
            assert int(out.item()) == int(torch.argmax(ref).item())
        assert ops.device_error() == 0
    finally:
        b.free()


def test_rowshard_fused_gives_up_when_a_rank_never_arrives():
    """A declared second rank that never runs: the last CTA's bounded wait
    expires, *out = -1, device error 3, and the context stays usable."""
    d, n = 1024, 256
    w_q, w_s = synth.weights_gpu(512, n, seed=7, device=dev())
    x = synth.activation_gpu(n, 8, dev())
    b0, b1 = Block(d), Block(d)  # rank 1's block stands in for a peer that never writes
    P = ctypes.c_void_p
    out = torch.zeros((), dtype=torch.int64, device=dev())
    try:
        check(lib().mli_gemv_rowshard_argmax(0, (P * 2)(b0.logits(0), b1.logits(0)),
                                             b0.base, x.data_ptr(), w_q.data_ptr(), w_s.data_ptr(), n, 512, 0, d,
                                             0, 2, 64, (ctypes.c_int * 2)(512, 512), out.data_ptr(), 100_000,
                                             None), "fused")
        torch.cuda.synchronize()
        assert int(out.item()) == -1
        assert ops.device_error() == 3
        assert ops.device_error() == 0
        assert argmax_dev(torch.arange(10, dtype=torch.float32, device=dev())) == 9
    finally:
        b0.free()
        b1.free()
