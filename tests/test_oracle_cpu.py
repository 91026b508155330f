"""CPU tests of the oracle (mli_oracle.c) against the reference's own outputs.

* quant_ref_script.npz: the reference quantiser script run unmodified on a
  synthetic weight file (tests/golden/make_golden_quant.py).
* ref_kernels_*.npz: the reference's CUDA kernels (src/model_cuda_v2_shared.cu,
  rebuilt for sm_100a) run on a B200 (tests/golden/make_golden_gpu.py).
"""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import synth

QUANT_KEYS = ["wq", "wk", "wv", "wo", "w1", "w2", "w3"]


def test_weight_quantiser_matches_reference_script(golden_dir):
    z = np.load(os.path.join(golden_dir, "quant_ref_script.npz"))
    for k in QUANT_KEYS:
        q, s = orc.quantize_weights(z[f"{k}_w"])
        assert np.array_equal(q, z[f"{k}_q"]), k
        assert np.array_equal(s.view(np.uint32), z[f"{k}_s"].view(np.uint32)), k


def test_weight_quantiser_edge_cases():
    w = np.zeros((3, 128), np.float32)
    w[1, :4] = [127.0, 0.5, 1.5, -2.5]  # scale 1.0 -> ties round half to even
    w[2, 64] = -1e-38                    # subnormal amax
    q, s = orc.quantize_weights(w)
    assert s[0, 0] == np.float32(1e-9) / np.float32(127.0)
    assert np.all(q[0] == 0)
    assert list(q[1, :4]) == [127, 0, 2, -2]
    assert s[1, 0] == 1.0
    assert q[2, 64] == -127


def _np_quantize_activation(x):
    """Independent numpy restatement of src/model_cuda_v2_shared.cu:434-454."""
    x = np.asarray(x, np.float32)
    amax = np.max(np.abs(x)).astype(np.float32)
    scale = np.float32(amax / np.float32(127.0))
    if scale < np.float32(1e-8):
        scale = np.float32(1e-8)
    inv = np.float32(np.float32(1.0) / scale)
    v = (x * inv).astype(np.float32)
    q = np.clip(np.rint(v), -127, 127).astype(np.int8)
    return q, np.array([scale], np.float32)


@pytest.mark.parametrize("n", [64, 2048, 8192, 1000])
def test_activation_quantiser_matches_numpy_restatement(n):
    for seed in range(3):
        x = synth.activation_np(n, seed, outliers=(seed == 2))
        q, s = orc.quantize_activation(x)
        q2, s2 = _np_quantize_activation(x)
        assert np.array_equal(q, q2)
        assert s.view(np.uint32)[0] == s2.view(np.uint32)[0]


def test_activation_quantiser_edges():
    q, s = orc.quantize_activation(np.zeros(256, np.float32))
    assert s[0] == np.float32(1e-8) and np.all(q == 0)
    x = np.zeros(128, np.float32)
    x[0], x[1], x[2], x[3] = 127.0, -127.0, 0.5, 2.5  # scale 1.0: ties to even
    q, s = orc.quantize_activation(x)
    assert s[0] == 1.0 and list(q[:4]) == [127, -127, 0, 2]
    xm = synth.activation_np(512, 7, m=4)
    qm, sm = orc.quantize_activation(xm)
    for t in range(4):
        qt, st = orc.quantize_activation(xm[t])
        assert np.array_equal(qm[t], qt) and sm[t] == st[0]


@pytest.mark.parametrize("d,n", [(64, 2048), (37, 8192), (512, 256)])
def test_group_dots_exact(d, n):
    w_q, _ = orc.quantize_weights(synth.weights_np(d, n, 1))
    xq, _ = orc.quantize_activation(synth.activation_np(n, 2, outliers=True))
    dots = orc.group_dots(xq, w_q)
    ref = (w_q.astype(np.int64).reshape(d, n // 64, 64) * xq.astype(np.int64).reshape(1, n // 64, 64)).sum(-1)
    assert np.array_equal(dots.astype(np.int64), ref)


@pytest.mark.parametrize("d,n", [(128, 2048), (64, 8192), (33, 3072)])
def test_gemv_oracles_within_tolerance_of_f64(d, n):
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, 3))
    x = synth.activation_np(n, 4)
    y = orc.gemv_w8a32(x, w_q, w_s)
    assert orc.max_abs_rel(y, orc.gemv_w8a32_f64(x, w_q, w_s)) < 1e-6
    xq, xs = orc.quantize_activation(synth.activation_np(n, 5, outliers=True))
    y8 = orc.gemv_w8a8(xq, xs, w_q, w_s)
    assert orc.max_abs_rel(y8, orc.gemv_w8a8_f64(xq, xs, w_q, w_s)) < 1e-6
    yb = orc.dequant_matvec(x, w_q, w_s)
    assert orc.max_abs_rel(yb, orc.gemv_w8a32_f64(x, w_q, w_s)) < 1e-5


def _ref_kernel_fixtures(golden_dir):
    return sorted(glob.glob(os.path.join(golden_dir, "ref_kernels_*.npz")))


def test_reference_kernel_fixtures_present(golden_dir):
    assert _ref_kernel_fixtures(golden_dir), "tests/golden/ref_kernels_*.npz missing"


def test_oracle_bit_exact_vs_reference_kernels(golden_dir):
    """The oracle reproduces the reference CUDA kernels' outputs bit for bit."""
    files = _ref_kernel_fixtures(golden_dir)
    if not files:
        pytest.skip("no reference-kernel fixtures")
    for f in files:
        z = np.load(f)
        w_q, w_s, x = z["w_q"], z["w_s"], z["x"]
        gs = int(z["group_size"])
        y = orc.gemv_w8a32(x, w_q, w_s, gs)
        assert np.array_equal(y.view(np.uint32), z["y_w8a32"].view(np.uint32)), f
        xq, xs = orc.quantize_activation(x)
        assert np.array_equal(xq, z["xq"]), f
        assert xs.view(np.uint32)[0] == z["xs"].view(np.uint32)[0], f
        y8 = orc.gemv_w8a8(z["xq"], z["xs"], w_q, w_s, gs)
        assert np.array_equal(y8.view(np.uint32), z["y_w8a8"].view(np.uint32)), f
