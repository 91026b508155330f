"""GPU parity of the CUDA kernels (through the C ABI) against the CPU oracle.

Tolerances (the ones the path is specified with):
  * int8 / index outputs (quantised activations, quantised weights, int32
    group dots): bit-exact.
  * W8A32 fp32 output: max|y - y_ref| / max|y_ref| <= 1e-5 against the
    oracle (the reference's own arithmetic order) and the fp64 recompute.
  * W8A8 fp32 output: <= 1e-6 of the fp64 recompute from the exact int32
    group dots (sum_g I_g * ws * xs), and of the oracle.
"""
import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200._lib import MliError, lib

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_W8A32 = 1e-5
TOL_W8A8 = 1e-6
GUARD = 64  # guard-band floats before and after every output


def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def up(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev())


class Guarded:
    """Output buffer with canary bands on both sides."""

    def __init__(self, n, dtype=torch.float32):
        self.n = n
        fill = float("nan") if dtype.is_floating_point else 0x5A
        self.buf = torch.full((n + 2 * GUARD,), fill, dtype=dtype, device=dev())
        self.t = self.buf[GUARD:GUARD + n]

    def check(self):
        head = self.buf[:GUARD].cpu().numpy()
        tail = self.buf[GUARD + self.n:].cpu().numpy()
        if self.buf.dtype.is_floating_point:
            assert np.all(np.isnan(head)) and np.all(np.isnan(tail)), "guard band overwritten"
        else:
            assert np.all(head == 0x5A) and np.all(tail == 0x5A), "guard band overwritten"
        return self.t.cpu().numpy()


def make_case(d, n, seed, outliers=False):
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, seed))
    x = synth.activation_np(n, seed + 1, outliers=outliers)
    return w_q, w_s, x


# (d, n): config shapes, ragged row counts, single group, fast-path limit,
# partial slices, and shapes that take the generic kernels (n % 256 != 0,
# more than eight slices).
SHAPES = [
    (2048, 2048), (512, 2048), (8192, 2048), (2048, 8192), (1024, 3072), (3072, 3072),
    (37, 2048), (1, 256), (300, 512), (5, 16384), (3, 16640), (9, 320), (7, 64),
    (129, 6144), (40, 1280), (16, 12288),
]


@pytest.mark.parametrize("d,n", SHAPES)
def test_w8a32_parity(d, n):
    w_q, w_s, x = make_case(d, n, d * 7 + n)
    y = Guarded(d)
    ops.matmul_int8(y.t, up(x), up(w_q), up(w_s), n, d, 64)
    torch.cuda.synchronize()
    got = y.check()
    assert orc.max_abs_rel(got, orc.gemv_w8a32(x, w_q, w_s)) <= TOL_W8A32
    assert orc.max_abs_rel(got, orc.gemv_w8a32_f64(x, w_q, w_s)) <= TOL_W8A32


@pytest.mark.parametrize("d,n", SHAPES)
def test_w8a8_parity(d, n):
    w_q, w_s, x = make_case(d, n, d * 11 + n, outliers=True)
    xq_ref, xs_ref = orc.quantize_activation(x)
    tx = up(x)
    xq = Guarded(n, torch.int8)
    xs = torch.empty(1, dtype=torch.float32, device=dev())
    ops.quantize_activation(xq.t, xs, tx, n)
    y = Guarded(d)
    ops.matmul_dp4a(y.t, xq.t, xs, up(w_q), up(w_s), n, d, 64)
    torch.cuda.synchronize()
    assert np.array_equal(xq.check(), xq_ref)
    assert xs.cpu().numpy().view(np.uint32)[0] == xs_ref.view(np.uint32)[0]
    got = y.check()
    assert orc.max_abs_rel(got, orc.gemv_w8a8_f64(xq_ref, xs_ref, w_q, w_s)) <= TOL_W8A8
    assert orc.max_abs_rel(got, orc.gemv_w8a8(xq_ref, xs_ref, w_q, w_s)) <= TOL_W8A8


@pytest.mark.parametrize("d,n", SHAPES)
def test_w8a8_fused_parity(d, n):
    w_q, w_s, x = make_case(d, n, d * 13 + n, outliers=True)
    xq_ref, xs_ref = orc.quantize_activation(x)
    y = Guarded(d)
    xq = Guarded(n, torch.int8)
    xs = torch.empty(1, dtype=torch.float32, device=dev())
    ops.matmul_dp4a_fused(y.t, up(x), up(w_q), up(w_s), n, d, 64, xq_out=xq.t, xs_out=xs)
    torch.cuda.synchronize()
    assert np.array_equal(xq.check(), xq_ref)
    assert xs.cpu().numpy().view(np.uint32)[0] == xs_ref.view(np.uint32)[0]
    got = y.check()
    assert orc.max_abs_rel(got, orc.gemv_w8a8_f64(xq_ref, xs_ref, w_q, w_s)) <= TOL_W8A8


def test_w8a8_fused_without_outputs():
    d, n = 1024, 2048
    w_q, w_s, x = make_case(d, n, 99, outliers=True)
    xq_ref, xs_ref = orc.quantize_activation(x)
    y = Guarded(d)
    ops.matmul_dp4a_fused(y.t, up(x), up(w_q), up(w_s), n, d, 64)
    torch.cuda.synchronize()
    assert orc.max_abs_rel(y.check(), orc.gemv_w8a8_f64(xq_ref, xs_ref, w_q, w_s)) <= TOL_W8A8


@pytest.mark.parametrize("gs", [32, 128])
def test_other_group_sizes(gs):
    d, n = 64, 1024
    w = synth.weights_np(d, n, 5)
    w_q, w_s = orc.quantize_weights(w, gs)
    x = synth.activation_np(n, 6)
    y = Guarded(d)
    ops.matmul_int8(y.t, up(x), up(w_q), up(w_s), n, d, gs)
    xq_ref, xs_ref = orc.quantize_activation(x)
    y8 = Guarded(d)
    ops.matmul_dp4a(y8.t, up(xq_ref), up(xs_ref), up(w_q), up(w_s), n, d, gs)
    torch.cuda.synchronize()
    assert orc.max_abs_rel(y.check(), orc.gemv_w8a32(x, w_q, w_s, gs)) <= TOL_W8A32
    assert orc.max_abs_rel(y8.check(), orc.gemv_w8a8_f64(xq_ref, xs_ref, w_q, w_s, gs)) <= TOL_W8A8


def test_misaligned_pointers_take_generic_path():
    d, n = 40, 2048
    w_q, w_s, x = make_case(d, n, 17)
    # shift activation / weights by 4 bytes inside larger buffers
    xb = torch.zeros(n + 4, dtype=torch.float32, device=dev())
    xb[1:1 + n] = up(x)
    wb = torch.zeros(d * n + 4, dtype=torch.int8, device=dev())
    wb[4:4 + d * n] = up(w_q.reshape(-1))
    y = Guarded(d)
    ops.matmul_int8(y.t, xb.data_ptr() + 4, wb.data_ptr() + 4, up(w_s), n, d, 64)
    torch.cuda.synchronize()
    assert orc.max_abs_rel(y.check(), orc.gemv_w8a32(x, w_q, w_s)) <= TOL_W8A32


def test_zero_activation():
    d, n = 64, 2048
    w_q, w_s, _ = make_case(d, n, 3)
    x = np.zeros(n, np.float32)
    xq = torch.empty(n, dtype=torch.int8, device=dev())
    xs = torch.empty(1, dtype=torch.float32, device=dev())
    y = Guarded(d)
    ops.matmul_dp4a_fused(y.t, up(x), up(w_q), up(w_s), n, d, 64, xq_out=xq, xs_out=xs)
    torch.cuda.synchronize()
    assert np.all(y.check() == 0.0)
    assert xs.item() == np.float32(1e-8) and int(xq.abs().max()) == 0


def test_group_dots_bit_exact():
    d, n = 300, 8192
    w_q, _, x = make_case(d, n, 23, outliers=True)
    xq, _ = orc.quantize_activation(x)
    out = torch.empty((d, n // 64), dtype=torch.int32, device=dev())
    ops.group_dots(out, up(xq), up(w_q), n, d, 64)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), orc.group_dots(xq, w_q))


def test_weight_quantiser_bit_exact(golden_dir):
    import os
    z = np.load(os.path.join(golden_dir, "quant_ref_script.npz"))
    cases = [(z[f"{k}_w"], z[f"{k}_q"], z[f"{k}_s"]) for k in ["wq", "wk", "w1", "w2"]]
    w = synth.weights_np(333, 2048, 8)
    q_ref, s_ref = orc.quantize_weights(w)
    cases.append((w, q_ref, s_ref))
    for w, q_ref, s_ref in cases:
        rows, cols = w.shape
        q = torch.empty((rows, cols), dtype=torch.int8, device=dev())
        s = torch.empty((rows, cols // 64), dtype=torch.float32, device=dev())
        ops.quantize_weights(q, s, up(w), rows, cols, 64)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), q_ref)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def _gemm_case(m, n, d, seed, workspace):
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, seed))
    x = synth.activation_np(n, seed + 1, m=m, outliers=True)
    xq_ref, xs_ref = orc.quantize_activation(x)
    xq = torch.empty((m, n), dtype=torch.int8, device=dev())
    xs = torch.empty(m, dtype=torch.float32, device=dev())
    ops.quantize_activation_rows(xq, xs, up(x), m, n)
    ws = None
    if workspace:
        ws = torch.zeros(ops.gemm_workspace_bytes(m, n, d), dtype=torch.uint8, device=dev())
    y = Guarded(m * d)
    tw, ts = up(w_q), up(w_s)
    ops.gemm_w8a8(y.t, xq, xs, tw, ts, m, n, d, 64, workspace=ws)
    torch.cuda.synchronize()
    assert np.array_equal(xq.cpu().numpy(), xq_ref)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), xs_ref.view(np.uint32))
    got = y.check().reshape(m, d)
    for t in range(m):
        ref = orc.gemv_w8a8_f64(xq_ref[t], xs_ref[t:t + 1], w_q, w_s)
        assert orc.max_abs_rel(got[t], ref) <= TOL_W8A8, t
    return got, (xq, xs, tw, ts, ws)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13])
def test_gemm_w8a8_cuda_core_parity(m):
    _gemm_case(m, 3072, 640, 31 + m, workspace=False)


# m >= 16 takes the tcgen05 kind::i8 path: token tiles of 16/32/64/128 (padded
# tokens), partial weight tiles, with and without split-K workspace.
@pytest.mark.parametrize("m,n,d", [(16, 256, 128), (16, 3072, 640), (17, 3072, 1024), (64, 1024, 300),
                                   (100, 2048, 384), (128, 8192, 256), (256, 3072, 512), (300, 1024, 200)])
@pytest.mark.parametrize("workspace", [False, True], ids=["no_ws", "splitk"])
def test_gemm_w8a8_tensor_core_parity(m, n, d, workspace):
    got, (xq, xs, tw, ts, ws) = _gemm_case(m, n, d, 7 * m + d, workspace)
    if ws is not None:
        ws.fill_(0x7F)  # the workspace may hold anything between calls
        y2 = torch.empty(m * d, dtype=torch.float32, device=dev())
        ops.gemm_w8a8(y2, xq, xs, tw, ts, m, n, d, 64, workspace=ws)
        torch.cuda.synchronize()
        assert np.array_equal(y2.cpu().numpy().reshape(m, d).view(np.uint32), got.view(np.uint32))
    assert ops.device_error() == 0


@pytest.mark.parametrize("m,n,d", [(16, 3072, 1024), (64, 3072, 3072), (256, 3072, 1024), (100, 8192, 384),
                                   (300, 1024, 200), (17, 2048, 130)])
def test_gemm_split_k_cluster_and_workspace_paths(m, n, d):
    """The K splits of a tile summed inside a thread-block cluster (default)
    and through the workspace (MLI_LAUNCH_NO_CLUSTER) both match the oracle,
    and each path is deterministic."""
    try:
        for clusters in (True, False):
            ops.set_gemm_clusters(clusters)
            got, (xq, xs, tw, ts, ws) = _gemm_case(m, n, d, 3 * m + d, workspace=True)
            y2 = torch.empty(m * d, dtype=torch.float32, device=dev())
            ops.gemm_w8a8(y2, xq, xs, tw, ts, m, n, d, 64, workspace=ws)
            torch.cuda.synchronize()
            assert np.array_equal(y2.cpu().numpy().reshape(m, d).view(np.uint32), got.view(np.uint32))
    finally:
        ops.set_gemm_clusters(True)
    assert ops.device_error() == 0


@pytest.mark.parametrize("m", [16, 64, 128, 256])
@pytest.mark.parametrize("pattern", ["max", "min", "mixed"])
def test_gemm_extreme_int8_operands(m, pattern):
    """Group dots at the ends of the int8 range: all -128 x -128 (I = 2^20),
    -128 x 127 (I = -1,040,384) and random bytes over the full range, with
    unit scales (every output an exact integer) and with random scales; the
    offset-MMA path (128-token tiles) and the refill path agree with the
    oracle exactly on the integer case."""
    n, d = 1024, 256
    rng = np.random.default_rng(5 + m)
    if pattern == "max":
        xq_h = np.full((m, n), -128, np.int8)
        wq_h = np.full((d, n), -128, np.int8)
    elif pattern == "min":
        xq_h = np.full((m, n), -128, np.int8)
        wq_h = np.full((d, n), 127, np.int8)
    else:
        xq_h = rng.integers(-128, 128, (m, n), dtype=np.int16).astype(np.int8)
        wq_h = rng.integers(-128, 128, (d, n), dtype=np.int16).astype(np.int8)
    for scales in ("unit", "random"):
        if scales == "unit":
            xs_h = np.ones(m, np.float32)
            ws_h = np.ones((d, n // 64), np.float32)
        else:
            xs_h = rng.uniform(1e-4, 1e-1, m).astype(np.float32)
            ws_h = rng.uniform(1e-5, 1e-2, (d, n // 64)).astype(np.float32)
        y = Guarded(m * d)
        ops.gemm_w8a8(y.t, up(xq_h), up(xs_h), up(wq_h), up(ws_h), m, n, d, 64)
        torch.cuda.synchronize()
        got = y.check().reshape(m, d)
        for t in sorted({0, m // 2, m - 1}):
            ref = orc.gemv_w8a8_f64(xq_h[t], xs_h[t:t + 1], wq_h, ws_h)
            if scales == "unit":  # sums of 16 integers of magnitude <= 2^20: exact in fp32
                assert np.array_equal(got[t].astype(np.float64), ref), (t, scales)
            else:
                assert orc.max_abs_rel(got[t], ref) <= TOL_W8A8, (t, scales)
    assert ops.device_error() == 0


def test_gemm_group_scale_range():
    """128-token tiles take the group scale as ws * 2^90: exact up to 2^38
    (checked at 2^37), refused through the device error word (code 5) at
    2^40."""
    m, n, d = 128, 1024, 128
    rng = np.random.default_rng(11)
    xq_h = rng.integers(-127, 128, (m, n), dtype=np.int16).astype(np.int8)
    wq_h = rng.integers(-127, 128, (d, n), dtype=np.int16).astype(np.int8)
    xs_h = rng.uniform(1e-3, 1e-2, m).astype(np.float32)
    ws_h = rng.uniform(1e-4, 1e-3, (d, n // 64)).astype(np.float32)
    ws_h[3, 5] = 2.0 ** 37
    y = torch.empty(m * d, dtype=torch.float32, device=dev())
    ops.gemm_w8a8(y, up(xq_h), up(xs_h), up(wq_h), up(ws_h), m, n, d, 64)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    got = y.cpu().numpy().reshape(m, d)
    for t in (0, 77, 127):
        ref = orc.gemv_w8a8_f64(xq_h[t], xs_h[t:t + 1], wq_h, ws_h)
        assert orc.max_abs_rel(got[t], ref) <= TOL_W8A8, t
    ws_h[3, 5] = 2.0 ** 40
    ops.gemm_w8a8(y, up(xq_h), up(xs_h), up(wq_h), up(ws_h), m, n, d, 64)
    torch.cuda.synchronize()
    assert ops.device_error() == 5


@pytest.mark.parametrize("m,n,d", [(16, 3072, 1024), (256, 3072, 1024), (256, 8192, 3072), (64, 2048, 8192)])
def test_gemm_plan_is_consistent(m, n, d):
    """mli_gemm_w8a8's plan on this GPU: K splits within [1, K chunks / 2],
    clusters of at most 16 that are the splits themselves, the workspace used
    only when given, and MLI_LAUNCH_NO_CLUSTER turning clusters off."""
    import ctypes

    out = (ctypes.c_int * 5)()
    need = ops.gemm_workspace_bytes(m, n, d)
    for ws_bytes in (0, need):
        assert lib().mli_debug_plan_gemm(m, n, d, ws_bytes, out) == 0
        bn, tiles, splits, cluster, via_ws = list(out)
        assert bn == (16 if m <= 16 else 32 if m <= 32 else 64 if m <= 64 else 128)
        assert tiles == -(-d // 128) * -(-m // bn)
        assert 1 <= splits <= max(1, n // 128 // 2)
        assert via_ws in (0, 1) and (via_ws == 0 or ws_bytes > 0)
        assert cluster == (1 if via_ws else splits) and cluster <= 16
    try:
        ops.set_gemm_clusters(False)
        assert lib().mli_debug_plan_gemm(m, n, d, need, out) == 0
        assert out[3] == 1
        assert lib().mli_debug_plan_gemm(m, n, d, 0, out) == 0
        assert out[2] == 1 and out[3] == 1 and out[4] == 0  # no workspace, no cluster: K is not split
    finally:
        ops.set_gemm_clusters(True)


# mli_gemm_w8a8_group: several independent GEMMs of m tokens in one launch,
# ragged shapes (partial row tiles, K from 2 to 64 chunks, padded tokens).
@pytest.mark.parametrize("m,shapes", [
    (16, [(640, 3072), (128, 256), (300, 1024), (1024, 8192)]),
    (100, [(384, 2048), (200, 1024), (256, 3072)]),
    (256, [(512, 3072), (1024, 3072), (128, 8192), (1024, 3072), (512, 3072), (256, 1024), (640, 2048)]),
])
def test_gemm_w8a8_group_parity(m, shapes):
    items, refs = [], []
    for i, (d, n) in enumerate(shapes):
        seed = 900 + 17 * i + m
        w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, seed))
        x = synth.activation_np(n, seed + 1, m=m, outliers=True)
        xq_ref, xs_ref = orc.quantize_activation(x)
        xq = torch.empty((m, n), dtype=torch.int8, device=dev())
        xs = torch.empty(m, dtype=torch.float32, device=dev())
        ops.quantize_activation_rows(xq, xs, up(x), m, n)
        y = Guarded(m * d)
        items.append((y, xq, xs, up(w_q), up(w_s), n, d))
        refs.append((w_q, w_s, xq_ref, xs_ref))
    ops.gemm_w8a8_group([(y.t, xq, xs, tw, ts, n, d) for (y, xq, xs, tw, ts, n, d) in items], m)
    torch.cuda.synchronize()
    firsts = []
    for (y, xq, xs, tw, ts, n, d), (w_q, w_s, xq_ref, xs_ref) in zip(items, refs):
        got = y.check().reshape(m, d)
        firsts.append(got.copy())
        for t in sorted({0, 1, m // 2, m - 1}):
            ref = orc.gemv_w8a8_f64(xq_ref[t], xs_ref[t:t + 1], w_q, w_s)
            assert orc.max_abs_rel(got[t], ref) <= TOL_W8A8, (d, n, t)
    # deterministic: a second launch gives the same bits
    outs = [torch.empty(m * d, dtype=torch.float32, device=dev()) for (_, _, _, _, _, n, d) in items]
    ops.gemm_w8a8_group([(o, xq, xs, tw, ts, n, d) for o, (_, xq, xs, tw, ts, n, d) in zip(outs, items)], m)
    torch.cuda.synchronize()
    for o, f, (_, _, _, _, _, n, d) in zip(outs, firsts, items):
        assert np.array_equal(o.cpu().numpy().reshape(m, d).view(np.uint32), f.view(np.uint32))
    assert ops.device_error() == 0


def _layer_items(shapes, m, seed):
    items = []
    for i, (d, n) in enumerate(shapes):
        q, s = synth.weights_torch(d, n, seed=seed + i, device=dev())
        x = synth.activation_gpu(n, seed + 50 + i, dev(), m=m, outliers=True)
        xq = torch.empty((m, n), dtype=torch.int8, device=dev())
        xs = torch.empty(m, dtype=torch.float32, device=dev())
        ops.quantize_activation_rows(xq, xs, x, m, n)
        items.append((Guarded(m * d), xq, xs, q, s, n, d))
    return items


def _check_items(items, m, got):
    for (y, xq, xs, q, s, n, d), yn in zip(items, got):
        xq_h, xs_h, q_h, s_h = xq.cpu().numpy(), xs.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy()
        for t in sorted({0, 1, m // 2, m - 1}):
            ref = orc.gemv_w8a8_f64(xq_h[t], xs_h[t:t + 1], q_h, s_h)
            assert orc.max_abs_rel(yn[t], ref) <= TOL_W8A8, (d, n, t)


# (d, n) sets with enough 128 x 128 output tiles for the persistent kernel:
# the Llama-3.2-3B projections of one layer, and ragged rows and tokens
# (partial last row tile and token tile, K of 8 to 24 chunks).
PERSISTENT_CASES = [
    (256, [(d, n) for (_, d, n) in synth.LLAMA_3B]),
    (300, [(d, n) for (_, d, n) in synth.LLAMA_3B]),
    (500, [(3000, 3072), (8100, 3072), (1000, 1024)]),
]


@pytest.mark.parametrize("m,shapes", PERSISTENT_CASES)
def test_gemm_persistent_group_parity(m, shapes):
    """mli_gemm_w8a8_group takes the persistent whole-tile kernel for these
    problems; sampled tokens of every matrix match the oracle, a second launch
    gives the same bits, and the split-K kernels agree within the tolerance."""
    items = _layer_items(shapes, m, 700)
    args = [(y.t, xq, xs, q, s, n, d) for (y, xq, xs, q, s, n, d) in items]
    plan = ops.gemm_group_plan(args, m)
    assert plan["persistent"], plan
    assert plan["ctas"] == min(plan["tiles"], torch.cuda.get_device_properties(0).multi_processor_count)
    ops.gemm_w8a8_group(args, m)
    torch.cuda.synchronize()
    got = [y.check().reshape(m, d) for (y, _, _, _, _, n, d) in items]
    _check_items(items, m, got)
    again = [torch.empty(m * d, dtype=torch.float32, device=dev()) for (_, _, _, _, _, n, d) in items]
    ops.gemm_w8a8_group([(o,) + a[1:] for o, a in zip(again, args)], m)
    torch.cuda.synchronize()
    for o, g in zip(again, got):
        assert np.array_equal(o.cpu().numpy().reshape(g.shape).view(np.uint32), g.view(np.uint32))
    try:
        ops.set_gemm_persistent(False)
        assert not ops.gemm_group_plan(args, m)["persistent"]
        ops.gemm_w8a8_group([(o,) + a[1:] for o, a in zip(again, args)], m)
        torch.cuda.synchronize()
    finally:
        ops.set_gemm_persistent(True)
    for o, g in zip(again, got):
        sk = o.cpu().numpy().reshape(g.shape)
        for t in (0, m - 1):
            assert orc.max_abs_rel(sk[t], g[t]) <= TOL_W8A8
    assert ops.device_error() == 0


def test_gemm_persistent_single_matrix():
    """mli_gemm_w8a8 on one matrix with enough tiles (8192 x 3072 at 512
    tokens: 256 tiles) runs on the persistent kernel too; at 256 tokens (128
    tiles, fewer than the SMs) it takes the split-K kernels."""
    m = 512
    items = _layer_items([(8192, 3072)], m, 900)
    y, xq, xs, q, s, n, d = items[0]
    assert ops.gemm_group_plan([(y.t, xq, xs, q, s, n, d)], m)["persistent"]
    assert not ops.gemm_group_plan([(y.t, xq[:256], xs[:256], q, s, n, d)], 256)["persistent"]
    ops.gemm_w8a8(y.t, xq, xs, q, s, m, n, d, 64)
    torch.cuda.synchronize()
    _check_items(items, m, [y.check().reshape(m, d)])
    assert ops.device_error() == 0


def test_gemm_w8a8_group_rejects_bad_arguments():
    m, n, d = 16, 1024, 128
    xq = torch.zeros((m, n), dtype=torch.int8, device=dev())
    xs = torch.ones(m, dtype=torch.float32, device=dev())
    w_q = torch.zeros((d, n), dtype=torch.int8, device=dev())
    w_s = torch.ones((d, n // 64), dtype=torch.float32, device=dev())
    y = torch.empty(m * d, dtype=torch.float32, device=dev())
    item = (y, xq, xs, w_q, w_s, n, d)
    with pytest.raises(MliError):
        ops.gemm_w8a8_group([], m)                      # no op
    with pytest.raises(MliError):
        ops.gemm_w8a8_group([item] * 9, m)              # more than MLI_GEMM_GROUP_MAX
    with pytest.raises(MliError):
        ops.gemm_w8a8_group([item], 8)                  # fewer than 16 tokens
    with pytest.raises(MliError):
        ops.gemm_w8a8_group([(y, xq, xs, w_q, w_s, 1000, d)], m)  # n % 128 != 0
    assert ops.device_error() == 0


def test_rows_are_independent_of_sharding():
    """Row r's result is bit-identical whether computed in the full matrix or
    in any row slice (the property the sharded classifier relies on)."""
    d, n = 4096, 2048
    w_q, w_s, x = make_case(d, n, 41)
    tw, ts, tx = up(w_q), up(w_s), up(x)
    full = torch.empty(d, dtype=torch.float32, device=dev())
    ops.matmul_int8(full, tx, tw, ts, n, d, 64)
    xq = torch.empty(n, dtype=torch.int8, device=dev())
    xs = torch.empty(1, dtype=torch.float32, device=dev())
    full8 = torch.empty(d, dtype=torch.float32, device=dev())
    ops.matmul_dp4a_fused(full8, tx, tw, ts, n, d, 64, xq_out=xq, xs_out=xs)
    for world in (2, 4, 8):
        chunk = d // world
        part = torch.empty(d, dtype=torch.float32, device=dev())
        part8 = torch.empty(d, dtype=torch.float32, device=dev())
        for r in range(world):
            ops.matmul_int8(part[r * chunk:(r + 1) * chunk], tx, tw[r * chunk:(r + 1) * chunk],
                            ts[r * chunk:(r + 1) * chunk], n, chunk, 64)
            ops.matmul_dp4a_fused(part8[r * chunk:(r + 1) * chunk], tx, tw[r * chunk:(r + 1) * chunk],
                                  ts[r * chunk:(r + 1) * chunk], n, chunk, 64)
        torch.cuda.synchronize()
        assert torch.equal(part.view(torch.int32), full.view(torch.int32))
        assert torch.equal(part8.view(torch.int32), full8.view(torch.int32))


def test_deterministic_and_stream_pdl_independent():
    d, n = 2048, 8192
    w_q, w_s, x = make_case(d, n, 43)
    tw, ts, tx = up(w_q), up(w_s), up(x)
    outs = []
    s = torch.cuda.Stream()
    for pdl in (True, False):
        ops.set_pdl(pdl)
        for stream in (None, s):
            y = torch.empty(d, dtype=torch.float32, device=dev())
            with torch.cuda.stream(s if stream is not None else torch.cuda.current_stream()):
                ops.matmul_int8(y, tx, tw, ts, n, d, 64)
            torch.cuda.synchronize()
            outs.append(y.view(torch.int32).clone())
    ops.set_pdl(True)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_dependent_chain_under_pdl(form):
    """A chain where every GEMV consumes the previous one's output, launched
    back to back on a side stream with programmatic dependent launch and
    captured into a CUDA graph, equals the same chain run without PDL, and its
    first link equals the oracle."""
    dims = [2048, 8192, 2048, 512, 2048, 2048, 8192, 2048]
    mats = []
    for i in range(len(dims) - 1):
        n, d = dims[i], dims[i + 1]
        w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, 500 + i, std=0.05))
        mats.append((n, d, up(w_q), up(w_s), w_q, w_s))
    x0 = synth.activation_np(dims[0], 9)
    s = torch.cuda.Stream()

    def run(pdl, graph):
        ops.set_pdl(pdl)
        bufs = [up(x0)] + [torch.empty(d, dtype=torch.float32, device=dev()) for d in dims[1:]]

        def issue():
            for i, (n, d, tw, ts, _, _) in enumerate(mats):
                if form == "w8a32":
                    ops.matmul_int8(bufs[i + 1], bufs[i], tw, ts, n, d, 64)
                else:
                    ops.matmul_dp4a_fused(bufs[i + 1], bufs[i], tw, ts, n, d, 64)

        with torch.cuda.stream(s):
            if graph:
                issue()  # warm-up
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    issue()
                for b in bufs[1:]:
                    b.fill_(float("nan"))
                g.replay()
            else:
                issue()
        torch.cuda.synchronize()
        ops.set_pdl(True)
        return [b.cpu().numpy() for b in bufs]

    ref = run(False, False)
    for graph in (False, True):
        got = run(True, graph)
        for a, b in zip(got[1:], ref[1:]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    n, d, _, _, w_q, w_s = mats[0]
    if form == "w8a32":
        assert orc.max_abs_rel(ref[1], orc.gemv_w8a32(x0, w_q, w_s)) <= TOL_W8A32
    else:
        xq, xs = orc.quantize_activation(x0)
        assert orc.max_abs_rel(ref[1], orc.gemv_w8a8_f64(xq, xs, w_q, w_s)) <= TOL_W8A8


def test_dropin_shim_matches_c_abi():
    from minillama_infra_b200._lib import DROPIN_SYMBOLS, dropin
    d, n = 512, 2048
    w_q, w_s, x = make_case(d, n, 47, outliers=True)
    tw, ts, tx = up(w_q), up(w_s), up(x)
    sh = dropin()
    y_shim = torch.empty(d, dtype=torch.float32, device=dev())
    y_abi = torch.empty(d, dtype=torch.float32, device=dev())
    getattr(sh, DROPIN_SYMBOLS["matmul_int8"])(y_shim.data_ptr(), tx.data_ptr(), tw.data_ptr(),
                                               ts.data_ptr(), n, d, 64)
    ops.matmul_int8(y_abi, tx, tw, ts, n, d, 64)
    xq = torch.empty(n, dtype=torch.int8, device=dev())
    xs = torch.empty(1, dtype=torch.float32, device=dev())
    getattr(sh, DROPIN_SYMBOLS["quantize_activation"])(xq.data_ptr(), xs.data_ptr(), tx.data_ptr(), n)
    y8_shim = torch.empty(d, dtype=torch.float32, device=dev())
    getattr(sh, DROPIN_SYMBOLS["matmul_dp4a"])(y8_shim.data_ptr(), xq.data_ptr(), xs.data_ptr(),
                                               tw.data_ptr(), ts.data_ptr(), n, d, 64)
    torch.cuda.synchronize()
    assert lib().mli_last_status() == 0
    assert torch.equal(y_shim.view(torch.int32), y_abi.view(torch.int32))
    xq_ref, xs_ref = orc.quantize_activation(x)
    assert np.array_equal(xq.cpu().numpy(), xq_ref)
    assert orc.max_abs_rel(y8_shim.cpu().numpy(), orc.gemv_w8a8_f64(xq_ref, xs_ref, w_q, w_s)) <= TOL_W8A8


def test_reference_kernels_match_oracle_bit_exact():
    """Pins the oracle: the reference's own kernels (rebuilt for sm_100a) give
    exactly the oracle's bits on the same inputs."""
    if not orc.ref_available():
        pytest.skip("oracle/_ref not built")
    ref = orc.ref()
    for d, n in [(256, 2048), (64, 8192), (48, 3072)]:
        w_q, w_s, x = make_case(d, n, d + n, outliers=True)
        tw, ts, tx = up(w_q), up(w_s), up(x)
        y = torch.empty(d, dtype=torch.float32, device=dev())
        y8 = torch.empty(d, dtype=torch.float32, device=dev())
        xq = torch.empty(n, dtype=torch.int8, device=dev())
        xs = torch.empty(1, dtype=torch.float32, device=dev())
        torch.cuda.synchronize()
        ref.ref_matmul_int8(y.data_ptr(), tx.data_ptr(), tw.data_ptr(), ts.data_ptr(), n, d, 64)
        ref.ref_quantize_activation(xq.data_ptr(), xs.data_ptr(), tx.data_ptr(), n)
        ref.ref_matmul_dp4a(y8.data_ptr(), xq.data_ptr(), xs.data_ptr(), tw.data_ptr(), ts.data_ptr(), n, d, 64)
        assert ref.ref_device_synchronize() == 0
        assert np.array_equal(y.cpu().numpy().view(np.uint32), orc.gemv_w8a32(x, w_q, w_s).view(np.uint32))
        xq_ref, xs_ref = orc.quantize_activation(x)
        assert np.array_equal(xq.cpu().numpy(), xq_ref)
        assert np.array_equal(y8.cpu().numpy().view(np.uint32),
                              orc.gemv_w8a8(xq_ref, xs_ref, w_q, w_s).view(np.uint32))


def test_invalid_arguments_raise():
    y = torch.empty(8, dtype=torch.float32, device=dev())
    with pytest.raises(MliError):
        ops.matmul_int8(y, 0, 0, 0, 64, 8, 64)
    with pytest.raises(MliError):
        ops.matmul_int8(y, y, y, y, 0, 8, 64)
    with pytest.raises(MliError):
        ops.quantize_activation(y, y, y, -1)


def test_no_device_errors_recorded():
    assert ops.device_error() == 0


# fp32 GEMV (the reference's `matmul`, the classifier's launcher): the
# classifier shape, config shapes, the generic path (n % 4 != 0, misaligned).
@pytest.mark.parametrize("d,n,offset", [(128256, 2048, 0), (2048, 2048, 0), (300, 8192, 0), (37, 100, 0),
                                        (64, 2048, 1), (5, 12288, 0), (3, 12800, 0)])
def test_f32_gemv_parity(d, n, offset):
    w = synth.weights_np(d, n, d + n)
    x = synth.activation_np(n, d + n + 1)
    wb = torch.zeros(d * n + offset, dtype=torch.float32, device=dev())
    wb[offset:] = up(w.reshape(-1))
    xb = torch.zeros(n + offset, dtype=torch.float32, device=dev())
    xb[offset:] = up(x)
    y = Guarded(d)
    ops.matmul(y.t, xb.data_ptr() + 4 * offset, wb.data_ptr() + 4 * offset, n, d)
    torch.cuda.synchronize()
    got = y.check()
    assert orc.max_abs_rel(got, orc.matmul_f32(x, w)) <= TOL_W8A32
    assert orc.max_abs_rel(got, orc.matmul_f64(x, w)) <= TOL_W8A32


def test_f32_gemv_through_dropin_shim():
    import ctypes

    from minillama_infra_b200._lib import DROPIN_SYMBOLS, dropin
    d, n = 1000, 2048
    w = synth.weights_np(d, n, 3)
    x = synth.activation_np(n, 4)
    tw, tx = up(w), up(x)
    y = Guarded(d)
    getattr(dropin(), DROPIN_SYMBOLS["matmul"])(ctypes.c_void_p(y.t.data_ptr()), ctypes.c_void_p(tx.data_ptr()),
                                               ctypes.c_void_p(tw.data_ptr()), n, d)
    torch.cuda.synchronize()
    assert lib().mli_last_status() == 0
    assert orc.max_abs_rel(y.check(), orc.matmul_f32(x, w)) <= TOL_W8A32
