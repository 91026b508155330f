"""The allocation-free batched W8A8 entry point (mli_gemm_w8a8_noalloc).

It exists for callers that cannot allocate device memory for a workspace:
a plugin whose host framework owns every byte of device memory through its
own pool, or a serving loop that must not allocate on the request path.  Its
split-K scratch is therefore a fixed array inside the library instead of a
caller's buffer.

The tests call it through the C ABI twice in a row and check both results
against mli_gemm_w8a8 given a workspace of its own, within the W8A8 tolerance
of the other parity tests.  The first case switches thread-block clusters off
and asserts, through the library's own plan, that the K splits are summed in
the scratch array; its second call uses other activations, so it reads an
array that still holds the first call's partial sums.  The other cases keep
the default plan (most shapes sum their splits inside clusters and never
touch the array).  This file is collected last so that a run stopping at the
first failure has run every other test first; it does not depend on them.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200._lib import MLI_OK, lib

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
TOL_W8A8 = 1e-6
SCRATCH_BYTES = 12 << 20


def _plan(m, n, d, ws_bytes):
    out = (ctypes.c_int * 5)()
    assert lib().mli_debug_plan_gemm(m, n, d, ws_bytes, out) == MLI_OK
    return list(out)


def _run_case(m, n, d, seeds):
    dev = torch.device("cuda:0")
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, m + d))
    tw, ts = torch.from_numpy(w_q).to(dev), torch.from_numpy(w_s).to(dev)
    ws = torch.zeros(max(256, ops.gemm_workspace_bytes(m, n, d)), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate(seeds):
        x = synth.activation_np(n, seed, m=m, outliers=True)
        xq_np, xs_np = orc.quantize_activation(x)
        xq, xs = torch.from_numpy(xq_np).to(dev), torch.from_numpy(xs_np).to(dev)
        y_ref = torch.empty((m, d), dtype=torch.float32, device=dev)
        ops.gemm_w8a8(y_ref, xq, xs, tw, ts, m, n, d, 64, workspace=ws)
        y = torch.full((m, d), float("nan"), dtype=torch.float32, device=dev)
        rc = lib().mli_gemm_w8a8_noalloc(y.data_ptr(), xq.data_ptr(), xs.data_ptr(), tw.data_ptr(),
                                         ts.data_ptr(), m, n, d, 64, stream)
        assert rc == MLI_OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        got, ref = y.cpu().numpy(), y_ref.cpu().numpy()
        assert not np.isnan(got).any(), f"call {call}: outputs not written"
        for t in range(m):
            assert orc.max_abs_rel(got[t], ref[t]) <= TOL_W8A8, (call, t)
        for t in (0, m - 1):
            exact = orc.gemv_w8a8_f64(xq_np[t], xs_np[t:t + 1], w_q, w_s)
            assert orc.max_abs_rel(got[t], exact) <= TOL_W8A8, (call, t)
    assert ops.device_error() == 0


@pytest.mark.parametrize("m,n,d", [(64, 8192, 3072), (16, 3072, 1024)])
def test_noalloc_scratch_array_path(m, n, d):
    """Clusters off: the splits are summed through the library's array."""
    ops.set_gemm_clusters(False)
    try:
        plan = _plan(m, n, d, SCRATCH_BYTES)
        assert plan[2] > 1 and plan[3] == 1 and plan[4] == 1, f"plan {plan} does not use the scratch array"
        _run_case(m, n, d, seeds=(m + 1, m + 2))
    finally:
        ops.set_gemm_clusters(True)


@pytest.mark.parametrize("m,n,d", [(256, 3072, 3072), (33, 1024, 300)])
def test_noalloc_default_plan(m, n, d):
    _run_case(m, n, d, seeds=(m + 1, m + 2))


def test_noalloc_rejects_shapes_without_scratch_path():
    dev = torch.device("cuda:0")
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    p = buf.data_ptr()
    # m < 16 is not a tensor-core shape; n % 128 != 0 neither
    assert lib().mli_gemm_w8a8_noalloc(p, p, p, p, p, 8, 1024, 128, 64, None) == 2
    assert lib().mli_last_status() == 2
    assert lib().mli_gemm_w8a8_noalloc(p, p, p, p, p, 32, 1088, 128, 64, None) == 2
    assert lib().mli_gemm_w8a8_noalloc(None, p, p, p, p, 32, 1024, 128, 64, None) == 1
