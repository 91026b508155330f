"""The allocation-free batched W8A8 entry point (mli_gemm_w8a8_noalloc).

It exists for callers that cannot allocate device memory for a workspace
(their framework's pool owns the device memory, or their serving loop must not
allocate), so its split-K scratch is a fixed array inside the library.  This
test calls it through the C ABI twice in a row -- the second call finds the
first call's leftovers in that shared array -- and checks both results
against mli_gemm_w8a8 given a workspace of its own, within the W8A8
tolerance of the other parity tests.  It lives in a file of its own so that a
run stopping at the first failure has run every other test first; it does not
depend on them having run.
"""
import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200._lib import MLI_OK, lib

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
TOL_W8A8 = 1e-6


@pytest.mark.parametrize("m,n,d", [(16, 3072, 1024), (64, 8192, 3072), (256, 3072, 3072), (33, 1024, 300)])
def test_noalloc_matches_workspace_entry_point(m, n, d):
    dev = torch.device("cuda:0")
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, m + d))
    x = synth.activation_np(n, m + 1, m=m, outliers=True)
    xq_np, xs_np = orc.quantize_activation(x)
    tw, ts = torch.from_numpy(w_q).to(dev), torch.from_numpy(w_s).to(dev)
    xq, xs = torch.from_numpy(xq_np).to(dev), torch.from_numpy(xs_np).to(dev)

    ws = torch.zeros(max(256, ops.gemm_workspace_bytes(m, n, d)), dtype=torch.uint8, device=dev)
    y_ref = torch.empty((m, d), dtype=torch.float32, device=dev)
    ops.gemm_w8a8(y_ref, xq, xs, tw, ts, m, n, d, 64, workspace=ws)
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()

    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        y = torch.full((m, d), float("nan"), dtype=torch.float32, device=dev)
        rc = lib().mli_gemm_w8a8_noalloc(y.data_ptr(), xq.data_ptr(), xs.data_ptr(), tw.data_ptr(),
                                         ts.data_ptr(), m, n, d, 64, stream)
        assert rc == MLI_OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert not np.isnan(got).any(), f"call {call}: outputs not written"
        for t in range(m):
            assert orc.max_abs_rel(got[t], ref[t]) <= TOL_W8A8, (call, t)
        for t in (0, m - 1):
            exact = orc.gemv_w8a8_f64(xq_np[t], xs_np[t:t + 1], w_q, w_s)
            assert orc.max_abs_rel(got[t], exact) <= TOL_W8A8, (call, t)
    assert ops.device_error() == 0


def test_noalloc_rejects_shapes_without_scratch_path():
    dev = torch.device("cuda:0")
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    p = buf.data_ptr()
    # m < 16 is not a tensor-core shape; n % 128 != 0 neither
    assert lib().mli_gemm_w8a8_noalloc(p, p, p, p, p, 8, 1024, 128, 64, None) == 2
    assert lib().mli_gemm_w8a8_noalloc(p, p, p, p, p, 32, 1088, 128, 64, None) == 2
    assert lib().mli_gemm_w8a8_noalloc(None, p, p, p, p, 32, 1024, 128, 64, None) == 1
