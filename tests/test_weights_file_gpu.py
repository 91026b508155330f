"""The int8 classifier read from the weight file drives the GPU path: the
W8A32 and fused W8A8 classifier GEMVs over the file's section match the oracle
within the path's tolerances, and the device argmax picks the oracle's row."""
import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200 import weights_file as wf

from test_weights_file_cpu import write_reference_file

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CFG = wf.ModelConfig(dim=512, hidden_dim=1024, n_layers=1, n_heads=8, n_kv_heads=2, vocab_size=6007, seq_len=64)


def test_file_classifier_on_gpu(tmp_path):
    dev = torch.device("cuda:0")
    path = str(tmp_path / "model_q8_group.bin")
    write_reference_file(path, CFG, seed=5)
    wf.append_int8_classifier(path)
    w_q, w_s = wf.read_int8_classifier(path)
    tq = torch.from_numpy(np.array(w_q)).to(dev)  # copies out of the read-only map
    ts = torch.from_numpy(np.array(w_s)).to(dev)
    x = synth.activation_np(CFG.dim, 11)
    tx = torch.from_numpy(x).to(dev)
    d, n = CFG.vocab_size, CFG.dim
    y = torch.empty(d, device=dev)
    ops.matmul_int8(y, tx, tq, ts, n, d, 64)
    y8 = torch.empty(d, device=dev)
    ops.matmul_dp4a_fused(y8, tx, tq, ts, n, d, 64)
    idx = torch.empty((), dtype=torch.int64, device=dev)
    from minillama_infra_b200._lib import check, lib
    check(lib().mli_argmax(y.data_ptr(), d, idx.data_ptr(), None), "argmax")
    torch.cuda.synchronize()
    ref = orc.gemv_w8a32_f64(x, np.asarray(w_q), np.asarray(w_s))
    assert orc.max_abs_rel(y.cpu().numpy(), ref) <= 1e-5
    xq, xs = orc.quantize_activation(x)
    assert orc.max_abs_rel(y8.cpu().numpy(), orc.gemv_w8a8_f64(xq, xs, np.asarray(w_q), np.asarray(w_s))) <= 1e-6
    assert int(idx.item()) == int(np.argmax(y.cpu().numpy()))
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 1e-4 * abs(top2[1]):  # no near tie: the oracle agrees on the row
        assert int(idx.item()) == int(np.argmax(ref))
    assert ops.device_error() == 0
