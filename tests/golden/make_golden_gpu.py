"""Generate tests/golden/ref_kernels_*.npz: outputs of the reference's own CUDA
kernels (src/model_cuda_v2_shared.cu: matmul_int8, quantize_activation,
matmul_dp4a), compiled unmodified for sm_100a into oracle/_ref/libmli_ref.so,
on small seeded inputs.  Needs a GPU; writes into the directory given as the
first argument (default: tests/golden next to this file).

    python tests/golden/make_golden_gpu.py [out_dir]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402
from minillama_infra_b200 import synth  # noqa: E402

# name: (d rows, n cols, activation kind)
CASES = {
    "2048": (32, 2048, "normal"),
    "8192": (8, 8192, "normal"),
    "3072_outliers": (16, 3072, "outliers"),
    "256": (8, 256, "normal"),
    "64_zero_x": (4, 64, "zero"),
}


def run_case(name, d, n, kind, out_dir):
    import torch

    ref = orc.ref()
    seed = sum(map(ord, name))
    w = synth.weights_np(d, n, seed)
    w_q, w_s = orc.quantize_weights(w)
    if kind == "zero":
        x = np.zeros(n, np.float32)
    else:
        x = synth.activation_np(n, seed + 1, outliers=(kind == "outliers"))
    dev = torch.device("cuda:0")
    tw = torch.from_numpy(w_q).to(dev)
    ts = torch.from_numpy(w_s).to(dev)
    tx = torch.from_numpy(x).to(dev)
    y = torch.empty(d, dtype=torch.float32, device=dev)
    y8 = torch.empty(d, dtype=torch.float32, device=dev)
    xq = torch.empty(n, dtype=torch.int8, device=dev)
    xs = torch.empty(1, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    ref.ref_matmul_int8(y.data_ptr(), tx.data_ptr(), tw.data_ptr(), ts.data_ptr(), n, d, 64)
    ref.ref_quantize_activation(xq.data_ptr(), xs.data_ptr(), tx.data_ptr(), n)
    ref.ref_matmul_dp4a(y8.data_ptr(), xq.data_ptr(), xs.data_ptr(), tw.data_ptr(), ts.data_ptr(), n, d, 64)
    assert ref.ref_device_synchronize() == 0
    assert ref.ref_last_error() == 0
    np.savez_compressed(
        os.path.join(out_dir, f"ref_kernels_{name}.npz"),
        w_q=w_q, w_s=w_s, x=x, group_size=np.int32(64),
        y_w8a32=y.cpu().numpy(), xq=xq.cpu().numpy(), xs=xs.cpu().numpy(), y_w8a8=y8.cpu().numpy())


def main():
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(out_dir, exist_ok=True)
    for name, (d, n, kind) in CASES.items():
        run_case(name, d, n, kind, out_dir)
        print("wrote", name)


if __name__ == "__main__":
    main()
