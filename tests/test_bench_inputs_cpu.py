"""The bench builds its weights with plain torch ops (synth.quantize_torch), so
that its reference arm never loads this repository's library.  Those ops must
give the reference quantiser's bytes: checked here against the reference
script's own output (tests/golden/quant_ref_script.npz) and the oracle."""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import synth

torch = pytest.importorskip("torch")


def test_torch_quantiser_matches_reference_script(golden_dir):
    z = np.load(os.path.join(golden_dir, "quant_ref_script.npz"))
    for k in ["wq", "wk", "wv", "wo", "w1", "w2", "w3"]:
        q, s = synth.quantize_torch(torch.from_numpy(z[f"{k}_w"]))
        assert np.array_equal(q.numpy(), z[f"{k}_q"]), k
        assert np.array_equal(s.numpy().view(np.uint32), z[f"{k}_s"].view(np.uint32)), k


@pytest.mark.parametrize("rows,cols,seed", [(333, 2048, 8), (64, 8192, 9), (7, 64, 10)])
def test_torch_quantiser_matches_oracle(rows, cols, seed):
    w = synth.weights_np(rows, cols, seed)
    w[0, :64] = 0.0  # a zero group: the 1e-9 guard
    q, s = synth.quantize_torch(torch.from_numpy(w))
    q_ref, s_ref = orc.quantize_weights(w)
    assert np.array_equal(q.numpy(), q_ref)
    assert np.array_equal(s.numpy().view(np.uint32), s_ref.view(np.uint32))
