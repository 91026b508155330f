"""Generate tests/golden/quant_ref_script.npz by running the reference's own
weight quantiser, scripts/quantize_int8_group.py, unmodified.

The script reads ``llama3_2_1B.bin`` from its working directory (:7, :11-13,
:31) and writes ``llama3_2_1B_q8_group.bin`` there (:36, :41-74).  This
generator writes a small synthetic fp32 weight file in that format (28-byte
header of 7 int32, then every tensor in export order, scripts/export.py:30-53)
into a temporary directory, runs the script there, and stores the fp32 inputs
of the seven quantised tensors together with the script's scales and int8
output.  The inputs include groups that are all zero (the 1e-9 guard of :59),
exact rounding ties (w / scale = k + 0.5, half-to-even at :63) and values at
+-amax (the clip of :64).

Run it where the reference tree exists (the path is required):
    python tests/golden/make_golden_quant.py /path/to/reference
"""
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "quant_ref_script.npz")

# dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len
CONFIG = (64, 128, 1, 4, 2, 16, 8)
GS = 64


def tensor_specs(cfg):
    dim, hidden, L, nh, nkv, vocab, _ = cfg
    kv = dim * nkv // nh
    # (name, element count, cols) in the script's `sizes` order (:17-25)
    return [
        ("token_embedding_table", vocab * dim, None),
        ("rms_att_weight", L * dim, None),
        ("wq", L * dim * dim, dim), ("wk", L * dim * kv, dim), ("wv", L * dim * kv, dim),
        ("wo", L * dim * dim, dim),
        ("rms_ffn_weight", L * dim, None),
        ("w1", L * dim * hidden, dim), ("w2", L * hidden * dim, hidden), ("w3", L * dim * hidden, dim),
        ("rms_final_weight", dim, None),
        ("wcls", vocab * dim, None),
    ]


def special_groups(w: np.ndarray, cols: int, rng) -> None:
    """Plant edge cases into a [rows][cols] view, group-aligned."""
    rows = w.shape[0]
    ng = cols // GS
    # 1) an all-zero group
    w[0, 0:GS] = 0.0
    # 2) a group with amax 127 -> scale exactly 1.0 and half-integer ties
    g = 1 % ng
    r = 1 % rows
    vals = np.array([127.0, -127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5], np.float32)
    w[r, g * GS:(g + 1) * GS] = 0.25
    w[r, g * GS:g * GS + vals.size] = vals
    # 3) a group with a single tiny non-zero value (subnormal scale)
    r = 2 % rows
    w[r, 0:GS] = 0.0
    w[r, 5] = np.float32(1e-38)
    # 4) a group where every value equals +-amax
    r = 3 % rows
    w[r, (ng - 1) * GS:ng * GS] = np.where(rng.random(GS) < 0.5, 0.03, -0.03).astype(np.float32)


def main(ref_root: str) -> None:
    script = os.path.join(ref_root, "scripts", "quantize_int8_group.py")
    rng = np.random.default_rng(20261201)
    specs = tensor_specs(CONFIG)
    tensors = {}
    for name, size, cols in specs:
        t = (rng.standard_normal(size, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        if cols is not None:
            special_groups(t.reshape(-1, cols), cols, rng)
        tensors[name] = t
    with tempfile.TemporaryDirectory() as tmp:
        with open(os.path.join(tmp, "llama3_2_1B.bin"), "wb") as f:
            f.write(struct.pack("7i", *CONFIG))
            for name, _, _ in specs:
                f.write(tensors[name].tobytes())
        subprocess.run([sys.executable, script], cwd=tmp, check=True, stdout=subprocess.DEVNULL)
        raw = open(os.path.join(tmp, "llama3_2_1B_q8_group.bin"), "rb").read()
    assert raw[:28] == struct.pack("7i", *CONFIG)
    off = 28
    out = {"config": np.array(CONFIG, np.int32)}
    for name, size, cols in specs:
        if cols is None:
            off += size * 4
            continue
        rows = size // cols
        ng = cols // GS
        s = np.frombuffer(raw, np.float32, rows * ng, off).reshape(rows, ng)
        off += rows * ng * 4
        q = np.frombuffer(raw, np.int8, size, off).reshape(rows, cols)
        off += size
        out[f"{name}_w"] = tensors[name].reshape(rows, cols)
        out[f"{name}_s"] = s.copy()
        out[f"{name}_q"] = q.copy()
    assert off == len(raw)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {sorted(k for k in out if k.endswith('_q'))}")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MLI_REF_ROOT")
    if not root:
        sys.exit("usage: make_golden_quant.py <reference tree> (or set MLI_REF_ROOT)")
    main(root)
