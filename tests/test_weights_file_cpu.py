"""The int8 classifier section of the quantised weight file (CPU): the
quantiser matches the oracle (itself pinned to the reference script) bit for
bit, the reference's own sections are left byte-identical, and malformed or
repeated appends are refused."""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import weights_file as wf

CFG = wf.ModelConfig(dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=300, seq_len=64)


def write_reference_file(path, cfg=CFG, seed=0):
    """A file laid out exactly as the reference's group-64 exporter writes it."""
    rng = np.random.default_rng(seed)
    wcls = (rng.standard_normal((cfg.vocab_size, cfg.dim), dtype=np.float32) * np.float32(0.02))
    wcls[3, 64:128] = 0.0                 # a zero group (scale guard)
    wcls[7, :64] = np.float32(0.5)        # a constant group: every value is the max
    wcls[9, 0] = np.float32(-1.0)         # a row whose max is negative-signed
    with open(path, "wb") as f:
        f.write(wf.HEADER.pack(cfg.dim, cfg.hidden_dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads,
                               cfg.vocab_size, cfg.seq_len))
        for name, size in wf.reference_sections(cfg):
            if name == "wcls":
                f.write(wcls.tobytes())
            else:
                f.write(rng.integers(0, 256, size, dtype=np.uint8).tobytes())
    return wcls


def test_quantize_rows_matches_oracle():
    rng = np.random.default_rng(1)
    w = rng.standard_normal((37, 256), dtype=np.float32) * np.float32(0.05)
    w[0, :64] = 0
    w[1, 64:128] = np.float32(0.25)
    q, s = wf.quantize_rows(w)
    q_ref, s_ref = orc.quantize_weights(w)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(s.view(np.uint32), s_ref.view(np.uint32))


def test_append_and_read_back(tmp_path):
    path = str(tmp_path / "model_q8_group.bin")
    wcls = write_reference_file(path)
    before = open(path, "rb").read()
    wf.append_int8_classifier(path, chunk_rows=128)  # several chunks
    after = open(path, "rb").read()
    assert after[:len(before)] == before  # the reference's sections are untouched
    w_q, w_s = wf.read_int8_classifier(path)
    q_ref, s_ref = orc.quantize_weights(wcls)
    assert w_q.shape == (CFG.vocab_size, CFG.dim) and w_s.shape == (CFG.vocab_size, CFG.dim // 64)
    assert np.array_equal(np.asarray(w_q), q_ref)
    assert np.array_equal(np.asarray(w_s).view(np.uint32), s_ref.view(np.uint32))
    assert wf.read_config(path) == CFG
    # the reference loader's walk (src/main_cuda.cpp:358-393) still lands on the same offsets
    assert wf.section_offset(CFG, "rms_final_weight") + CFG.dim * 4 == wf.section_offset(CFG, "wcls")
    del w_q, w_s


def test_refuses_a_second_append_and_foreign_files(tmp_path):
    path = str(tmp_path / "m.bin")
    write_reference_file(path)
    wf.append_int8_classifier(path)
    with pytest.raises(ValueError):
        wf.append_int8_classifier(path)
    bare = str(tmp_path / "bare.bin")
    write_reference_file(bare)
    with pytest.raises(ValueError):
        wf.read_int8_classifier(bare)
    # a truncated file is not a reference file
    with open(bare, "rb+") as f:
        f.truncate(os.path.getsize(bare) - 4)
    with pytest.raises(ValueError):
        wf.append_int8_classifier(bare)
