"""The end-to-end decode harness, on the CPU: the synthetic weight file and
tokenizer follow the reference's formats, the reference's report is parsed,
and the drop-in build of the reference's decoder binds the forward pass's
GEMV launchers (matmul_int8, matmul_dp4a, quantize_activation and the fp32
classifier's matmul) to libmli_dropin.so (checked from the dynamic linker's
own binding log, at load time, without running anything on a GPU)."""
import os
import struct
import subprocess

import numpy as np
import pytest

from minillama_infra_b200 import weights_file as wf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN_EXE = os.path.join(ROOT, "oracle", "_ref", "minillama_dropin")
SMALL = wf.ModelConfig(dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=300,
                       seq_len=64)


def _sections(path, c):
    raw = np.fromfile(path, np.uint8)
    out, off = {}, wf.HEADER.size
    for name, size in wf.reference_sections(c):
        out[name] = raw[off:off + size]
        off += size
    assert off == raw.size
    return out


def test_synthetic_model_follows_the_reference_layout(tmp_path):
    pytest.importorskip("torch")
    p = str(tmp_path / "m.bin")
    size = wf.write_synthetic_model(p, SMALL, seed=3)
    assert size == os.path.getsize(p)
    assert wf.read_config(p) == SMALL
    sec = _sections(p, SMALL)
    emb = sec["token_embedding_table"].view(np.float32)
    assert np.array_equal(sec["wcls"].view(np.float32), emb)  # tied classifier
    assert np.all(sec["rms_att_weight"].view(np.float32) == 1.0)
    L, d, h, kv = SMALL.n_layers, SMALL.dim, SMALL.hidden_dim, SMALL.kv_dim
    for name, rows, cols in (("wq", d, d), ("wk", kv, d), ("w1", h, d), ("w2", d, h)):
        b = sec[name]
        n_s = L * rows * cols // 64
        s = b[:n_s * 4].view(np.float32).reshape(L, rows, cols // 64)
        q = b[n_s * 4:].view(np.int8).reshape(L, rows, cols // 64, 64)
        # the reference quantiser puts each group's largest |w| at exactly +-127
        assert np.all(np.abs(q.astype(np.int32)).max(axis=-1) == 127), name
        assert np.all(s > 0), name


def test_tokenizer_file_format(tmp_path):
    p = str(tmp_path / "tokenizer.bin")
    wf.write_tokenizer(p, 50, {7: ".", 9: "hello"})
    raw = open(p, "rb").read()
    (max_len,), off, vocab = struct.unpack_from("<i", raw), 4, []
    for _ in range(50):  # src/tokenizer.cpp:7-16
        _score, n = struct.unpack_from("<fi", raw, off)
        off += 8
        vocab.append(raw[off:off + n].decode())
        off += n
    assert off == len(raw)
    assert vocab[7] == "." and vocab[9] == "hello" and vocab[3] == "<3>"
    assert max_len == max(len(v) for v in vocab)


def test_parse_reference_report():
    import bench

    text = "\n".join([
        "Peak VRAM: 2054.12 MB",
        "   -> Throughput:      410.50 tok/s",
        "   -> Throughput:      420.00 tok/s",
        "| Context Len | TTFT (ms) | TPOT (ms/tok) | Throughput (tok/s) |",
        "|          53 |     12.00 |          2.50 |              400.00 |",
        "Stage 6 dp4a Benchmark",
        "  -> Throughput:       500.25 tok/s",
    ])
    p = bench.parse_reference_output(text)
    assert p["w8a32_tok_s"] == [410.5, 420.0] and p["w8a8_tok_s"] == [500.25]
    assert p["context_scaling"][0]["context"] == 53 and p["peak_vram_mb"] == 2054.12


@pytest.mark.skipif(not os.path.exists(DROPIN_EXE), reason="reference decoder not built (oracle/Makefile)")
def test_dropin_decoder_binds_the_shim():
    env = dict(os.environ, LD_BIND_NOW="1", LD_DEBUG="bindings")
    r = subprocess.run([DROPIN_EXE, "/nonexistent"], env=env, capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "Cannot open" in r.stdout  # the reference's own error path
    bound = {}
    for ln in r.stderr.splitlines():
        if "binding file" not in ln or "normal symbol" not in ln:
            continue
        src, dst = ln.split(" to ", 1)
        sym = ln.split("`")[-1].rstrip("'")
        if "libref_model.so" in src:
            bound[sym] = dst.split(" [")[0].rsplit("/", 1)[-1]
    for sym in ("_Z11matmul_int8PfS_PaS_iii", "_Z11matmul_dp4aPfPKaPKfS1_S3_iii", "_Z19quantize_activationPaPfPKfi",
                "_Z6matmulPfS_S_ii"):
        assert bound.get(sym) == "libmli_dropin.so", (sym, bound.get(sym))
    # everything else of the forward pass stays the reference's own
    assert bound.get("_Z12forward_cudaiiP6ConfigP21TransformerWeightsGPUP11RunStateGPU",
                     "libref_model.so") == "libref_model.so"
