"""INT8 group-64 classifier section for MiniLlama-Infra's quantised weight file.

The reference's exporter (scripts/quantize_int8_group.py:41-74) writes, after the
28-byte config (7 int32: dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size,
seq_len), the fp32 token embedding, the layers' norms and int8 group-64 matrices (each
as fp32 scales then int8 rows), the final norm and, last, the fp32 classifier `wcls`
(vocab_size x dim, written but never read: src/main_cuda.cpp:393 ties wcls to the
embedding).  The classifier GEMV is the largest per-token read of a decode step, so this
module quantises it with the same group-64 scheme and appends it as a self-describing
section after everything the reference writes.  The reference's loader reads the file
front to back up to the final norm and ignores the rest, so it keeps working unchanged;
a loader that knows the section finds it from the end of the file:

    ... reference content ...
    fp32  scales [rows][cols / group]          (rows = vocab_size, cols = dim)
    int8  w_q    [rows][cols]
    trailer, 32 bytes: b"MLIQ8CLS", int32 version (1), int32 rows, int32 cols,
                       int32 group, int64 byte offset of the scales

The quantiser is the reference's (scripts/quantize_int8_group.py:55-64): per row and
64-column group, scale = max|w| / 127 (a zero group gets 1e-9 / 127), q = round half to
even of w / scale in fp32, clipped to +-127.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"MLIQ8CLS"
VERSION = 1
TRAILER = struct.Struct("<8siiiiq")  # magic, version, rows, cols, group, scales offset
GROUP = 64
HEADER = struct.Struct("<7i")


@dataclass(frozen=True)
class ModelConfig:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int

    @property
    def kv_dim(self) -> int:
        return self.dim * self.n_kv_heads // self.n_heads


def read_config(path: str) -> ModelConfig:
    with open(path, "rb") as f:
        return ModelConfig(*HEADER.unpack(f.read(HEADER.size)))


def reference_sections(c: ModelConfig, group: int = GROUP):
    """(name, bytes) of every section the reference's group-64 exporter writes
    after the config, in order (scripts/quantize_int8_group.py:14-26, 41-74)."""
    L, d, h, kv = c.n_layers, c.dim, c.hidden_dim, c.kv_dim

    def q(elems):  # fp32 scales, then int8
        return elems // group * 4 + elems

    return [
        ("token_embedding_table", c.vocab_size * d * 4), ("rms_att_weight", L * d * 4),
        ("wq", q(L * d * d)), ("wk", q(L * d * kv)), ("wv", q(L * d * kv)), ("wo", q(L * d * d)),
        ("rms_ffn_weight", L * d * 4),
        ("w1", q(L * d * h)), ("w2", q(L * h * d)), ("w3", q(L * d * h)),
        ("rms_final_weight", d * 4), ("wcls", c.vocab_size * d * 4),
    ]


def section_offset(c: ModelConfig, name: str, group: int = GROUP) -> int:
    off = HEADER.size
    for n, size in reference_sections(c, group):
        if n == name:
            return off
        off += size
    raise KeyError(name)


def quantize_rows(w: np.ndarray, group: int = GROUP):
    """The reference's group-wise quantiser: (int8 [rows][cols], fp32 [rows][cols/group])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % group:
        raise ValueError(f"cols {cols} is not a multiple of the group size {group}")
    m = w.reshape(rows, cols // group, group)
    amax = np.max(np.abs(m), axis=2, keepdims=True)
    amax[amax == 0] = np.float32(1e-9)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.round(m / scale), -127, 127).astype(np.int8)
    return q.reshape(rows, cols), scale.reshape(rows, cols // group)


def append_int8_classifier(path: str, chunk_rows: int = 8192) -> None:
    """Quantises the file's fp32 classifier (its last reference section) and
    appends the int8 section and trailer.  The file must be exactly the
    reference exporter's output (no section appended yet)."""
    c = read_config(path)
    expected = HEADER.size + sum(size for _, size in reference_sections(c))
    if os.path.getsize(path) != expected:
        raise ValueError(f"{path}: {os.path.getsize(path)} bytes, expected {expected} "
                         "(not a reference group-64 file, or a section is already appended)")
    rows, cols = c.vocab_size, c.dim
    src = np.memmap(path, dtype=np.float32, mode="r", offset=section_offset(c, "wcls"), shape=(rows, cols))
    q_all = np.empty((rows, cols), np.int8)
    s_all = np.empty((rows, cols // GROUP), np.float32)
    for r0 in range(0, rows, chunk_rows):
        q_all[r0:r0 + chunk_rows], s_all[r0:r0 + chunk_rows] = quantize_rows(src[r0:r0 + chunk_rows])
    del src
    with open(path, "ab") as f:
        scales_off = f.tell()
        f.write(s_all.tobytes())
        f.write(q_all.tobytes())
        f.write(TRAILER.pack(MAGIC, VERSION, rows, cols, GROUP, scales_off))


def read_int8_classifier(path: str):
    """(w_q int8 [rows][cols], w_s fp32 [rows][cols/group]) memory-mapped from
    the appended section; raises if the file has none."""
    size = os.path.getsize(path)
    if size < TRAILER.size:
        raise ValueError(f"{path}: too small")
    with open(path, "rb") as f:
        f.seek(size - TRAILER.size)
        magic, version, rows, cols, group, off = TRAILER.unpack(f.read(TRAILER.size))
    if magic != MAGIC or version != VERSION:
        raise ValueError(f"{path}: no int8 classifier section")
    n_s = rows * (cols // group)
    if off + n_s * 4 + rows * cols + TRAILER.size != size:
        raise ValueError(f"{path}: inconsistent int8 classifier section")
    w_s = np.memmap(path, dtype=np.float32, mode="r", offset=off, shape=(rows, cols // group))
    w_q = np.memmap(path, dtype=np.int8, mode="r", offset=off + n_s * 4, shape=(rows, cols))
    return w_q, w_s


# ---------------------------------------------------------------------------
# synthetic model and tokenizer files (no checkpoint is available offline)
# ---------------------------------------------------------------------------
LLAMA_1B = ModelConfig(dim=2048, hidden_dim=8192, n_layers=16, n_heads=32, n_kv_heads=8,
                       vocab_size=128256, seq_len=131072)


def write_synthetic_model(path: str, c: ModelConfig = LLAMA_1B, seed: int = 0, device="cpu",
                          std: float = 0.02) -> int:
    """Writes a group-64 weight file in the reference exporter's layout
    (scripts/quantize_int8_group.py:41-74; the loader is src/main_cuda.cpp:340-393):
    the 28-byte config, the fp32 token embedding, the norms (all ones), every
    layer's matrices quantised with the reference scheme (fp32 scales of all
    layers, then their int8 rows), the final norm and the fp32 classifier (the
    embedding again: the 1B model ties them).  Weights are N(0, std) from a
    seeded torch generator on `device`.  Returns the file size."""
    import torch

    from .synth import quantize_torch

    L, d, h, kv = c.n_layers, c.dim, c.hidden_dim, c.kv_dim
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def randn(rows, cols):
        return torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32) * std

    ones = np.ones(L * d, np.float32).tobytes()
    with open(path, "wb") as f:
        f.write(HEADER.pack(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size,
                            c.seq_len))
        emb_off = f.tell()
        for r0 in range(0, c.vocab_size, 8192):
            f.write(randn(min(8192, c.vocab_size - r0), d).cpu().numpy().tobytes())
        f.write(ones)  # rms_att_weight
        for name, rows, cols in (("wq", d, d), ("wk", kv, d), ("wv", kv, d), ("wo", d, d), (None, 0, 0),
                                 ("w1", h, d), ("w2", d, h), ("w3", h, d)):
            if name is None:
                f.write(ones)  # rms_ffn_weight
                continue
            qs, ss = [], []
            for _ in range(L):
                q, s = quantize_torch(randn(rows, cols))
                qs.append(q.cpu().numpy())
                ss.append(s.cpu().numpy())
            for s in ss:
                f.write(s.tobytes())
            for q in qs:
                f.write(q.tobytes())
        f.write(np.ones(d, np.float32).tobytes())  # rms_final_weight
        emb_bytes = c.vocab_size * d * 4
        f.flush()
        with open(path, "rb") as src:  # wcls: the embedding again
            src.seek(emb_off)
            for done in range(0, emb_bytes, 1 << 26):
                f.write(src.read(min(1 << 26, emb_bytes - done)))
        size = f.tell()
    expected = HEADER.size + sum(sz for _, sz in reference_sections(c))
    if size != expected:
        raise AssertionError(f"wrote {size} bytes, the layout needs {expected}")
    return size


def write_tokenizer(path: str, vocab_size: int, tokens=None) -> None:
    """A tokenizer.bin in the reference's format (src/tokenizer.cpp:7-16):
    int32 max_len, then per token fp32 score, int32 length, bytes.  Token i is
    the text `<i>` unless `tokens` ({id: text}) names it."""
    import struct as _s

    tokens = tokens or {}
    texts = [tokens.get(i, f"<{i}>").encode() for i in range(vocab_size)]
    with open(path, "wb") as f:
        f.write(_s.pack("<i", max(len(t) for t in texts)))
        for i, t in enumerate(texts):
            f.write(_s.pack("<fi", 0.0, len(t)))
            f.write(t)
