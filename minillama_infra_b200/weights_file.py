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
