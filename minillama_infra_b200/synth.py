"""Seeded synthetic workloads with the shapes and value distributions of the
Llama-3.2 decode GEMVs (no real checkpoints are available offline).

Weights are fp32 N(0, 0.02), quantised per row per 64-column group with the
reference scheme (scripts/quantize_int8_group.py:55-71); activations are fp32
N(0, 1); the W8A8 workload scales 1% of the channels by 20 to mimic outliers.
"""
from __future__ import annotations

import numpy as np

GROUP = 64

# (name, rows d, cols n) of the seven per-layer projections.
LLAMA_1B = [
    ("wq", 2048, 2048), ("wk", 512, 2048), ("wv", 512, 2048), ("wo", 2048, 2048),
    ("w_gate", 8192, 2048), ("w_up", 8192, 2048), ("w_down", 2048, 8192),
]
LLAMA_1B_LAYERS = 16
LLAMA_3B = [
    ("wq", 3072, 3072), ("wk", 1024, 3072), ("wv", 1024, 3072), ("wo", 3072, 3072),
    ("w_gate", 8192, 3072), ("w_up", 8192, 3072), ("w_down", 3072, 8192),
]
CLASSIFIER_1B = ("wcls", 128256, 2048)


def gemv_bytes(d: int, n: int, m: int = 1, group: int = GROUP) -> int:
    """Algorithmic bytes of one call: int8 weights + fp32 scales + fp32 x + fp32 y."""
    return d * n + d * (n // group) * 4 + m * n * 4 + m * d * 4


def gemv_ops(d: int, n: int, m: int = 1) -> int:
    return 2 * m * d * n


# --------------------------------------------------------------------------
# CPU (numpy) generators for parity-test sizes
# --------------------------------------------------------------------------
def weights_np(rows: int, cols: int, seed: int, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)).astype(np.float32)


def activation_np(n: int, seed: int, m: int | None = None, outliers: bool = False) -> np.ndarray:
    rng = np.random.default_rng(seed)
    shape = (n,) if m is None else (m, n)
    x = rng.standard_normal(shape, dtype=np.float32)
    if outliers:
        idx = outlier_channels(n, seed)
        x[..., idx] *= np.float32(20.0)
    return x


def outlier_channels(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed ^ 0x5EED)
    return np.sort(rng.choice(n, size=max(1, n // 100), replace=False))


# --------------------------------------------------------------------------
# GPU (torch) generators for full-size workloads
# --------------------------------------------------------------------------
def weights_gpu(rows: int, cols: int, seed: int, device, std: float = 0.02):
    """(int8 [rows][cols], fp32 [rows][cols/64]) quantised on the GPU with
    mli_quantize_weights (bit-identical to the reference quantiser)."""
    import torch

    from . import ops

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.empty((rows, cols), dtype=torch.int8, device=device)
    s = torch.empty((rows, cols // GROUP), dtype=torch.float32, device=device)
    # generate in row blocks to bound the fp32 staging buffer
    block = max(1, (64 << 20) // (cols * 4))
    for r0 in range(0, rows, block):
        r1 = min(rows, r0 + block)
        w = torch.randn((r1 - r0, cols), generator=g, device=device, dtype=torch.float32) * std
        ops.quantize_weights(q[r0:r1], s[r0:r1], w, r1 - r0, cols, GROUP)
    return q, s


def quantize_torch(w, group: int = GROUP):
    """The reference weight quantiser (scripts/quantize_int8_group.py:55-64) in
    plain torch ops, on whatever device `w` lives: amax per (row, group), zero
    amax -> float32(1e-9), scale = amax / 127 (fp32), q = clip(round-half-even(
    w / scale), +-127).  IEEE fp32 division and torch.round (ties to even) make
    it bit-identical to the script and to mli_quantize_weights; the bench
    builds its workloads with it so that the reference arm never loads this
    repository's library."""
    import torch

    rows, cols = w.shape
    g = w.reshape(rows, cols // group, group)
    amax = g.abs().amax(dim=-1)
    amax = torch.where(amax == 0, torch.full_like(amax, 1e-9), amax)
    scale = amax / 127.0
    q = torch.round(g / scale.unsqueeze(-1)).clamp_(-127.0, 127.0).to(torch.int8)
    return q.reshape(rows, cols), scale


def weights_torch(rows: int, cols: int, seed: int, device, std: float = 0.02):
    """The same (int8, fp32 scales) as weights_gpu, from the same seeded
    normal draws, quantised with quantize_torch (no library call)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.empty((rows, cols), dtype=torch.int8, device=device)
    s = torch.empty((rows, cols // GROUP), dtype=torch.float32, device=device)
    block = max(1, (64 << 20) // (cols * 4))
    for r0 in range(0, rows, block):
        r1 = min(rows, r0 + block)
        w = torch.randn((r1 - r0, cols), generator=g, device=device, dtype=torch.float32) * std
        q[r0:r1], s[r0:r1] = quantize_torch(w)
    return q, s


def activation_gpu(n: int, seed: int, device, m: int | None = None, outliers: bool = False):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shape = (n,) if m is None else (m, n)
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if outliers:
        idx = torch.from_numpy(outlier_channels(n, seed)).to(device)
        x[..., idx] *= 20.0
    return x
